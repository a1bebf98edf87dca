// prefill.cu -- causal chunked prefill entry points of the C ABI
// (pa_paged_attention_prefill, pa_paged_attention_prefill_wmma,
// pa_prefill_workspace_size).
//
// Semantics (gb10-attn kernels/paged_attn_prefill.cu:55-74): the Sq queries of
// sequence b are the trailing Sq tokens of its context, so query s sits at
// position ctx - Sq + s and attends to keys [0, ctx - Sq + s]; a query with no
// key (ctx - Sq + s < 0) is written as zeros.
//
// Tensor-core path (prefill_tc.cu): fp16 / bf16 pools, head_dim 64 or 128,
// block_size a multiple of 16.  CUDA-core path (every other case, and
// pa_paged_attention_prefill_simt): the split-KV decode kernel with one
// pseudo-sequence per query row (qlen = Sq): row b*Sq + s reads block table
// row b and sees ctx - Sq + s + 1 keys.  The balanced tile scheduler spreads
// the triangular work evenly over the SMs.
#include "decode_host.h"
#include "common.cuh"

namespace pa {
namespace prefill {
bool tc_eligible(int dtype, int64_t D, int64_t BS, int64_t NB);
int launch_tc(float* out, const float* q, const void* k, const void* v, int dtype,
              const int32_t* bt, const int32_t* ctx, int64_t B, int64_t Sq, int64_t H,
              int64_t HKV, int64_t D, int64_t BS, int64_t NB, int64_t MB, double scale,
              int32_t* dev_status, cudaStream_t s);
}  // namespace prefill

static int prefill_checks(int64_t B, int64_t Sq, int64_t H, int64_t HKV, int64_t D) {
  if (B < 0 || Sq < 0 || H <= 0 || HKV <= 0 || D <= 0) return PA_ERR_INVALID_ARGUMENT;
  if (H % HKV != 0) return PA_ERR_NUM_HEADS;           // paged_attn_prefill.cu:148
  if (D % 32 != 0) return PA_ERR_HEAD_DIM;             // paged_attn_prefill.cu:149
  return PA_OK;
}

static decode::DecodeArgs prefill_args(float* out, const float* q, const void* k,
                                       const void* v, int dt, const int32_t* bt,
                                       const int32_t* ctx, int64_t B, int64_t Sq, int64_t H,
                                       int64_t HKV, int64_t D, int64_t BS, int64_t NB,
                                       int64_t MB, double scale, int32_t* dev_status) {
  decode::DecodeArgs a;
  a.out = out;
  a.lse = nullptr;
  a.q = q;
  a.k_cache = k;
  a.v_cache = v;
  a.dtype = dt;
  a.block_tables = bt;
  a.context_lens = ctx;
  a.B = B;
  a.H = H;
  a.HKV = HKV;
  a.D = D;
  a.BS = BS;
  a.NB = NB;
  a.MB = MB;
  a.scale = scale;
  a.num_splits = 0;
  a.dev_status = dev_status;
  a.qlen = Sq;
  a.empty_fill = 0.f;
  return a;
}

}  // namespace pa

extern "C" int pa_prefill_workspace_size(int64_t num_seqs, int64_t num_queries,
                                         int64_t num_heads, int64_t num_kv_heads,
                                         int64_t head_dim, int kv_dtype, int64_t block_size,
                                         int64_t max_blocks, size_t* bytes) {
  if (!bytes) return PA_ERR_INVALID_ARGUMENT;
  int st = pa::prefill_checks(num_seqs, num_queries, num_heads, num_kv_heads, head_dim);
  if (st) return st;
  if (kv_dtype == PA_DTYPE_E4M3) return PA_ERR_DTYPE;  // FP8 pools: decode only
  if (num_seqs == 0 || num_queries == 0) {
    *bytes = 0;
    return PA_OK;
  }
  pa::decode::DecodeArgs a = pa::prefill_args(
      nullptr, nullptr, nullptr, nullptr, kv_dtype, nullptr, nullptr, num_seqs, num_queries,
      num_heads, num_kv_heads, head_dim, block_size, 1, max_blocks, 1.0, nullptr);
  return pa::decode::workspace_bytes(a, bytes);
}

extern "C" int pa_paged_attention_prefill_simt(
    float* out, const float* q, const void* k_cache, const void* v_cache, int kv_dtype,
    const int32_t* block_tables, const int32_t* context_lens, int64_t num_seqs,
    int64_t num_queries, int64_t num_heads, int64_t num_kv_heads, int64_t head_dim,
    int64_t block_size, int64_t num_blocks, int64_t max_blocks, double scale, void* workspace,
    size_t workspace_bytes, int32_t* dev_status, void* stream) {
  int st = pa::prefill_checks(num_seqs, num_queries, num_heads, num_kv_heads, head_dim);
  if (st) return st;
  if (kv_dtype == PA_DTYPE_E4M3) return PA_ERR_DTYPE;  // FP8 pools: decode only
  if (num_seqs == 0 || num_queries == 0) return PA_OK;
  pa::decode::DecodeArgs a = pa::prefill_args(
      out, q, k_cache, v_cache, kv_dtype, block_tables, context_lens, num_seqs, num_queries,
      num_heads, num_kv_heads, head_dim, block_size, num_blocks, max_blocks, scale, dev_status);
  return pa::decode::launch(a, workspace, workspace_bytes, static_cast<cudaStream_t>(stream));
}

extern "C" int pa_paged_attention_prefill(float* out, const float* q, const void* k_cache,
                                          const void* v_cache, int kv_dtype,
                                          const int32_t* block_tables,
                                          const int32_t* context_lens, int64_t num_seqs,
                                          int64_t num_queries, int64_t num_heads,
                                          int64_t num_kv_heads, int64_t head_dim,
                                          int64_t block_size, int64_t num_blocks,
                                          int64_t max_blocks, double scale, void* workspace,
                                          size_t workspace_bytes, int32_t* dev_status,
                                          void* stream) {
  int st = pa::prefill_checks(num_seqs, num_queries, num_heads, num_kv_heads, head_dim);
  if (st) return st;
  if (kv_dtype == PA_DTYPE_E4M3) return PA_ERR_DTYPE;  // FP8 pools: decode only
  if (num_seqs == 0 || num_queries == 0) return PA_OK;
  if (pa::prefill::tc_eligible(kv_dtype, head_dim, block_size, num_blocks))
    return pa::prefill::launch_tc(out, q, k_cache, v_cache, kv_dtype, block_tables, context_lens,
                                  num_seqs, num_queries, num_heads, num_kv_heads, head_dim,
                                  block_size, num_blocks, max_blocks, scale, dev_status,
                                  static_cast<cudaStream_t>(stream));
  return pa_paged_attention_prefill_simt(out, q, k_cache, v_cache, kv_dtype, block_tables,
                                         context_lens, num_seqs, num_queries, num_heads,
                                         num_kv_heads, head_dim, block_size, num_blocks,
                                         max_blocks, scale, workspace, workspace_bytes,
                                         dev_status, stream);
}

extern "C" int pa_paged_attention_prefill_wmma(
    float* out, const float* q, const void* k_cache, const void* v_cache, int kv_dtype,
    const int32_t* block_tables, const int32_t* context_lens, int64_t num_seqs,
    int64_t num_queries, int64_t num_heads, int64_t num_kv_heads, int64_t head_dim,
    int64_t block_size, int64_t num_blocks, int64_t max_blocks, double scale, void* workspace,
    size_t workspace_bytes, int32_t* dev_status, void* stream) {
  // argument checks of paged_attn_wmma.cu:220-225,242-243,264-269
  if (kv_dtype != PA_DTYPE_F16 && kv_dtype != PA_DTYPE_BF16) return PA_ERR_DTYPE;
  if (block_size != 16) return PA_ERR_BLOCK_SIZE;
  if (num_heads <= 0 || num_kv_heads <= 0) return PA_ERR_INVALID_ARGUMENT;
  if (num_heads % num_kv_heads != 0) return PA_ERR_NUM_HEADS;
  if (head_dim % 16 != 0 || (head_dim != 32 && head_dim != 64 && head_dim != 128))
    return PA_ERR_HEAD_DIM;
  return pa_paged_attention_prefill(out, q, k_cache, v_cache, kv_dtype, block_tables,
                                         context_lens, num_seqs, num_queries, num_heads,
                                         num_kv_heads, head_dim, block_size, num_blocks,
                                         max_blocks, scale, workspace, workspace_bytes,
                                         dev_status, stream);
}
