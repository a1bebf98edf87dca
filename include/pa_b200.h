/*
 * pa_b200.h -- C ABI of libpa_b200.so, the B200 (sm_100a) paged-attention
 * library.
 *
 * This is the drop-in boundary.  Every entry point takes plain device
 * pointers, 64-bit sizes and an opaque CUDA stream (`void*`, a cudaStream_t;
 * NULL = legacy default stream, which is where the reference launches), and
 * returns an `int` status (PA_OK = 0, see pa_strerror).  No torch types, no
 * exceptions, no host synchronisation, no allocation: scratch memory is passed
 * in by the caller (sizes from the *_workspace_size queries).
 *
 * Each entry point replaces one function of the reference's operator API
 * (gb10-attn, kernels/*.h, loaded by hetero-serve through
 * torch.utils.cpp_extension.load_inline), or one call of hetero-serve's KV
 * pool; the replaced interface is cited beside each declaration.  Tensor
 * layouts are the reference's:
 *
 *   q            [B, H, D]        fp32, contiguous  (decode)
 *   q            [B, Sq, H, D]    fp32, contiguous  (prefill)
 *   k/v cache    [NB, BS, HKV, D] one layer's view pool[layer, 0|1] of the
 *                                 [n_layer, 2, NB, BS, HKV, D] pool, any of
 *                                 fp32 / fp16 / bf16 / fp64 (PA_DTYPE_*), or
 *                                 fp8 e4m3 for decode
 *   block_tables [B, MB]          int32; token j of sequence b lives in block
 *                                 block_tables[b][j / BS], row j % BS
 *   context_lens [B]              int32
 *   out          like q           fp32
 *
 * All element offsets are computed in 64 bits, so pools of more than 2^31
 * elements are addressed correctly.
 *
 * Device-side validation: the kernels never read outside the pool.  A block
 * id outside [0, NB) or a context longer than MB*BS is clamped to a safe read
 * and reported by OR-ing a PA_DEVERR_* bit into `*dev_status` (an int32 in
 * device memory, optional: pass NULL to skip reporting).  The reference does
 * not check these (undefined behaviour there).
 */
#ifndef PA_B200_H_
#define PA_B200_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define PA_B200_ABI_VERSION 1

#if defined(__GNUC__)
#define PA_API __attribute__((visibility("default")))
#else
#define PA_API
#endif

/* element type of the KV pool (and of write_kv sources) */
typedef enum pa_dtype {
  PA_DTYPE_F32 = 0,
  PA_DTYPE_F16 = 1,
  PA_DTYPE_BF16 = 2,
  PA_DTYPE_F64 = 3,
  /* OCP FP8 E4M3 ("e4m3fn": no infinities, max 448, 0x7f/0xff NaN), one
   * byte per element, dequantised as value * scale with an fp32 scale per KV
   * head (pa_paged_attention_v3_fp8, pa_write_kv_scaled; the entry points
   * without scales use 1.0).  Decode and write_kv only. */
  PA_DTYPE_E4M3 = 4
} pa_dtype;

/* host-side status codes (return values) */
typedef enum pa_status {
  PA_OK = 0,
  PA_ERR_INVALID_ARGUMENT = 1, /* null pointer, negative size, bad shape     */
  PA_ERR_NUM_HEADS = 2,        /* n_head must be divisible by n_kv_head      */
  PA_ERR_HEAD_DIM = 3,         /* head_dim not supported by this entry point */
  PA_ERR_DTYPE = 4,            /* KV dtype not supported by this entry point */
  PA_ERR_BLOCK_SIZE = 5,       /* block_size not supported by this entry     */
  PA_ERR_ALIGNMENT = 6,        /* a pointer is not 16-byte aligned           */
  PA_ERR_WORKSPACE = 7,        /* workspace missing or too small             */
  PA_ERR_CUDA = 8,             /* a CUDA call failed; see pa_last_cuda_error */
  PA_ERR_TOO_LARGE = 9,        /* a size exceeds a documented limit          */
  PA_ERR_NO_DEVICE = 10        /* no sm_100 device is current                */
} pa_status;

/* device-side error bits OR-ed into *dev_status */
#define PA_DEVERR_BLOCK_ID 0x1   /* block id outside [0, num_blocks)          */
#define PA_DEVERR_CONTEXT 0x2    /* context_lens[b] > max_blocks * block_size */
#define PA_DEVERR_TIMEOUT 0x4    /* a bounded pipeline wait gave up           */
#define PA_DEVERR_MERGE 0x8      /* a split-merge arrival never registered;
                                    its rows are NaN                           */
#define PA_DEVERR_RANGE 0x10     /* tensor-core prefill on an fp16 pool: a
                                    query element times scale is at or beyond
                                    the fp16 range (|x| >= 65520)             */

PA_API int pa_abi_version(void);

/* Failure-path test hook, no counterpart in the reference.  Sets the number
 * of compare-and-swap rounds a decode CTA spends registering its split piece
 * with the merge counter before it gives up (default 1 << 20, never reached
 * in practice).  A give-up writes NaN into the rows of that piece and ORs
 * PA_DEVERR_MERGE into *dev_status; 0 makes every arrival give up, which lets
 * a test drive that path without a fault or a hang.  `rounds` < 0 restores
 * the default.  Process-wide; applies to launches made after the call.
 * Returns the previous value. */
PA_API int pa_set_merge_arrive_rounds(int rounds);
PA_API const char* pa_strerror(int status);
/* cudaError_t of the most recent PA_ERR_CUDA on this thread (0 if none) */
PA_API int pa_last_cuda_error(void);

/* ------------------------------------------------------------------------ */
/* decode                                                                    */
/* ------------------------------------------------------------------------ */

/* Replaces `int64_t choose_num_splits(int64_t num_seqs, int64_t num_heads,
 * int64_t max_context)` (kernels/paged_attn_v3.h:17, body
 * kernels/paged_attn_v3.cu:170-190).  Same integer formula, evaluated with the
 * current device's SM count (148 on B200).  Returns -1 if no device. */
PA_API int64_t pa_choose_num_splits(int64_t num_seqs, int64_t num_heads,
                             int64_t max_context);

/* Bytes of scratch the decode entry points need for these sizes (plan tables,
 * merge counters and split partials).  `num_splits` <= 0 means automatic.
 * Returns 0 and sets *bytes; errors as for the launch. */
PA_API int pa_decode_workspace_size(int64_t num_seqs, int64_t num_heads,
                             int64_t num_kv_heads, int64_t head_dim,
                             int kv_dtype, int64_t block_size,
                             int64_t max_blocks, int64_t num_splits,
                             size_t* bytes);

/* Replaces `torch::Tensor paged_attention_v3(q, k_cache, v_cache,
 * block_tables, context_lens, double scale, int64_t num_splits)`
 * (kernels/paged_attn_v3.h:13-16, kernels/paged_attn_v3.cu:192-261).
 *
 * Split-KV decode: out[b,h,:] = softmax(scale * q[b,h] . K[b,:,kv(h)]) V.
 * kv(h) = h / (H / HKV).  num_splits <= 0: the B200 scheduler splits the
 * total work evenly over the SMs (one persistent CTA per SM); num_splits > 0:
 * B * num_splits * (kv-head groups) pieces of equal token count.  Either way
 * the pieces are merged with the log-sum-exp rule of
 * kernels/paged_attn_v3.cu:139-165.  A sequence with context_lens[b] <= 0
 * yields NaN (as the reference's v3 does).  `lse` (nullable, fp32 [B, H])
 * receives ln(sum_j exp(scale * q.k_j)) per row, for cross-device merges.
 * head_dim in {32, 64, 128, 256}; any block_size >= 1; K/V 16-byte aligned. */
PA_API int pa_paged_attention_v3(float* out, float* lse, const float* q,
                          const void* k_cache, const void* v_cache,
                          int kv_dtype, const int32_t* block_tables,
                          const int32_t* context_lens, int64_t num_seqs,
                          int64_t num_heads, int64_t num_kv_heads,
                          int64_t head_dim, int64_t block_size,
                          int64_t num_blocks, int64_t max_blocks,
                          double scale, int64_t num_splits, void* workspace,
                          size_t workspace_bytes, int32_t* dev_status,
                          void* stream);

/* Replaces `torch::Tensor paged_attention(q, k_cache, v_cache, block_tables,
 * context_lens, double scale)` (kernels/paged_attn_v1.h:13-15,
 * kernels/paged_attn_v1.cu:112-159).  Same result as v3 with automatic
 * splitting; the reference's v1 leaves rows with context_lens <= 0
 * uninitialised, this writes NaN. */
PA_API int pa_paged_attention(float* out, const float* q, const void* k_cache,
                       const void* v_cache, int kv_dtype,
                       const int32_t* block_tables, const int32_t* context_lens,
                       int64_t num_seqs, int64_t num_heads,
                       int64_t num_kv_heads, int64_t head_dim,
                       int64_t block_size, int64_t num_blocks,
                       int64_t max_blocks, double scale, void* workspace,
                       size_t workspace_bytes, int32_t* dev_status,
                       void* stream);

/* Replaces `torch::Tensor paged_attention_v2(q, k_cache, v_cache,
 * block_tables, context_lens, double scale)` (kernels/paged_attn_v2.h:13-15,
 * kernels/paged_attn_v2.cu:124-177).  As pa_paged_attention. */
PA_API int pa_paged_attention_v2(float* out, const float* q, const void* k_cache,
                          const void* v_cache, int kv_dtype,
                          const int32_t* block_tables,
                          const int32_t* context_lens, int64_t num_seqs,
                          int64_t num_heads, int64_t num_kv_heads,
                          int64_t head_dim, int64_t block_size,
                          int64_t num_blocks, int64_t max_blocks,
                          double scale, void* workspace,
                          size_t workspace_bytes, int32_t* dev_status,
                          void* stream);

/* pa_paged_attention_v3 for callers that cannot allocate device memory when
 * they decode -- FFI hosts that only receive device pointers from elsewhere
 * and have no allocator of their own, or serving loops that reserve all device
 * memory up front.  No counterpart in the reference (its v3 allocates its
 * scratch with torch::empty on every call).  Same arguments as
 * pa_paged_attention_v3 minus the workspace: the scratch is an 8 MiB array
 * inside the library (PA_NOALLOC_SCRATCH_BYTES, held on every GPU that loads
 * the library until exit); sizes whose pa_decode_workspace_size exceeds it
 * return PA_ERR_TOO_LARGE without launching.  The first call on a device
 * looks up the array's device address (cudaGetSymbolAddress) with that device
 * current; make that first call before any stream capture.  The address is
 * kept for the life of the process: do not use this entry point across a
 * cudaDeviceReset of the device.  All calls on a device share the array, so
 * calls that overlap on the GPU race: order them.
 * Calls no cudaMalloc / cudaFree and no allocating library routine. */
#define PA_NOALLOC_SCRATCH_BYTES (8u << 20)
PA_API int pa_paged_attention_v3_noalloc(
    float* out, float* lse, const float* q, const void* k_cache,
    const void* v_cache, int kv_dtype, const int32_t* block_tables,
    const int32_t* context_lens, int64_t num_seqs, int64_t num_heads,
    int64_t num_kv_heads, int64_t head_dim, int64_t block_size,
    int64_t num_blocks, int64_t max_blocks, double scale, int64_t num_splits,
    int32_t* dev_status, void* stream);

/* Decode of an FP8 (PA_DTYPE_E4M3) KV pool: an addition (the reference has
 * fp32/fp16/fp64 pools only; FP8 KV is listed as not measured in its
 * docs/REPORT.md:270).  Same arguments and results as pa_paged_attention_v3
 * with the pool's elements dequantised as K = k_cache * k_scale[h],
 * V = v_cache * v_scale[h]: k_scale / v_scale are device fp32 arrays of
 * num_kv_heads entries (NULL = 1.0) for this layer.  kv_dtype must be
 * PA_DTYPE_E4M3; the workspace is pa_decode_workspace_size's for that dtype. */
PA_API int pa_paged_attention_v3_fp8(float* out, float* lse, const float* q,
                                     const void* k_cache, const void* v_cache,
                                     const float* k_scale, const float* v_scale,
                                     int kv_dtype, const int32_t* block_tables,
                                     const int32_t* context_lens, int64_t num_seqs,
                                     int64_t num_heads, int64_t num_kv_heads,
                                     int64_t head_dim, int64_t block_size,
                                     int64_t num_blocks, int64_t max_blocks,
                                     double scale, int64_t num_splits, void* workspace,
                                     size_t workspace_bytes, int32_t* dev_status,
                                     void* stream);

/* Merge per-device partial results of one decode (sequence-sharded
 * long-context decode): out[b,h,:] = sum_r w_r out_r[b,h,:] / sum_r w_r with
 * w_r = exp(lse_r[b,h] - max_r lse_r[b,h]); the log-sum-exp rule of
 * kernels/paged_attn_v3.cu:139-165 applied to normalised partials.
 * outs: [R, B*H, D] fp32 contiguous; lses: [R, B*H].  lse_out nullable.
 * Rows where every partial is empty (lse = -inf) yield NaN. */
PA_API int pa_merge_states(float* out, float* lse_out, const float* outs,
                    const float* lses, int64_t num_parts, int64_t rows,
                    int64_t head_dim, void* stream);

/* ------------------------------------------------------------------------ */
/* sequence-sharded decode over peer memory (one process per GPU)           */
/* ------------------------------------------------------------------------ */
/* The same merge as pa_merge_states with the partials read straight from the
 * other GPUs' memory instead of an all-gather.  The reference is single-GPU
 * (docs/REPORT.md:274); these entry points are additions.
 *
 * Each rank allocates one exchange buffer (pa_ipc_alloc, zeroed), sends the
 * handle to every other rank by any host channel, maps theirs (pa_ipc_open)
 * and builds a device array peer_bases[world] of every rank's buffer address
 * in its own address space (its own buffer at index rank).  Layout of a
 * buffer, from pa_peer_exchange_layout for `rows` = num_seqs * num_heads:
 *   slot s (s = 0, 1) at s * slot_bytes: out [rows, head_dim] fp32 at +0,
 *   lse [rows] fp32 at +lse_offset; flags (u32 per rank) at flags_offset.
 * Step with epoch e (1, 2, 3, ..., the same on every rank, e != 0): the rank's
 * decode writes its partial (out, lse of its token range, e.g.
 * pa_paged_attention_v3 with lse) into slot e & 1 of its OWN buffer; then
 * pa_merge_peer_partials on the same stream raises flag e on every peer,
 * waits (bounded, 1 s) for every peer's flag e, and writes the merged
 * out [rows, head_dim] (and lse_out, nullable) on this device.  A wait that
 * gives up writes NaN rows and ORs PA_DEVERR_TIMEOUT into *dev_status
 * (nullable).  Every rank must call it once per epoch, in the same order.
 * world <= 32. */
#define PA_IPC_HANDLE_BYTES 64
PA_API int pa_peer_exchange_layout(int64_t rows, int64_t head_dim, size_t* lse_offset,
                                   size_t* slot_bytes, size_t* flags_offset,
                                   size_t* total_bytes);
/* cudaMalloc + zero + an IPC handle (PA_IPC_HANDLE_BYTES bytes) for it. */
PA_API int pa_ipc_alloc(size_t bytes, void** dev_ptr, void* handle);
/* Map another process's buffer; returns its address in this process. */
PA_API int pa_ipc_open(const void* handle, void** dev_ptr);
PA_API int pa_ipc_close(void* dev_ptr);  /* unmap a pa_ipc_open address   */
PA_API int pa_ipc_free(void* dev_ptr);   /* free a pa_ipc_alloc buffer    */
PA_API int pa_merge_peer_partials(float* out, float* lse_out,
                                  const uint64_t* peer_bases, int64_t world,
                                  int64_t rank, int64_t rows, int64_t head_dim,
                                  uint32_t epoch, int32_t* dev_status,
                                  void* stream);

/* ------------------------------------------------------------------------ */
/* prefill                                                                   */
/* ------------------------------------------------------------------------ */

/* Bytes of scratch the prefill entry points need for these sizes. */
PA_API int pa_prefill_workspace_size(int64_t num_seqs, int64_t num_queries,
                              int64_t num_heads, int64_t num_kv_heads,
                              int64_t head_dim, int kv_dtype,
                              int64_t block_size, int64_t max_blocks,
                              size_t* bytes);

/* Replaces `torch::Tensor paged_attention_prefill(q, k_cache, v_cache,
 * block_tables, context_lens, double scale)` (kernels/paged_attn_prefill.h:
 * 13-15, kernels/paged_attn_prefill.cu:120-175).  Causal chunked prefill:
 * query s of sequence b sits at position ctx - Sq + s and attends to keys
 * [0, ctx - Sq + s]; rows with no key are written as 0.  q/out [B,Sq,H,D]
 * fp32.  fp16/bf16 pools run on the tcgen05 tensor cores (fp32 softmax and
 * accumulation); fp32/fp64 pools on the CUDA cores. */
PA_API int pa_paged_attention_prefill(float* out, const float* q, const void* k_cache,
                               const void* v_cache, int kv_dtype,
                               const int32_t* block_tables,
                               const int32_t* context_lens, int64_t num_seqs,
                               int64_t num_queries, int64_t num_heads,
                               int64_t num_kv_heads, int64_t head_dim,
                               int64_t block_size, int64_t num_blocks,
                               int64_t max_blocks, double scale,
                               void* workspace, size_t workspace_bytes,
                               int32_t* dev_status, void* stream);

/* Replaces `torch::Tensor paged_attention_prefill_wmma(q, k_cache, v_cache,
 * block_tables, context_lens, double scale)` (kernels/paged_attn_wmma.h:
 * 13-15, kernels/paged_attn_wmma.cu:212-274): the tensor-core prefill.  Keeps
 * the reference's argument checks (fp16 pool -- bf16 is also accepted here --,
 * block_size == 16, head_dim % 16 == 0 and in {32, 64, 128}). */
PA_API int pa_paged_attention_prefill_wmma(
    float* out, const float* q, const void* k_cache, const void* v_cache,
    int kv_dtype, const int32_t* block_tables, const int32_t* context_lens,
    int64_t num_seqs, int64_t num_queries, int64_t num_heads,
    int64_t num_kv_heads, int64_t head_dim, int64_t block_size,
    int64_t num_blocks, int64_t max_blocks, double scale, void* workspace,
    size_t workspace_bytes, int32_t* dev_status, void* stream);

/* CUDA-core form of pa_paged_attention_prefill for every pool dtype (no
 * reference counterpart of its own: it is the reference's scalar prefill
 * path, kept callable so the tensor-core path can be checked against it).
 * Same arguments and workspace as pa_paged_attention_prefill. */
PA_API int pa_paged_attention_prefill_simt(
    float* out, const float* q, const void* k_cache, const void* v_cache,
    int kv_dtype, const int32_t* block_tables, const int32_t* context_lens,
    int64_t num_seqs, int64_t num_queries, int64_t num_heads,
    int64_t num_kv_heads, int64_t head_dim, int64_t block_size,
    int64_t num_blocks, int64_t max_blocks, double scale, void* workspace,
    size_t workspace_bytes, int32_t* dev_status, void* stream);

/* ------------------------------------------------------------------------ */
/* KV pool writer                                                            */
/* ------------------------------------------------------------------------ */

/* Replaces hetero-serve `TorchBlockAllocator.write_kv(block_ids, start, k, v)`
 * (heteroserve/kv/torch_blocks.py:92, un-vendored; call sites
 * harness/repro_crash.py:56-58 and harness/gb10_extended.sbatch:43-50).
 *
 * For every layer l < num_layers, kv head h < num_kv_heads and token
 * t < num_tokens, with position p = start + t:
 *   K_l[block_ids[p / BS], p % BS, h, :] = convert(k_src[l, h, t, :])
 *   V_l[...]                             = convert(v_src[l, h, t, :])
 * where K_l = k_layers[l] and V_l = v_layers[l] point at [NB, BS, HKV, D]
 * arrays of `pool_dtype` (one per-layer tensor each, or views into one
 * [n_layer, 2, NB, BS, HKV, D] pool) and convert() rounds to nearest even.
 * k_layers / v_layers are HOST arrays of num_layers device pointers.
 * Sources are device arrays of `src_dtype` with head_dim contiguous and the
 * given element strides (the reference passes contiguous [L, H, T, D]).
 * block_ids: device int32 [num_block_ids].  Offsets are 64-bit. */
PA_API int pa_write_kv(void* const* k_layers, void* const* v_layers, int pool_dtype,
                const void* k_src, const void* v_src, int src_dtype,
                int64_t src_layer_stride, int64_t src_head_stride,
                int64_t src_token_stride, const int32_t* block_ids,
                int64_t num_block_ids, int64_t start, int64_t num_tokens,
                int64_t num_layers, int64_t num_kv_heads, int64_t head_dim,
                int64_t block_size, int64_t num_blocks, int32_t* dev_status,
                void* stream);

/* pa_write_kv with per-(layer, kv head) scales for an FP8 pool: element x is
 * stored as e4m3(x / scale) (IEEE fp32 division, then round to nearest even,
 * saturating to +-448; NaN stays NaN).  k_scales / v_scales: device fp32
 * [num_layers, num_kv_heads] (NULL = 1.0); ignored for other pool dtypes. */
PA_API int pa_write_kv_scaled(void* const* k_layers, void* const* v_layers, int pool_dtype,
                              const void* k_src, const void* v_src, int src_dtype,
                              int64_t src_layer_stride, int64_t src_head_stride,
                              int64_t src_token_stride, const int32_t* block_ids,
                              int64_t num_block_ids, int64_t start, int64_t num_tokens,
                              int64_t num_layers, int64_t num_kv_heads, int64_t head_dim,
                              int64_t block_size, int64_t num_blocks,
                              const float* k_scales, const float* v_scales,
                              int32_t* dev_status, void* stream);

/* One sequence of a pa_write_kv_batch call: the arguments pa_write_kv takes
 * per sequence.  k_src / v_src: device [num_layers, num_kv_heads, num_tokens,
 * head_dim] of the call's src_dtype, head_dim contiguous, the given element
 * strides; block_ids: device int32 [num_block_ids]; token t lands at sequence
 * position start + t. */
typedef struct pa_kv_seq {
  const void* k_src;
  const void* v_src;
  int64_t src_layer_stride, src_head_stride, src_token_stride;
  const int32_t* block_ids;
  int64_t num_block_ids;
  int64_t start;
  int64_t num_tokens;
} pa_kv_seq;

/* pa_write_kv_scaled for many sequences in one call, an addition (the
 * reference's TorchBlockAllocator.write_kv, heteroserve/kv/torch_blocks.py:92,
 * writes one sequence per call, as pa_write_kv does): the result equals one
 * pa_write_kv_scaled per entry of `seqs` (a HOST array of num_seqs), with up
 * to 32 sequences and 64 layers per kernel launch.  Entries are validated
 * before anything is launched; sequences must not write the same pool row. */
PA_API int pa_write_kv_batch(void* const* k_layers, void* const* v_layers, int pool_dtype,
                             int src_dtype, const pa_kv_seq* seqs, int64_t num_seqs,
                             int64_t num_layers, int64_t num_kv_heads, int64_t head_dim,
                             int64_t block_size, int64_t num_blocks, const float* k_scales,
                             const float* v_scales, int32_t* dev_status, void* stream);

/* One decode step's K/V append for a batch, an addition (the reference
 * writes whole sequences with write_kv only): for every layer l < num_layers,
 * sequence b < num_seqs with positions[b] >= 0 and kv head h,
 *   K_l[block_tables[b][p / BS], p % BS, h, :] = convert(k_new[l, b, h, :])
 * (and V likewise) with p = positions[b], the slot of the sequence's next
 * token.  k_new / v_new: device [num_layers, num_seqs, num_kv_heads,
 * head_dim], contiguous, of src_dtype; block_tables: device int32
 * [num_seqs, max_blocks]; positions: device int32 [num_seqs] (< 0 skips the
 * sequence).  Conversion and FP8 scales as pa_write_kv_scaled (scales
 * nullable).  A position past the block table is skipped and reported as
 * PA_DEVERR_CONTEXT, a block id outside [0, num_blocks) as PA_DEVERR_BLOCK_ID. */
PA_API int pa_append_kv(void* const* k_layers, void* const* v_layers, int pool_dtype,
                        const void* k_new, const void* v_new, int src_dtype,
                        const int32_t* block_tables, int64_t max_blocks,
                        const int32_t* positions, int64_t num_seqs, int64_t num_layers,
                        int64_t num_kv_heads, int64_t head_dim, int64_t block_size,
                        int64_t num_blocks, const float* k_scales, const float* v_scales,
                        int32_t* dev_status, void* stream);

/* One layer of a serving loop's decode step, an addition (the reference's
 * decode takes fp32 q and returns fp32 out, kernels/paged_attn_v3.cu:211-214,
 * and writes K/V only through write_kv): pa_paged_attention_v3 with
 *   - q [num_seqs, num_heads, head_dim] and out (same shape) of io_dtype
 *     (PA_DTYPE_F32, PA_DTYPE_F16 or PA_DTYPE_BF16; out is rounded to nearest
 *     even; lse, when given, stays fp32 [num_seqs, num_heads]);
 *   - when k_new / v_new are given (device [num_seqs, num_kv_heads, head_dim]
 *     of io_dtype, both or neither), sequence b's new K / V row stored at
 *     position context_lens[b] - 1 of its pages (converted as pa_write_kv
 *     does) inside the same launch, before the attention reads it: the
 *     append and the decode are one kernel.  context_lens counts the new
 *     token; sequences with context_lens[b] == 0 append nothing.
 * FP8 pools with k_new return PA_ERR_DTYPE (use pa_append_kv, which takes the
 * scales).  Workspace: pa_decode_workspace_size for the same shape. */
PA_API int pa_decode_layer_step(void* out, float* lse, const void* q, int io_dtype,
                                void* k_cache, void* v_cache, int kv_dtype,
                                const void* k_new, const void* v_new,
                                const int32_t* block_tables, const int32_t* context_lens,
                                int64_t num_seqs, int64_t num_heads, int64_t num_kv_heads,
                                int64_t head_dim, int64_t block_size, int64_t num_blocks,
                                int64_t max_blocks, double scale, int64_t num_splits,
                                void* workspace, size_t workspace_bytes, int32_t* dev_status,
                                void* stream);

/* Opt-in check of a block table (the reference has none): counts entries
 * used by context_lens that fall outside [0, num_blocks), and sequences whose
 * context exceeds max_blocks * block_size.  Writes the two counts to the
 * device int32 pair counts[0..1]. */
PA_API int pa_validate_block_tables(const int32_t* block_tables,
                             const int32_t* context_lens, int64_t num_seqs,
                             int64_t max_blocks, int64_t block_size,
                             int64_t num_blocks, int32_t* counts,
                             void* stream);

#ifdef __cplusplus
}
#endif

#endif /* PA_B200_H_ */
