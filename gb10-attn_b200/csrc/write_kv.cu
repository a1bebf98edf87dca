// write_kv.cu -- KV-pool writer (C ABI pa_write_kv, pa_write_kv_scaled), its
// many-sequence form (pa_write_kv_batch) and the batched one-token append of
// a decode step (pa_append_kv).
//
// Replaces hetero-serve TorchBlockAllocator.write_kv(block_ids, start, k, v)
// (heteroserve/kv/torch_blocks.py:92, un-vendored; behaviour from the call
// sites harness/repro_crash.py:52-58 and gb10-attn docs/REPORT.md:141-179):
// token t of the source, at sequence position p = start + t, goes to row
// p % BS of block block_ids[p / BS] of every layer's K and V pool, for every
// kv head, converted to the pool dtype with round-to-nearest-even (FP8 E4M3
// pools: x / scale[layer, head] first, saturating at +-448; an addition).
//
// The reference did this with torch indexing on one [n_layer, 2, NB, BS, H, D]
// tensor and faulted once that tensor passed 2^31 elements
// (gb10-attn README.md:109-132).  Here every offset is 64-bit and each layer's
// K and V are separate base pointers (monolithic pool views or one tensor per
// layer alike), in one launch for all layers.
//
// Memory-bound gather/scatter: each thread moves 8 elements of one
// (layer, K|V, token, head) row, 16-byte vector stores into the pool.
#include <algorithm>

#include "common.cuh"

namespace pa {
namespace writekv {

constexpr int kMaxLayers = 64;  // layers per launch; more are split on the host

struct Params {
  char* k_layers[kMaxLayers];
  char* v_layers[kMaxLayers];
  const char* k_src;
  const char* v_src;
  int64_t src_layer_stride, src_head_stride, src_token_stride;  // elements
  const int32_t* block_ids;
  int64_t n_ids;
  int64_t start, T, L, HKV, D, BS, NB;
  // Batched append (pa_append_kv): source token t is the next token of
  // sequence t, at position positions[t] (< 0: none), and block_ids is the
  // [T, n_ids] block table.  Null for the one-sequence writer.
  const int32_t* positions;
  // FP8 pools: [L, HKV] quantisation scales (null = 1); this launch's layers
  const float* k_scales;
  const float* v_scales;
  int32_t* dev_status;
};

template <typename S>
__device__ __forceinline__ float to_f32(S x);
template <> __device__ __forceinline__ float to_f32<float>(float x) { return x; }
template <> __device__ __forceinline__ float to_f32<__half>(__half x) { return __half2float(x); }
template <> __device__ __forceinline__ float to_f32<__nv_bfloat16>(__nv_bfloat16 x) {
  return __bfloat162float(x);
}

template <typename P>
__device__ __forceinline__ P from_f32(float x);
template <> __device__ __forceinline__ float from_f32<float>(float x) { return x; }
template <> __device__ __forceinline__ double from_f32<double>(float x) { return (double)x; }
template <> __device__ __forceinline__ __half from_f32<__half>(float x) { return __float2half_rn(x); }
template <> __device__ __forceinline__ __nv_bfloat16 from_f32<__nv_bfloat16>(float x) {
  return __float2bfloat16_rn(x);
}
// round to nearest even, saturating to the largest finite e4m3 (+-448)
template <> __device__ __forceinline__ __nv_fp8_e4m3 from_f32<__nv_fp8_e4m3>(float x) {
  __nv_fp8_e4m3 r;
  r.__x = __nv_cvt_float_to_fp8(x, __NV_SATFINITE, __NV_E4M3);
  return r;
}

// One pool element group: E elements of source row (l, kv, h, t) from `src`
// converted into `dst` (VEC: 8 elements with 16-byte accesses, else 1).
template <typename S, typename P, bool VEC>
__device__ __forceinline__ void convert_chunk(const S* src, P* dst, float qs) {
  if constexpr (VEC) {
    float f[8];
    if constexpr (sizeof(S) == 4) {
      const float4 a = __ldcs(reinterpret_cast<const float4*>(src));
      const float4 b = __ldcs(reinterpret_cast<const float4*>(src) + 1);
      f[0] = a.x; f[1] = a.y; f[2] = a.z; f[3] = a.w;
      f[4] = b.x; f[5] = b.y; f[6] = b.z; f[7] = b.w;
    } else {
      const uint4 u = __ldcs(reinterpret_cast<const uint4*>(src));
      const S* s8 = reinterpret_cast<const S*>(&u);
#pragma unroll
      for (int e = 0; e < 8; ++e) f[e] = to_f32<S>(s8[e]);
    }
    if constexpr (sizeof(P) == 1) {
      uint2 u;
      P* d8 = reinterpret_cast<P*>(&u);
#pragma unroll
      for (int e = 0; e < 8; ++e) d8[e] = from_f32<P>(__fdiv_rn(f[e], qs));
      *reinterpret_cast<uint2*>(dst) = u;
    } else if constexpr (sizeof(P) == 2) {
      uint4 u;
      P* d8 = reinterpret_cast<P*>(&u);
#pragma unroll
      for (int e = 0; e < 8; ++e) d8[e] = from_f32<P>(f[e]);
      *reinterpret_cast<uint4*>(dst) = u;
    } else if constexpr (sizeof(P) == 4) {
      reinterpret_cast<float4*>(dst)[0] = make_float4(f[0], f[1], f[2], f[3]);
      reinterpret_cast<float4*>(dst)[1] = make_float4(f[4], f[5], f[6], f[7]);
    } else {
#pragma unroll
      for (int e = 0; e < 8; e += 2)
        reinterpret_cast<double2*>(dst)[e / 2] = make_double2((double)f[e], (double)f[e + 1]);
    }
  } else {
    if constexpr (sizeof(P) == 1)
      *dst = from_f32<P>(__fdiv_rn(to_f32<S>(*src), qs));
    else
      *dst = from_f32<P>(to_f32<S>(*src));
  }
}

// Work unit = one token row (layer l, K or V, source token t): all HKV heads
// x D elements of that token, which land contiguously in one page row of the
// pool.  A CTA takes `rpi` rows per iteration (several when a row has fewer
// element groups than the CTA has threads); the row's position, page and
// block id are resolved once per row, and the head / group split of an
// element group is a shift when D / E is a power of two.
template <typename S, typename P, bool VEC>
__global__ void __launch_bounds__(256) write_kv_kernel(const __grid_constant__ Params p,
                                                       int32_t per_tok, int32_t per_head_shift,
                                                       int32_t rpi) {
  constexpr int E = VEC ? 8 : 1;
  const int32_t per_head = (int32_t)(p.D / E);
  const int64_t n_rows = p.L * 2 * p.T;
  const int sub = threadIdx.x / per_tok;  // row within this CTA's iteration
  const int32_t c0 = threadIdx.x - sub * per_tok;
  const int32_t cstep = rpi > 1 ? per_tok : (int32_t)blockDim.x;
  if (sub >= rpi) return;
  for (int64_t row = (int64_t)blockIdx.x * rpi + sub; row < n_rows;
       row += (int64_t)gridDim.x * rpi) {
    const int64_t t = row % p.T;
    const int64_t lk = row / p.T;
    const int kv = (int)(lk & 1);
    const int64_t l = lk >> 1;
    int64_t pos, page, blk;
    if (p.positions) {
      pos = p.positions[t];
      if (pos < 0) continue;
      page = pos / p.BS;
      if (page >= p.n_ids) {  // past the sequence's block table
        if (c0 == 0) report(p.dev_status, PA_DEVERR_CONTEXT);
        continue;
      }
      blk = p.block_ids[t * p.n_ids + page];
    } else {
      pos = p.start + t;
      page = pos / p.BS;
      if (page >= p.n_ids) {
        if (c0 == 0) report(p.dev_status, PA_DEVERR_BLOCK_ID);
        continue;
      }
      blk = p.block_ids[page];
    }
    if (blk < 0 || blk >= p.NB) {
      if (c0 == 0) report(p.dev_status, PA_DEVERR_BLOCK_ID);
      continue;
    }
    const S* src = reinterpret_cast<const S*>(kv ? p.v_src : p.k_src) + l * p.src_layer_stride +
                   t * p.src_token_stride;
    P* dst = reinterpret_cast<P*>(kv ? p.v_layers[l] : p.k_layers[l]) +
             (blk * p.BS + (pos - page * p.BS)) * p.HKV * p.D;
    const float* sc = kv ? p.v_scales : p.k_scales;
    for (int32_t c = c0; c < per_tok; c += cstep) {
      const int32_t h = per_head_shift >= 0 ? (c >> per_head_shift) : c / per_head;
      const int32_t ch = c - h * per_head;
      float qs = 1.f;  // FP8: stored value = x / scale
      if constexpr (sizeof(P) == 1) {
        if (sc) qs = sc[l * p.HKV + h];
      }
      convert_chunk<S, P, VEC>(src + h * p.src_head_stride + (int64_t)ch * E,
                               dst + (int64_t)c * E, qs);
    }
  }
}

// Batched writer (pa_write_kv_batch): up to kMaxSeqs sequences per launch,
// each with its own source, strides, block ids, start and token count.  Work
// rows are numbered sequence by sequence (row0[s] .. row0[s + 1]); within a
// sequence, as in write_kv_kernel, row = (2 l + kv) T + t.
constexpr int kMaxSeqs = 32;

struct SeqDesc {
  const char* k_src;  // this launch's first layer
  const char* v_src;
  int64_t layer_stride, head_stride, token_stride;  // elements
  const int32_t* block_ids;
  int64_t n_ids, start, T;
};

struct BatchParams {
  char* k_layers[kMaxLayers];
  char* v_layers[kMaxLayers];
  SeqDesc seq[kMaxSeqs];
  int64_t row0[kMaxSeqs + 1];
  int32_t n_seqs;
  int64_t L, HKV, D, BS, NB;
  const float* k_scales;  // FP8 pools: [L, HKV] of this launch's layers (null = 1)
  const float* v_scales;
  int32_t* dev_status;
};

template <typename S, typename P, bool VEC>
__global__ void __launch_bounds__(256) write_kv_batch_kernel(const __grid_constant__ BatchParams p,
                                                             int32_t per_tok, int32_t per_head_shift,
                                                             int32_t rpi) {
  constexpr int E = VEC ? 8 : 1;
  const int32_t per_head = (int32_t)(p.D / E);
  const int64_t n_rows = p.row0[p.n_seqs];
  const int sub = threadIdx.x / per_tok;
  const int32_t c0 = threadIdx.x - sub * per_tok;
  const int32_t cstep = rpi > 1 ? per_tok : (int32_t)blockDim.x;
  if (sub >= rpi) return;
  int s = 0;  // rows only grow along the loop, so the sequence index does too
  for (int64_t row = (int64_t)blockIdx.x * rpi + sub; row < n_rows;
       row += (int64_t)gridDim.x * rpi) {
    while (s + 1 < p.n_seqs && p.row0[s + 1] <= row) ++s;
    const SeqDesc& q = p.seq[s];
    const int64_t r = row - p.row0[s];
    const int64_t t = r % q.T;
    const int64_t lk = r / q.T;
    const int kv = (int)(lk & 1);
    const int64_t l = lk >> 1;
    const int64_t pos = q.start + t;
    const int64_t page = pos / p.BS;
    if (page >= q.n_ids) {
      if (c0 == 0) report(p.dev_status, PA_DEVERR_BLOCK_ID);
      continue;
    }
    const int64_t blk = q.block_ids[page];
    if (blk < 0 || blk >= p.NB) {
      if (c0 == 0) report(p.dev_status, PA_DEVERR_BLOCK_ID);
      continue;
    }
    const S* src = reinterpret_cast<const S*>(kv ? q.v_src : q.k_src) + l * q.layer_stride +
                   t * q.token_stride;
    P* dst = reinterpret_cast<P*>(kv ? p.v_layers[l] : p.k_layers[l]) +
             (blk * p.BS + (pos - page * p.BS)) * p.HKV * p.D;
    const float* sc = kv ? p.v_scales : p.k_scales;
    for (int32_t c = c0; c < per_tok; c += cstep) {
      const int32_t h = per_head_shift >= 0 ? (c >> per_head_shift) : c / per_head;
      const int32_t ch = c - h * per_head;
      float qs = 1.f;  // FP8: stored value = x / scale
      if constexpr (sizeof(P) == 1) {
        if (sc) qs = sc[l * p.HKV + h];
      }
      convert_chunk<S, P, VEC>(src + h * q.head_stride + (int64_t)ch * E, dst + (int64_t)c * E, qs);
    }
  }
}

// Launch geometry shared by both writers: element groups per token row, rows
// per CTA iteration, the head shift and the grid (SMs x 16 at most).
struct Geometry {
  int64_t per_tok;
  int rpi, shift;
  int64_t blocks;
};
static int geometry(int64_t D, int64_t HKV, int64_t n_rows, bool vec, Geometry* g) {
  const int64_t per_head = vec ? D / 8 : D;
  g->per_tok = HKV * per_head;
  if (g->per_tok > (int64_t(1) << 30)) return PA_ERR_TOO_LARGE;
  int sms = 148;
  if (device_sm_count(&sms) != PA_OK) return PA_ERR_NO_DEVICE;
  constexpr int kThreads = 256;
  g->rpi = g->per_tok >= kThreads ? 1 : (int)(kThreads / g->per_tok);
  g->shift = -1;
  if ((per_head & (per_head - 1)) == 0) {
    g->shift = 0;
    while ((int64_t(1) << g->shift) < per_head) ++g->shift;
  }
  g->blocks = std::max<int64_t>(1, std::min<int64_t>((n_rows + g->rpi - 1) / g->rpi, (int64_t)sms * 16));
  return PA_OK;
}

template <typename S, typename P>
static int launch_batch_typed(const BatchParams& p, bool vec, cudaStream_t s) {
  const int64_t n_rows = p.row0[p.n_seqs];
  if (n_rows == 0) return PA_OK;
  Geometry g;
  const int st = geometry(p.D, p.HKV, n_rows, vec, &g);
  if (st != PA_OK) return st;
  if (vec)
    write_kv_batch_kernel<S, P, true><<<(unsigned)g.blocks, 256, 0, s>>>(p, (int32_t)g.per_tok, g.shift, g.rpi);
  else
    write_kv_batch_kernel<S, P, false><<<(unsigned)g.blocks, 256, 0, s>>>(p, (int32_t)g.per_tok, g.shift, g.rpi);
  return cuda_status(cudaGetLastError());
}

template <typename S>
static int launch_batch_src(const BatchParams& p, int pool_dtype, bool vec, cudaStream_t s) {
  switch (pool_dtype) {
    case PA_DTYPE_F16: return launch_batch_typed<S, __half>(p, vec, s);
    case PA_DTYPE_BF16: return launch_batch_typed<S, __nv_bfloat16>(p, vec, s);
    case PA_DTYPE_F32: return launch_batch_typed<S, float>(p, vec, s);
    case PA_DTYPE_F64: return launch_batch_typed<S, double>(p, vec, s);
    case PA_DTYPE_E4M3: return launch_batch_typed<S, __nv_fp8_e4m3>(p, vec, s);
    default: return PA_ERR_DTYPE;
  }
}

template <typename S, typename P>
static int launch_typed(const Params& p, bool vec, cudaStream_t s) {
  const int64_t per_head = vec ? p.D / 8 : p.D;
  const int64_t per_tok = p.HKV * per_head;
  const int64_t n_rows = p.L * 2 * p.T;
  if (n_rows == 0 || per_tok == 0) return PA_OK;
  if (per_tok > (int64_t(1) << 30)) return PA_ERR_TOO_LARGE;
  int sms = 148;
  if (device_sm_count(&sms) != PA_OK) return PA_ERR_NO_DEVICE;
  constexpr int kThreads = 256;
  const int rpi = per_tok >= kThreads ? 1 : (int)(kThreads / per_tok);
  int shift = -1;
  if ((per_head & (per_head - 1)) == 0) {
    shift = 0;
    while ((int64_t(1) << shift) < per_head) ++shift;
  }
  const int64_t blocks =
      std::max<int64_t>(1, std::min<int64_t>((n_rows + rpi - 1) / rpi, (int64_t)sms * 16));
  if (vec)
    write_kv_kernel<S, P, true><<<(unsigned)blocks, kThreads, 0, s>>>(p, (int32_t)per_tok, shift, rpi);
  else
    write_kv_kernel<S, P, false><<<(unsigned)blocks, kThreads, 0, s>>>(p, (int32_t)per_tok, shift, rpi);
  return cuda_status(cudaGetLastError());
}

template <typename S>
static int launch_src(const Params& p, int pool_dtype, bool vec, cudaStream_t s) {
  switch (pool_dtype) {
    case PA_DTYPE_F16: return launch_typed<S, __half>(p, vec, s);
    case PA_DTYPE_BF16: return launch_typed<S, __nv_bfloat16>(p, vec, s);
    case PA_DTYPE_F32: return launch_typed<S, float>(p, vec, s);
    case PA_DTYPE_F64: return launch_typed<S, double>(p, vec, s);
    case PA_DTYPE_E4M3: return launch_typed<S, __nv_fp8_e4m3>(p, vec, s);
    default: return PA_ERR_DTYPE;
  }
}

}  // namespace writekv
}  // namespace pa

extern "C" int pa_write_kv(void* const* k_layers, void* const* v_layers, int pool_dtype,
                           const void* k_src, const void* v_src, int src_dtype,
                           int64_t src_layer_stride, int64_t src_head_stride,
                           int64_t src_token_stride, const int32_t* block_ids,
                           int64_t num_block_ids, int64_t start, int64_t num_tokens,
                           int64_t num_layers, int64_t num_kv_heads, int64_t head_dim,
                           int64_t block_size, int64_t num_blocks, int32_t* dev_status,
                           void* stream) {
  return pa_write_kv_scaled(k_layers, v_layers, pool_dtype, k_src, v_src, src_dtype,
                            src_layer_stride, src_head_stride, src_token_stride, block_ids,
                            num_block_ids, start, num_tokens, num_layers, num_kv_heads,
                            head_dim, block_size, num_blocks, nullptr, nullptr, dev_status,
                            stream);
}

extern "C" int pa_write_kv_scaled(void* const* k_layers, void* const* v_layers, int pool_dtype,
                                  const void* k_src, const void* v_src, int src_dtype,
                                  int64_t src_layer_stride, int64_t src_head_stride,
                                  int64_t src_token_stride, const int32_t* block_ids,
                                  int64_t num_block_ids, int64_t start, int64_t num_tokens,
                                  int64_t num_layers, int64_t num_kv_heads, int64_t head_dim,
                                  int64_t block_size, int64_t num_blocks,
                                  const float* k_scales, const float* v_scales,
                                  int32_t* dev_status, void* stream) {
  using namespace pa;
  using writekv::kMaxLayers;
  if (num_tokens < 0 || num_layers < 0 || num_kv_heads <= 0 || head_dim <= 0 ||
      block_size <= 0 || num_blocks < 0 || start < 0 || num_block_ids < 0)
    return PA_ERR_INVALID_ARGUMENT;
  if (num_tokens == 0 || num_layers == 0) return PA_OK;
  if (!k_layers || !v_layers || !k_src || !v_src || !block_ids) return PA_ERR_INVALID_ARGUMENT;
  if (src_dtype != PA_DTYPE_F32 && src_dtype != PA_DTYPE_F16 && src_dtype != PA_DTYPE_BF16)
    return PA_ERR_DTYPE;
  const int ps = dtype_size(pool_dtype), ss = dtype_size(src_dtype);
  if (ps == 0) return PA_ERR_DTYPE;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  for (int64_t l0 = 0; l0 < num_layers; l0 += kMaxLayers) {
    const int64_t nl = std::min<int64_t>(kMaxLayers, num_layers - l0);
    writekv::Params p = {};
    bool vec = (head_dim % 8 == 0) && aligned16(k_src) && aligned16(v_src) &&
               (src_layer_stride * ss) % 16 == 0 && (src_head_stride * ss) % 16 == 0 &&
               (src_token_stride * ss) % 16 == 0 && (head_dim * ps) % 16 == 0;
    for (int64_t l = 0; l < nl; ++l) {
      p.k_layers[l] = static_cast<char*>(k_layers[l0 + l]);
      p.v_layers[l] = static_cast<char*>(v_layers[l0 + l]);
      if (!p.k_layers[l] || !p.v_layers[l]) return PA_ERR_INVALID_ARGUMENT;
      vec = vec && aligned16(p.k_layers[l]) && aligned16(p.v_layers[l]);
    }
    p.k_src = static_cast<const char*>(k_src) + l0 * src_layer_stride * ss;
    p.v_src = static_cast<const char*>(v_src) + l0 * src_layer_stride * ss;
    p.src_layer_stride = src_layer_stride;
    p.src_head_stride = src_head_stride;
    p.src_token_stride = src_token_stride;
    p.block_ids = block_ids;
    p.n_ids = num_block_ids;
    p.start = start;
    p.T = num_tokens;
    p.L = nl;
    p.HKV = num_kv_heads;
    p.D = head_dim;
    p.BS = block_size;
    p.NB = num_blocks;
    p.k_scales = k_scales ? k_scales + l0 * num_kv_heads : nullptr;
    p.v_scales = v_scales ? v_scales + l0 * num_kv_heads : nullptr;
    p.dev_status = dev_status;
    int st;
    switch (src_dtype) {
      case PA_DTYPE_F32: st = writekv::launch_src<float>(p, pool_dtype, vec, s); break;
      case PA_DTYPE_F16: st = writekv::launch_src<__half>(p, pool_dtype, vec, s); break;
      default: st = writekv::launch_src<__nv_bfloat16>(p, pool_dtype, vec, s); break;
    }
    if (st) return st;
  }
  return PA_OK;
}

extern "C" int pa_write_kv_batch(void* const* k_layers, void* const* v_layers, int pool_dtype,
                                 int src_dtype, const pa_kv_seq* seqs, int64_t num_seqs,
                                 int64_t num_layers, int64_t num_kv_heads, int64_t head_dim,
                                 int64_t block_size, int64_t num_blocks, const float* k_scales,
                                 const float* v_scales, int32_t* dev_status, void* stream) {
  using namespace pa;
  using writekv::kMaxLayers;
  using writekv::kMaxSeqs;
  if (num_seqs < 0 || num_layers < 0 || num_kv_heads <= 0 || head_dim <= 0 || block_size <= 0 ||
      num_blocks < 0)
    return PA_ERR_INVALID_ARGUMENT;
  if (num_seqs == 0 || num_layers == 0) return PA_OK;
  if (!k_layers || !v_layers || !seqs) return PA_ERR_INVALID_ARGUMENT;
  if (src_dtype != PA_DTYPE_F32 && src_dtype != PA_DTYPE_F16 && src_dtype != PA_DTYPE_BF16)
    return PA_ERR_DTYPE;
  const int ps = dtype_size(pool_dtype), ss = dtype_size(src_dtype);
  if (ps == 0) return PA_ERR_DTYPE;
  // every sequence is checked before anything is launched
  bool vec_src = head_dim % 8 == 0 && (head_dim * ps) % 16 == 0;
  for (int64_t i = 0; i < num_seqs; ++i) {
    const pa_kv_seq& q = seqs[i];
    if (q.num_tokens < 0 || q.start < 0 || q.num_block_ids < 0) return PA_ERR_INVALID_ARGUMENT;
    if (q.num_tokens == 0) continue;
    if (!q.k_src || !q.v_src || !q.block_ids) return PA_ERR_INVALID_ARGUMENT;
    vec_src = vec_src && aligned16(q.k_src) && aligned16(q.v_src) &&
              (q.src_layer_stride * ss) % 16 == 0 && (q.src_head_stride * ss) % 16 == 0 &&
              (q.src_token_stride * ss) % 16 == 0;
  }
  for (int64_t l = 0; l < num_layers; ++l) {
    if (!k_layers[l] || !v_layers[l]) return PA_ERR_INVALID_ARGUMENT;
    vec_src = vec_src && aligned16(k_layers[l]) && aligned16(v_layers[l]);
  }
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  for (int64_t l0 = 0; l0 < num_layers; l0 += kMaxLayers) {
    const int64_t nl = std::min<int64_t>(kMaxLayers, num_layers - l0);
    int64_t i = 0;
    while (i < num_seqs) {
      writekv::BatchParams p = {};
      for (int64_t l = 0; l < nl; ++l) {
        p.k_layers[l] = static_cast<char*>(k_layers[l0 + l]);
        p.v_layers[l] = static_cast<char*>(v_layers[l0 + l]);
      }
      // the next (up to) kMaxSeqs sequences with tokens
      int n = 0;
      int64_t rows = 0;
      for (; i < num_seqs && n < kMaxSeqs; ++i) {
        const pa_kv_seq& q = seqs[i];
        if (q.num_tokens == 0) continue;
        writekv::SeqDesc& d = p.seq[n];
        d.k_src = static_cast<const char*>(q.k_src) + l0 * q.src_layer_stride * ss;
        d.v_src = static_cast<const char*>(q.v_src) + l0 * q.src_layer_stride * ss;
        d.layer_stride = q.src_layer_stride;
        d.head_stride = q.src_head_stride;
        d.token_stride = q.src_token_stride;
        d.block_ids = q.block_ids;
        d.n_ids = q.num_block_ids;
        d.start = q.start;
        d.T = q.num_tokens;
        p.row0[n] = rows;
        rows += nl * 2 * q.num_tokens;
        ++n;
      }
      if (n == 0) break;
      p.row0[n] = rows;
      p.n_seqs = n;
      p.L = nl;
      p.HKV = num_kv_heads;
      p.D = head_dim;
      p.BS = block_size;
      p.NB = num_blocks;
      p.k_scales = k_scales ? k_scales + l0 * num_kv_heads : nullptr;
      p.v_scales = v_scales ? v_scales + l0 * num_kv_heads : nullptr;
      p.dev_status = dev_status;
      int st;
      switch (src_dtype) {
        case PA_DTYPE_F32: st = writekv::launch_batch_src<float>(p, pool_dtype, vec_src, s); break;
        case PA_DTYPE_F16: st = writekv::launch_batch_src<__half>(p, pool_dtype, vec_src, s); break;
        default: st = writekv::launch_batch_src<__nv_bfloat16>(p, pool_dtype, vec_src, s); break;
      }
      if (st) return st;
    }
  }
  return PA_OK;
}

extern "C" int pa_append_kv(void* const* k_layers, void* const* v_layers, int pool_dtype,
                            const void* k_new, const void* v_new, int src_dtype,
                            const int32_t* block_tables, int64_t max_blocks,
                            const int32_t* positions, int64_t num_seqs, int64_t num_layers,
                            int64_t num_kv_heads, int64_t head_dim, int64_t block_size,
                            int64_t num_blocks, const float* k_scales, const float* v_scales,
                            int32_t* dev_status, void* stream) {
  using namespace pa;
  using writekv::kMaxLayers;
  if (num_seqs < 0 || num_layers < 0 || num_kv_heads <= 0 || head_dim <= 0 ||
      block_size <= 0 || num_blocks < 0 || max_blocks < 0)
    return PA_ERR_INVALID_ARGUMENT;
  if (num_seqs == 0 || num_layers == 0) return PA_OK;
  if (!k_layers || !v_layers || !k_new || !v_new || !block_tables || !positions)
    return PA_ERR_INVALID_ARGUMENT;
  if (src_dtype != PA_DTYPE_F32 && src_dtype != PA_DTYPE_F16 && src_dtype != PA_DTYPE_BF16)
    return PA_ERR_DTYPE;
  const int ps = dtype_size(pool_dtype), ss = dtype_size(src_dtype);
  if (ps == 0) return PA_ERR_DTYPE;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  // source [num_layers, num_seqs, num_kv_heads, head_dim], contiguous
  const int64_t head_stride = head_dim, seq_stride = num_kv_heads * head_dim;
  const int64_t layer_stride = num_seqs * seq_stride;
  for (int64_t l0 = 0; l0 < num_layers; l0 += kMaxLayers) {
    const int64_t nl = std::min<int64_t>(kMaxLayers, num_layers - l0);
    writekv::Params p = {};
    bool vec = (head_dim % 8 == 0) && aligned16(k_new) && aligned16(v_new) &&
               (head_dim * ss) % 16 == 0 && (head_dim * ps) % 16 == 0;
    for (int64_t l = 0; l < nl; ++l) {
      p.k_layers[l] = static_cast<char*>(k_layers[l0 + l]);
      p.v_layers[l] = static_cast<char*>(v_layers[l0 + l]);
      if (!p.k_layers[l] || !p.v_layers[l]) return PA_ERR_INVALID_ARGUMENT;
      vec = vec && aligned16(p.k_layers[l]) && aligned16(p.v_layers[l]);
    }
    p.k_src = static_cast<const char*>(k_new) + l0 * layer_stride * ss;
    p.v_src = static_cast<const char*>(v_new) + l0 * layer_stride * ss;
    p.src_layer_stride = layer_stride;
    p.src_head_stride = head_stride;
    p.src_token_stride = seq_stride;
    p.block_ids = block_tables;
    p.n_ids = max_blocks;
    p.positions = positions;
    p.T = num_seqs;
    p.L = nl;
    p.HKV = num_kv_heads;
    p.D = head_dim;
    p.BS = block_size;
    p.NB = num_blocks;
    p.k_scales = k_scales ? k_scales + l0 * num_kv_heads : nullptr;
    p.v_scales = v_scales ? v_scales + l0 * num_kv_heads : nullptr;
    p.dev_status = dev_status;
    int st;
    switch (src_dtype) {
      case PA_DTYPE_F32: st = writekv::launch_src<float>(p, pool_dtype, vec, s); break;
      case PA_DTYPE_F16: st = writekv::launch_src<__half>(p, pool_dtype, vec, s); break;
      default: st = writekv::launch_src<__nv_bfloat16>(p, pool_dtype, vec, s); break;
    }
    if (st) return st;
  }
  return PA_OK;
}
