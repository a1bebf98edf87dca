// prefill_tc.cu -- causal paged prefill on the sm_100a tensor cores
// (tcgen05.mma, tensor memory, tiled TMA).
//
// Replaces the reference's WMMA prefill (gb10-attn kernels/paged_attn_wmma.cu:
// 36-210: one warp per 16 queries x one page, P rounded to half, O rescaled
// through shared memory) with a B200 design:
//
//   * CTA = 128 query rows x one head.  KV tiles of 128 keys = 8 pages of 16
//     tokens, loaded by one producer warp with 3-D tiled TMA (box = 16 rows x
//     64 head-dim elements of one KV head, 128-byte swizzle) into a ring of
//     K/V stages -- the block table turns each 16-row group into a row
//     coordinate, so the page gather costs no extra pass.
//   * S = Q K^T accumulates in TMEM (double-buffered, 2 x 128 columns) from one
//     elected thread's tcgen05.mma (A = Q from shared memory, B = K from
//     shared memory, M = 128, N = 128, K = 16 per instruction).
//   * Four softmax warps (thread = query row = TMEM lane) read S with
//     tcgen05.ld, apply the causal rule of paged_attn_prefill.cu:62-65, keep
//     the running max / sum in fp32, and write P back into the S columns of
//     TMEM; O += P V then takes A = P straight from TMEM (no shared-memory
//     round trip) and B = V from shared memory (MN-major), O in TMEM.
//   * Rescaling of O is lazy: the reference max only moves when a row's max
//     grows by more than 2^8, so O (in TMEM) is rarely touched; the result is
//     exact because the final division uses the same reference max.
//   * Precision: A and B of one kind::f16 MMA share a type.  For bf16 pools Q
//     and P are split into bf16 hi + lo parts (two MMAs each): plain bf16 Q
//     and P measured 2.7-4.0e-3 max-abs against the fp32 oracle, over the
//     2e-3 bar; the split gives ~1e-5.  fp16 pools use single fp16 MMAs.
//
// Every wait is bounded; on a timeout the CTA reports PA_DEVERR_TIMEOUT, stops
// issuing work, and still frees its tensor memory before it exits.
#include <cudaTypedefs.h>

#include <algorithm>
#include <mutex>
#include <vector>

#include "common.cuh"
#include "decode_host.h"
#include "tcgen05.cuh"

namespace pa {
namespace prefill {

constexpr int BM = 128;  // query rows per CTA
constexpr int BN = 128;  // keys per KV tile
constexpr int kSoftmaxWarps = 8;  // two per TMEM lane quadrant
constexpr int kMmaWarp = 8;
constexpr int kTmaWarp = 9;
constexpr int kThreads = 320;
constexpr uint32_t kTmemCols = 512;

struct Params {
  CUtensorMap tmap_k;  // 3-D [D, HKV, NB*BS] views of the pool, box {64, 1, 16}
  CUtensorMap tmap_v;
  float* out;                    // [B, Sq, H, D]
  const float* q;                // [B, Sq, H, D]
  const int32_t* block_tables;   // [B, MB]
  const int32_t* context_lens;   // [B]
  int32_t* dev_status;
  int64_t B, Sq, H, HKV, MB, NB, BS;
  int32_t n_qtiles;
  float qscale;                  // scale * log2(e)
};

template <typename T>
struct Fmt;
template <> struct Fmt<__nv_bfloat16> { static constexpr int id = 1; static constexpr bool split = true; };
template <> struct Fmt<__half> { static constexpr int id = 0; static constexpr bool split = false; };

template <typename T, int D>
struct Cfg {
  static constexpr bool SPLIT = Fmt<T>::split;
  static constexpr int NH = D / 64;                 // 64-element (128-byte) column halves
  static constexpr uint32_t Q_BYTES = BM * D * 2;   // one Q part
  static constexpr uint32_t KV_BYTES = BN * D * 2;  // K or V of one tile
  // K stages are freed as soon as S = Q K^T is done, V stages after P V, so
  // the K ring runs one tile deeper.
  static constexpr int NK = D == 128 ? 3 : 4;
  static constexpr int NV = D == 128 ? 2 : 4;
  static constexpr uint32_t OFF_QH = 0;
  static constexpr uint32_t OFF_QL = Q_BYTES;
  static constexpr uint32_t OFF_K = Q_BYTES * (SPLIT ? 2 : 1);
  static constexpr uint32_t OFF_V = OFF_K + NK * KV_BYTES;
  static constexpr uint32_t OFF_BAR = OFF_V + NV * KV_BYTES;
  static constexpr uint32_t SMEM = OFF_BAR + 192 + 1024;  // + barriers + alignment slack
  static_assert(SMEM <= 227 * 1024, "shared memory budget");
  // TMEM columns: S buffers at 0 and 128, O at 256, row-max / sum exchange
  // slots of the softmax warp pairs at 384..387
  static constexpr uint32_t COL_S0 = 0, COL_S1 = 128, COL_O = 256, COL_X = 384;
};

__device__ __forceinline__ uint32_t pack2(float lo, float hi, __nv_bfloat16*) {
  uint32_t r;
  asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
  return r;
}
__device__ __forceinline__ uint32_t pack2(float lo, float hi, __half*) {
  uint32_t r;
  asm("cvt.rn.f16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
  return r;
}
__device__ __forceinline__ float unpack_lo(uint32_t u, __nv_bfloat16*) { return __uint_as_float(u << 16); }
__device__ __forceinline__ float unpack_hi(uint32_t u, __nv_bfloat16*) { return __uint_as_float(u & 0xffff0000u); }
__device__ __forceinline__ float unpack_lo(uint32_t u, __half*) {
  return __half2float(__ushort_as_half((unsigned short)(u & 0xffffu)));
}
__device__ __forceinline__ float unpack_hi(uint32_t u, __half*) {
  return __half2float(__ushort_as_half((unsigned short)(u >> 16)));
}

// Two fp32 values -> packed 16-bit pair (first value in the low half).  For
// bf16 also the remainder pair: hi = the fp32 bits truncated to bf16 (exact),
// lo = round-to-nearest bf16 of the exact fp32 remainder x - hi, so hi + lo
// carries x to ~2^-16 relative.  fp16: one round-to-nearest pair, lo unused.
__device__ __forceinline__ void split_pair(float a, float b, uint32_t& hi, uint32_t& lo,
                                           __nv_bfloat16*) {
  const uint32_t ua = __float_as_uint(a), ub = __float_as_uint(b);
  hi = __byte_perm(ua, ub, 0x7632);
  const float ra = a - __uint_as_float(ua & 0xffff0000u);
  const float rb = b - __uint_as_float(ub & 0xffff0000u);
  lo = pack2(ra, rb, (__nv_bfloat16*)nullptr);
}
__device__ __forceinline__ void split_pair(float a, float b, uint32_t& hi, uint32_t& lo, __half*) {
  hi = pack2(a, b, (__half*)nullptr);
  lo = 0;
}

// Byte offset of element (r, k) of a [rows x D] K-major tile stored as D/64
// swizzled 128-byte-row halves of `rows * 128` bytes each (the layout the
// tensor core reads with a SWIZZLE_128B descriptor, and TMA writes).
__device__ __forceinline__ uint32_t sw128_offset(int r, int k, int rows) {
  const int half = k >> 6, kk = k & 63, chunk = kk >> 3;
  return (uint32_t)(half * rows * 128 + (r >> 3) * 1024 + (r & 7) * 128 +
                    ((chunk ^ (r & 7)) << 4) + (kk & 7) * 2);
}

// Warp-uniform bounded wait: lane 0 waits, the verdict is broadcast, then
// every lane observes the completed phase itself (acquire).  The warp never
// diverges around the .sync.aligned tcgen05 loads / stores that follow.
__device__ __forceinline__ bool warp_wait(uint64_t* bar, uint32_t parity, int32_t* abort_flag) {
  int ok = 1;
  if ((threadIdx.x & 31) == 0) ok = mbar_wait(bar, parity, abort_flag) ? 1 : 0;
  ok = __shfl_sync(0xffffffffu, ok, 0);
  if (ok) (void)mbar_wait(bar, parity, abort_flag);
  return ok != 0;
}

template <typename T, int D>
__global__ void __launch_bounds__(kThreads, 1) prefill_tc_kernel(const __grid_constant__ Params p) {
  using C = Cfg<T, D>;
  constexpr int NK = C::NK, NV = C::NV;
  extern __shared__ unsigned char smem_raw[];
  // 1024-byte alignment for the 128-byte-swizzle atoms
  unsigned char* smem = smem_raw + ((1024 - (smem_u32(smem_raw) & 1023)) & 1023);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + C::OFF_BAR);
  uint64_t* k_full = bars;               // [NK] K tile landed
  uint64_t* k_empty = k_full + NK;       // [NK] S = Q K^T done with it
  uint64_t* v_full = k_empty + NK;       // [NV] V tile landed
  uint64_t* v_empty = v_full + NV;       // [NV] P V done with it
  uint64_t* s_full = v_empty + NV;       // [2] S tile in TMEM
  uint64_t* p_full = s_full + 2;         // [2] P written to TMEM (softmax warps)
  uint64_t* o_ready = p_full + 2;        // PV of a tile done
  uint64_t* q_ready = o_ready + 1;       // Q in shared memory (softmax warps)
  uint64_t* pair_bar = q_ready + 1;     // [4] max / sum exchange of a warp pair (64 threads)
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(pair_bar + 4);
  int32_t* abort_s = reinterpret_cast<int32_t*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  // Consecutive CTAs take the query tiles of one (sequence, head), longest
  // first: the CTAs resident together share that head's K/V in L2.
  const int64_t c = blockIdx.x;
  const int qt = p.n_qtiles - 1 - (int)(c % p.n_qtiles);
  const int64_t bh = c / p.n_qtiles;
  const int64_t b = bh / p.H, h = bh % p.H;
  const int64_t kv_h = h / (p.H / p.HKV);
  const int64_t q0 = (int64_t)qt * BM;

  if (threadIdx.x == 0) {
    for (int s = 0; s < NK; ++s) {
      mbar_init(&k_full[s], 1);
      mbar_init(&k_empty[s], 1);
    }
    for (int s = 0; s < NV; ++s) {
      mbar_init(&v_full[s], 1);
      mbar_init(&v_empty[s], 1);
    }
    for (int s = 0; s < 2; ++s) {
      mbar_init(&s_full[s], 1);
      mbar_init(&p_full[s], kSoftmaxWarps * 32);
    }
    mbar_init(o_ready, 1);
    mbar_init(q_ready, kSoftmaxWarps * 32);
    for (int qd = 0; qd < 4; ++qd) mbar_init(&pair_bar[qd], 64);
    *abort_s = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == kMmaWarp) {
    tc::tmem_alloc(tmem_slot, kTmemCols);
    tc::tmem_relinquish();
  }
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
  const uint32_t tmem = *tmem_slot;

  // keys this tile of queries needs: [0, min(ctx, ctx - Sq + q_last + 1))
  int64_t ctx = p.context_lens[b];
  const int64_t max_ctx = p.MB * p.BS;
  if (ctx > max_ctx) {
    if (threadIdx.x == 0) report(p.dev_status, PA_DEVERR_CONTEXT);
    ctx = max_ctx;
  }
  const int64_t q_last = min(q0 + BM, p.Sq) - 1;
  const int64_t key_end = min(ctx, ctx - p.Sq + q_last + 1);
  const int n_tiles = key_end > 0 ? (int)((key_end + BN - 1) / BN) : 0;

  if (warp < kSoftmaxWarps) {
    // ------------------------------------------------------------------ softmax
    // Warp w serves query rows 32 * (w % 4) .. +31 (its TMEM lane quadrant) and
    // key columns 64 * (w / 4) .. +63 of each S tile; the two warps of a
    // quadrant share each row's max through shared memory.
    const int quad = warp & 3, ch = warp >> 2;
    const int r = quad * 32 + lane;  // query row in the tile = TMEM lane
    const int64_t qrow = q0 + r;
    const bool row_valid = qrow < p.Sq;
    const int64_t q_abs = ctx - p.Sq + qrow;  // absolute position of this query
    // Q tile -> shared memory, pre-scaled, hi (+ lo) parts, swizzled: warp w
    // converts rows 16w .. 16w+15.
    {
      unsigned char* qh = smem + C::OFF_QH;
      unsigned char* ql = smem + C::OFF_QL;
      constexpr int EPT = D / 32;  // elements per lane per row
#pragma unroll
      for (int i = 0; i < BM / kSoftmaxWarps; ++i) {
        const int rr = warp * (BM / kSoftmaxWarps) + i;
        const int64_t qr = q0 + rr;
        float x[EPT];
        if (qr < p.Sq) {
          const float* src = p.q + ((b * p.Sq + qr) * p.H + h) * D + lane * EPT;
#pragma unroll
          for (int e = 0; e < EPT; e += 2) {
            const float2 v = *reinterpret_cast<const float2*>(src + e);
            x[e] = v.x * p.qscale;
            x[e + 1] = v.y * p.qscale;
          }
        } else {
#pragma unroll
          for (int e = 0; e < EPT; ++e) x[e] = 0.f;
        }
#pragma unroll
        for (int e = 0; e < EPT; e += 2) {
          const uint32_t off = sw128_offset(rr, lane * EPT + e, BM);
          uint32_t hi, lo;
          split_pair(x[e], x[e + 1], hi, lo, (T*)nullptr);
          *reinterpret_cast<uint32_t*>(qh + off) = hi;
          if constexpr (C::SPLIT) *reinterpret_cast<uint32_t*>(ql + off) = lo;
        }
      }
      tc::fence_proxy_async_smem();
      mbar_arrive(q_ready);
    }

    constexpr int HC = BN / 2;  // key columns per warp
    const uint32_t lane_base = tmem + ((uint32_t)(quad * 32) << 16);
    float m_ref = -INFINITY, l = 0.f;
    bool ok = true;
    for (int j = 0; j < n_tiles && ok; ++j) {
      if (!warp_wait(&s_full[j & 1], (j >> 1) & 1, abort_s)) { ok = false; break; }
      tc::fence_after_sync();
      const uint32_t scol = ((j & 1) ? C::COL_S1 : C::COL_S0);
      float s[HC];
#pragma unroll
      for (int c4 = 0; c4 < HC / 32; ++c4) {
        uint32_t u[32];
        tc::tmem_ld32(lane_base + scol + ch * HC + 32 * c4, u);
        tc::tmem_wait_ld();
#pragma unroll
        for (int i = 0; i < 32; ++i) s[32 * c4 + i] = __uint_as_float(u[i]);
      }
      // causal rule + context bound (kernels/paged_attn_prefill.cu:62-65):
      // this warp's keys k0 + c, c < HC, are visible when c < lim
      const int64_t k0 = (int64_t)j * BN + ch * HC;
      const int64_t vis = row_valid ? min(q_abs + 1, ctx) - k0 : 0;
      const int lim = vis <= 0 ? 0 : (vis >= HC ? HC : (int)vis);
      float mt = -INFINITY;
#pragma unroll
      for (int i = 0; i < HC; ++i) {
        s[i] = (i < lim) ? s[i] : -INFINITY;
        mt = fmaxf(mt, s[i]);
      }
      // row max over both column halves, exchanged through TMEM slot j & 1 (a
      // warp is at most one tile ahead of its partner, so the slots alternate)
      tc::tmem_st1(lane_base + C::COL_X + 2 * (j & 1) + ch, __float_as_uint(mt));
      tc::tmem_wait_st();
      tc::fence_before_sync();
      mbar_arrive(&pair_bar[quad]);
      if (!warp_wait(&pair_bar[quad], j & 1, abort_s)) { ok = false; break; }
      tc::fence_after_sync();
      {
        const uint32_t other = tc::tmem_ld1(lane_base + C::COL_X + 2 * (j & 1) + (ch ^ 1));
        tc::tmem_wait_ld();
        mt = fmaxf(mt, __uint_as_float(other));
      }
      // The reference max of a row moves only when the row's max grows by more
      // than 2^8 (then O and l are rescaled); the O rescale is done by the
      // whole warp (tcgen05.ld/st are warp-collective) on its half of O's
      // columns, factor 1 for rows that keep their reference.
      const bool need = mt > m_ref + 8.f;
      const float factor = need ? fast_exp2(m_ref - mt) : 1.f;  // 0 on a row's first visible tile
      if (__any_sync(0xffffffffu, need) && j > 0) {
        if (!warp_wait(o_ready, (j - 1) & 1, abort_s)) { ok = false; break; }
        tc::fence_after_sync();
#pragma unroll
        for (int c4 = 0; c4 < D / 64; ++c4) {
          uint32_t u[32];
          const uint32_t col = lane_base + C::COL_O + ch * (D / 2) + 32 * c4;
          tc::tmem_ld32(col, u);
          tc::tmem_wait_ld();
#pragma unroll
          for (int i = 0; i < 32; ++i) u[i] = __float_as_uint(__uint_as_float(u[i]) * factor);
          tc::tmem_st32(col, u);
        }
        tc::tmem_wait_st();
      }
      if (need) {
        l *= factor;
        m_ref = mt;
      }
      float lsum = 0.f;
#pragma unroll
      for (int i = 0; i < HC; ++i) {
        const float e = (i < lim) ? fast_exp2(s[i] - m_ref) : 0.f;
        s[i] = e;
        lsum += e;
      }
      l += lsum;
      // Keys of this tile past the context (tail of the last page) get P = 0,
      // but 0 * NaN is NaN: zero their V rows in the stage before P V runs
      // (an unwritten pool row may hold anything).  The warp pair of quadrant
      // q zeroes rows 32q .. 32q+31, each warp half of every row.
      {
        const int64_t vr = (int64_t)j * BN + r;
        if (vr >= ctx) {
          unsigned char* vrow = smem + C::OFF_V + (j % NV) * C::KV_BYTES +
                                (r >> 3) * 1024 + (r & 7) * 128;
#pragma unroll
          for (int hf = 0; hf < C::NH; ++hf)
#pragma unroll
            for (int c16 = ch * 4; c16 < ch * 4 + 4; ++c16)
              *reinterpret_cast<uint4*>(vrow + hf * (BN * 128) + c16 * 16) = make_uint4(0, 0, 0, 0);
          tc::fence_proxy_async_smem();
        }
      }
      // P into the S columns: column c of the S buffer holds keys 2c (low half)
      // and 2c+1; P hi in columns [0, 64), P lo in [64, 128).
      {
        uint32_t uh[32], ul[32];
#pragma unroll
        for (int i = 0; i < 32; ++i) split_pair(s[2 * i], s[2 * i + 1], uh[i], ul[i], (T*)nullptr);
        tc::tmem_st32(lane_base + scol + ch * 32, uh);
        if constexpr (C::SPLIT) tc::tmem_st32(lane_base + scol + BN / 2 + ch * 32, ul);
      }
      tc::tmem_wait_st();
      tc::fence_before_sync();
      mbar_arrive(&p_full[j & 1]);
    }

    // epilogue: O / l -> out (this warp's half of the columns); the pair's
    // partial sums meet through slot n_tiles & 1 (phase n_tiles of pair_bar)
    if (ok) {
      tc::tmem_st1(lane_base + C::COL_X + 2 * (n_tiles & 1) + ch, __float_as_uint(l));
      tc::tmem_wait_st();
      tc::fence_before_sync();
      mbar_arrive(&pair_bar[quad]);
      if (warp_wait(&pair_bar[quad], n_tiles & 1, abort_s)) {
        tc::fence_after_sync();
        const uint32_t other = tc::tmem_ld1(lane_base + C::COL_X + 2 * (n_tiles & 1) + (ch ^ 1));
        tc::tmem_wait_ld();
        l += __uint_as_float(other);
      } else {
        ok = false;
      }
    }
    constexpr int HD = D / 2;
    float o[HD];
#pragma unroll
    for (int i = 0; i < HD; ++i) o[i] = 0.f;
    if (ok && n_tiles > 0) {
      if (warp_wait(o_ready, (n_tiles - 1) & 1, abort_s)) {
        tc::fence_after_sync();
#pragma unroll
        for (int c4 = 0; c4 < HD / 32; ++c4) {
          uint32_t u[32];
          tc::tmem_ld32(lane_base + C::COL_O + ch * HD + 32 * c4, u);
          tc::tmem_wait_ld();
#pragma unroll
          for (int i = 0; i < 32; ++i) o[32 * c4 + i] = __uint_as_float(u[i]);
        }
        const float inv = l > 0.f ? 1.f / l : 0.f;
#pragma unroll
        for (int i = 0; i < HD; ++i) o[i] *= inv;
      } else {
        ok = false;
      }
    }
    if (row_valid) {
      float* dst = p.out + ((b * p.Sq + qrow) * p.H + h) * D + ch * HD;
#pragma unroll
      for (int i = 0; i < HD; i += 4)
        *reinterpret_cast<float4*>(dst + i) = make_float4(o[i], o[i + 1], o[i + 2], o[i + 3]);
    }
    if (!ok && lane == 0) report(p.dev_status, PA_DEVERR_TIMEOUT);
  } else if (warp == kMmaWarp) {
    // ------------------------------------------------------------- MMA issuer
    if (lane == 0 && n_tiles > 0) {
      constexpr uint32_t idesc_s = tc::idesc_f16(Fmt<T>::id, BM, BN, false);
      constexpr uint32_t idesc_o = tc::idesc_f16(Fmt<T>::id, BM, D, true);
      const uint32_t qh = smem_u32(smem + C::OFF_QH), ql = smem_u32(smem + C::OFF_QL);
      bool ok = mbar_wait(q_ready, 0, abort_s);
      tc::fence_after_sync();
      auto issue_s = [&](int jj) -> bool {
        const int st = jj % NK;
        if (!mbar_wait(&k_full[st], (jj / NK) & 1, abort_s)) return false;
        tc::fence_after_sync();
        const uint32_t kb = smem_u32(smem + C::OFF_K + st * C::KV_BYTES);
        const uint32_t dcol = tmem + ((jj & 1) ? C::COL_S1 : C::COL_S0);
#pragma unroll
        for (int part = 0; part < (C::SPLIT ? 2 : 1); ++part) {
          const uint32_t qb = part ? ql : qh;
#pragma unroll
          for (int kk = 0; kk < D / 16; ++kk) {
            const uint32_t koff = (kk >> 2) * (BN * 128) + (kk & 3) * 32;
            const uint32_t qoff = (kk >> 2) * (BM * 128) + (kk & 3) * 32;
            tc::mma_ss(dcol, tc::smem_desc_sw128(qb + qoff, 16, 1024),
                       tc::smem_desc_sw128(kb + koff, 16, 1024), idesc_s, (part | kk) != 0);
          }
        }
        tc::mma_commit(&s_full[jj & 1]);
        tc::mma_commit(&k_empty[st]);
        return true;
      };
      if (ok) ok = issue_s(0);
      for (int j = 0; j < n_tiles && ok; ++j) {
        if (j + 1 < n_tiles && !issue_s(j + 1)) { ok = false; break; }
        if (!mbar_wait(&p_full[j & 1], (j >> 1) & 1, abort_s)) { ok = false; break; }
        const int vs = j % NV;
        if (!mbar_wait(&v_full[vs], (j / NV) & 1, abort_s)) { ok = false; break; }
        tc::fence_after_sync();
        const uint32_t vb = smem_u32(smem + C::OFF_V + vs * C::KV_BYTES);
        const uint32_t pcol = tmem + ((j & 1) ? C::COL_S1 : C::COL_S0);
#pragma unroll
        for (int part = 0; part < (C::SPLIT ? 2 : 1); ++part) {
#pragma unroll
          for (int kk = 0; kk < BN / 16; ++kk) {
            tc::mma_ts(tmem + C::COL_O, pcol + part * (BN / 2) + kk * 8,
                       tc::smem_desc_sw128(vb + kk * 16 * 128, BN * 128, 1024), idesc_o,
                       (j > 0 || part > 0 || kk > 0) ? 1u : 0u);
          }
        }
        tc::mma_commit(&v_empty[vs]);
        tc::mma_commit(o_ready);
      }
      if (!ok) report(p.dev_status, PA_DEVERR_TIMEOUT);
    }
  } else if (warp == kTmaWarp) {
    // ------------------------------------------------------------- TMA producer
    // Lane l < 8 * NH loads one 16-row group x 64-column half of the K tile
    // (then of the V tile); the K tile of j runs up to NK tiles ahead, the V
    // tile up to NV.  Block ids are read one tile ahead of their use.
    constexpr int NBOX = 8 * C::NH;
    const int g16 = lane / C::NH;
    const int hf = lane % C::NH;
    const int32_t* bt = p.block_tables + b * p.MB;
    auto group_row = [&](int j) -> int32_t {
      if (lane >= NBOX || j >= n_tiles) return 0;
      const int64_t t = (int64_t)j * BN + g16 * 16;  // first token of the group
      const int64_t pg = t / p.BS;
      int64_t blk = (t < ctx && pg < p.MB) ? bt[pg] : bt[0];
      if (blk < 0 || blk >= p.NB) {
        report(p.dev_status, PA_DEVERR_BLOCK_ID);
        blk = 0;
      }
      return (int32_t)(blk * p.BS + (t - pg * p.BS));
    };
    auto load = [&](bool is_v, int j, int32_t row) -> bool {
      const int st = is_v ? j % NV : j % NK;
      const int n = is_v ? NV : NK;
      uint64_t* empty = is_v ? &v_empty[st] : &k_empty[st];
      uint64_t* full = is_v ? &v_full[st] : &k_full[st];
      if (!warp_wait(empty, ((j / n) & 1) ^ 1, abort_s)) return false;
      if (lane == 0) mbar_arrive_expect_tx(full, C::KV_BYTES);
      __syncwarp();
      if (lane < NBOX) {
        unsigned char* dst = smem + (is_v ? C::OFF_V : C::OFF_K) + st * C::KV_BYTES +
                             hf * (BN * 128) + g16 * 16 * 128;
        tc::tma_load_3d(dst, is_v ? &p.tmap_v : &p.tmap_k, hf * 64, (int32_t)kv_h, row, full);
      }
      return true;
    };
    // K runs NK - NV tiles ahead of V: issue order K0..K(d-1), then (K j+d, V j)
    constexpr int AHEAD = NK - NV;
    int32_t rows_k[AHEAD + 1];
    bool ok = true;
    for (int j = 0; j < AHEAD && j < n_tiles && ok; ++j) ok = load(false, j, group_row(j));
    for (int j = 0; j < n_tiles && ok; ++j) {
      const int jk = j + AHEAD;
      if (jk < n_tiles) ok = load(false, jk, group_row(jk));
      if (ok) ok = load(true, j, group_row(j));
    }
    (void)rows_k;
    if (!ok && lane == 0) report(p.dev_status, PA_DEVERR_TIMEOUT);
  }

  tc::fence_before_sync();
  __syncthreads();
  if (warp == kMmaWarp) {
    tc::fence_after_sync();
    tc::tmem_dealloc(tmem, kTmemCols);
  }
}

// ---------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------

static PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  });
  return fn;
}

static int make_map(CUtensorMap* m, const void* base, int dtype, int64_t D, int64_t HKV,
                    int64_t rows) {
  auto fn = encode_fn();
  if (!fn) return PA_ERR_CUDA;
  const cuuint64_t dims[3] = {(cuuint64_t)D, (cuuint64_t)HKV, (cuuint64_t)rows};
  const cuuint64_t strides[2] = {(cuuint64_t)(D * 2), (cuuint64_t)(HKV * D * 2)};
  const cuuint32_t box[3] = {64, 1, 16};
  const cuuint32_t estr[3] = {1, 1, 1};
  const CUresult r = fn(m, dtype == PA_DTYPE_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16
                                                   : CU_TENSOR_MAP_DATA_TYPE_FLOAT16,
                        3, const_cast<void*>(base), dims, strides, box, estr,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                        CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? PA_OK : PA_ERR_CUDA;
}

template <typename T, int D>
static int launch_typed(const Params& p, int64_t grid, cudaStream_t s) {
  using C = Cfg<T, D>;
  auto kern = prefill_tc_kernel<T, D>;
  static std::mutex mu;
  static std::vector<int> done;
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_status(e);
  {
    std::lock_guard<std::mutex> lk(mu);
    if (std::find(done.begin(), done.end(), dev) == done.end()) {
      e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM);
      if (e != cudaSuccess) return cuda_status(e);
      done.push_back(dev);
    }
  }
  kern<<<(unsigned)grid, kThreads, C::SMEM, s>>>(p);
  return cuda_status(cudaGetLastError());
}

// True when the tensor-core path handles these arguments.
bool tc_eligible(int dtype, int64_t D, int64_t BS, int64_t NB) {
  return (dtype == PA_DTYPE_F16 || dtype == PA_DTYPE_BF16) && (D == 64 || D == 128) &&
         BS % 16 == 0 && NB * BS <= (int64_t(1) << 31) - 1;
}

int launch_tc(float* out, const float* q, const void* k, const void* v, int dtype,
              const int32_t* bt, const int32_t* ctx, int64_t B, int64_t Sq, int64_t H,
              int64_t HKV, int64_t D, int64_t BS, int64_t NB, int64_t MB, double scale,
              int32_t* dev_status, cudaStream_t s) {
  if (!out || !q || !k || !v || !bt || !ctx) return PA_ERR_INVALID_ARGUMENT;
  if (!aligned16(k) || !aligned16(v) || !aligned16(q) || !aligned16(out)) return PA_ERR_ALIGNMENT;
  int sms = 0;
  if (device_sm_count(&sms) != PA_OK) return PA_ERR_NO_DEVICE;
  Params p;
  int st = make_map(&p.tmap_k, k, dtype, D, HKV, NB * BS);
  if (st) return st;
  st = make_map(&p.tmap_v, v, dtype, D, HKV, NB * BS);
  if (st) return st;
  p.out = out;
  p.q = q;
  p.block_tables = bt;
  p.context_lens = ctx;
  p.dev_status = dev_status;
  p.B = B;
  p.Sq = Sq;
  p.H = H;
  p.HKV = HKV;
  p.MB = MB;
  p.NB = NB;
  p.BS = BS;
  p.n_qtiles = (int32_t)((Sq + BM - 1) / BM);
  p.qscale = (float)scale * kLog2e;
  const int64_t grid = (int64_t)p.n_qtiles * B * H;
  if (grid <= 0) return PA_OK;
  if (grid > (int64_t(1) << 31) - 1) return PA_ERR_TOO_LARGE;
  if (dtype == PA_DTYPE_BF16)
    return D == 128 ? launch_typed<__nv_bfloat16, 128>(p, grid, s)
                    : launch_typed<__nv_bfloat16, 64>(p, grid, s);
  return D == 128 ? launch_typed<__half, 128>(p, grid, s) : launch_typed<__half, 64>(p, grid, s);
}

}  // namespace prefill
}  // namespace pa
