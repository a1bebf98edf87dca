// prefill_tc.cu -- causal paged prefill on the sm_100a tensor cores
// (tcgen05.mma, tensor memory, tiled TMA).
//
// Replaces the reference's WMMA prefill (gb10-attn kernels/paged_attn_wmma.cu:
// 36-210: one warp per 16 queries x one page, P rounded to half, O rescaled
// through shared memory) with a B200 design:
//
//   * CTA = 128 query rows x one head.  KV tiles of 128 keys = 8 pages of 16
//     tokens, loaded by one producer warp with 3-D tiled TMA (box = 16 rows x
//     64 head-dim elements of one KV head, 128-byte swizzle) into separate K
//     and V rings (a K stage is freed once S = Q K^T is done, so the K ring
//     runs a tile deeper) -- the block table, staged in shared memory, turns
//     each 16-row group into a row coordinate, so the page gather costs no
//     extra pass.
//   * S = Q K^T accumulates in TMEM (double-buffered, 2 x 128 columns) from one
//     elected thread's tcgen05.mma (A = Q from shared memory, B = K from
//     shared memory, M = 128, N = 128, K = 16 per instruction).
//   * Two softmax warpgroups alternate over the KV tiles (ping-pong): group g
//     takes tiles j % 2 == g, so one group's exponentials overlap the other's
//     MMAs.  Thread = query row = TMEM lane: it reads S with tcgen05.ld,
//     applies the causal rule of paged_attn_prefill.cu:62-65, keeps its
//     group's running max / sum in fp32, and writes P back into the S columns
//     of TMEM; O_g += P V then takes A = P straight from TMEM (no shared-memory
//     round trip) and B = V from shared memory (MN-major), with one O
//     accumulator per group in TMEM.  The epilogue merges the two groups'
//     (max, sum, O) with the log-sum-exp rule.
//   * Rescaling of O is lazy: the reference max only moves when a row's max
//     grows by more than 2^8, so O (in TMEM) is rarely touched; the result is
//     exact because the final division uses the same reference max.
//   * Precision: A and B of one kind::f16 MMA share a type.  For bf16 pools Q
//     and P are split into bf16 hi + lo parts (two MMAs each): plain bf16 Q
//     and P measured 2.7-4.0e-3 max-abs against the fp32 oracle, over the
//     2e-3 bar; the split gives ~2e-5.  fp16 pools use single fp16 MMAs.
//   * The softmax runs on packed fp32 pairs (add/fma .f32x2) and builds P's
//     hi / lo parts with integer byte permutes (both truncations; hi + lo
//     still carries P to 2^-16), so exp2 dominates its instruction stream.
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
// Warpgroups 0-1: softmax (warpgroup g takes the KV tiles j % 2 == g);
// warpgroup 2: warp 8 issues the MMAs, warp 9 the TMA loads, warps 10-11 idle.
// Registers: 384 threads launched at 168 (64512); setmaxnreg gives the
// softmax warpgroups 232 and the rest 40: 256 x 232 + 128 x 40 = 64512.
constexpr int kSoftmaxWarps = 8;
constexpr int kMmaWarp = 8;
constexpr int kTmaWarp = 9;
constexpr int kThreads = 384;
constexpr int kSoftmaxRegs = 232, kOtherRegs = 40;
static_assert(256 * kSoftmaxRegs + 128 * kOtherRegs <= kThreads * 168, "register split");
constexpr uint32_t kTmemCols = 512;
// block ids the TMA warp stages in shared memory per refill (32 tiles at 16-token pages)
constexpr int kBtChunk = 256;

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
  // mbarriers: K and V full/empty rings, s_full/p_full/o_ready pairs, q_ready,
  // 4 pair barriers; then the TMEM address and the abort flag
  static constexpr uint32_t N_BARS = 2 * NK + 2 * NV + 2 * 3 + 1 + 4;
  static constexpr uint32_t OFF_BT = OFF_BAR + ((N_BARS * 8 + 8 + 15) / 16) * 16;
  static constexpr uint32_t SMEM = OFF_BT + kBtChunk * 4 + 1024;  // + alignment slack
  static_assert(SMEM <= 227 * 1024, "shared memory budget");
  // TMEM columns: S buffers at 0 and 128 (tiles j % 2), O of the two
  // softmax warpgroups at 256 and 256 + D
  static constexpr uint32_t COL_S0 = 0, COL_S1 = 128, COL_O = 256;
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

// Softmax weights (p0, p1) of two adjacent keys -> the MMA operand pair(s).
// bf16: hi = the fp32 bits truncated to bf16, lo = the remainder p - hi
// (exact in fp32) truncated to bf16; hi + lo carries p to 2^-16 relative,
// with integer byte permutes instead of conversions.  fp16: one
// round-to-nearest pair.
__device__ __forceinline__ void p_pair(float p0, float p1, uint32_t& hi, uint32_t& lo,
                                       __nv_bfloat16*) {
  const uint32_t a = __float_as_uint(p0), b = __float_as_uint(p1);
  hi = __byte_perm(a, b, 0x7632);
  const float2 r = fma2(make_float2(__uint_as_float(a & 0xffff0000u), __uint_as_float(b & 0xffff0000u)),
                        make_float2(-1.f, -1.f), make_float2(p0, p1));
  lo = __byte_perm(__float_as_uint(r.x), __float_as_uint(r.y), 0x7632);
}
__device__ __forceinline__ void p_pair(float p0, float p1, uint32_t& hi, uint32_t& lo, __half*) {
  hi = pack2(p0, p1, (__half*)nullptr);
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
  uint64_t* o_ready = p_full + 2;        // [2] P V of a tile of group j % 2 done
  uint64_t* q_ready = o_ready + 2;       // Q in shared memory (softmax warps)
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
      mbar_init(&p_full[s], 4 * 32);  // one warpgroup per tile
      mbar_init(&o_ready[s], 1);
    }
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
    asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(kSoftmaxRegs));
    // Warp w serves query rows 32 * (w % 4) .. +31 (its TMEM lane quadrant)
    // of the tiles of warpgroup w / 4.
    const int quad = warp & 3;
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
      constexpr int RPW = BM / kSoftmaxWarps;  // rows per warp
      // every row's global load is issued before the first shared store, so
      // the warp waits on global memory once
      float x[RPW][EPT];
#pragma unroll
      for (int i = 0; i < RPW; ++i) {
        const int64_t qr = q0 + warp * RPW + i;
        const float* src = p.q + ((b * p.Sq + qr) * p.H + h) * D + lane * EPT;
        if constexpr (EPT == 4) {
          const float4 v = qr < p.Sq ? __ldg(reinterpret_cast<const float4*>(src)) : make_float4(0.f, 0.f, 0.f, 0.f);
          x[i][0] = v.x, x[i][1] = v.y, x[i][2] = v.z, x[i][3] = v.w;
        } else {
#pragma unroll
          for (int e = 0; e < EPT; e += 2) {
            const float2 v = qr < p.Sq ? __ldg(reinterpret_cast<const float2*>(src + e)) : make_float2(0.f, 0.f);
            x[i][e] = v.x, x[i][e + 1] = v.y;
          }
        }
      }
#pragma unroll
      for (int i = 0; i < RPW; ++i) {
        const int rr = warp * RPW + i;
#pragma unroll
        for (int e = 0; e < EPT; e += 2) {
          const uint32_t off = sw128_offset(rr, lane * EPT + e, BM);
          uint32_t hi, lo;
          split_pair(x[i][e] * p.qscale, x[i][e + 1] * p.qscale, hi, lo, (T*)nullptr);
          *reinterpret_cast<uint32_t*>(qh + off) = hi;
          if constexpr (C::SPLIT) *reinterpret_cast<uint32_t*>(ql + off) = lo;
        }
      }
      tc::fence_proxy_async_smem();
      mbar_arrive(q_ready);
    }

    // Warpgroup g = warp / 4 takes the KV tiles j with j % 2 == g (S buffer
    // g) and keeps, per query row, its own running reference max, sum and O
    // accumulator (TMEM columns COL_O + g * D); the two partial states are
    // merged with the log-sum-exp rule once, after the last tile.  Two tiles'
    // softmax are in flight at a time and no cross-warp reduction sits on the
    // per-tile path.
    const int grp = warp >> 2;
    const uint32_t lane_base = tmem + ((uint32_t)(quad * 32) << 16);
    const uint32_t ocol = C::COL_O + grp * D;
    float m_ref = -INFINITY, l = 0.f;
    bool ok = true;
    int last_j = -1;
    for (int j = grp; j < n_tiles && ok; j += 2) {
      if (!warp_wait(&s_full[grp], (j >> 1) & 1, abort_s)) { ok = false; break; }
      tc::fence_after_sync();
      const uint32_t scol = grp ? C::COL_S1 : C::COL_S0;
      // causal rule + context bound (kernels/paged_attn_prefill.cu:62-65):
      // keys k0 + c of this tile are visible when c < lim
      const int64_t k0 = (int64_t)j * BN;
      const int64_t vis = row_valid ? min(q_abs + 1, ctx) - k0 : 0;
      const int lim = vis <= 0 ? 0 : (vis >= BN ? BN : (int)vis);
      // pass 1: row max over the visible keys (S streamed from TMEM, 32
      // columns at a time); tiles with every key visible to all of the warp's
      // rows skip the per-key mask
      const bool full = __all_sync(0xffffffffu, lim == BN);
      float mt = -INFINITY;
      if (full) {
        float m4[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
#pragma unroll
        for (int c4 = 0; c4 < BN / 32; ++c4) {
          uint32_t u[32];
          tc::tmem_ld32(lane_base + scol + 32 * c4, u);
          tc::tmem_wait_ld();
#pragma unroll
          for (int i = 0; i < 32; ++i) m4[i & 3] = fmaxf(m4[i & 3], __uint_as_float(u[i]));
        }
        mt = fmaxf(fmaxf(m4[0], m4[1]), fmaxf(m4[2], m4[3]));
      } else {
#pragma unroll
        for (int c4 = 0; c4 < BN / 32; ++c4) {
          uint32_t u[32];
          tc::tmem_ld32(lane_base + scol + 32 * c4, u);
          tc::tmem_wait_ld();
#pragma unroll
          for (int i = 0; i < 32; ++i)
            if (32 * c4 + i < lim) mt = fmaxf(mt, __uint_as_float(u[i]));
        }
      }
      // The reference max of a row moves only when the row's max grows by more
      // than 2^8 (then this group's O and l are rescaled); the O rescale is
      // done by the whole warp (tcgen05.ld/st are warp-collective), factor 1
      // for rows that keep their reference.
      const bool need = mt > m_ref + 8.f;
      const float factor = need ? fast_exp2(m_ref - mt) : 1.f;  // 0 on a row's first visible tile
      if (__any_sync(0xffffffffu, need) && j >= 2) {
        // the group's previous P V (tile j - 2) must have finished
        if (!warp_wait(&o_ready[grp], ((j >> 1) - 1) & 1, abort_s)) { ok = false; break; }
        tc::fence_after_sync();
#pragma unroll
        for (int c4 = 0; c4 < D / 32; ++c4) {
          uint32_t u[32];
          tc::tmem_ld32(lane_base + ocol + 32 * c4, u);
          tc::tmem_wait_ld();
#pragma unroll
          for (int i = 0; i < 32; ++i) u[i] = __float_as_uint(__uint_as_float(u[i]) * factor);
          tc::tmem_st32(lane_base + ocol + 32 * c4, u);
        }
        tc::tmem_wait_st();
      }
      if (need) {
        l *= factor;
        m_ref = mt;
      }
      // Keys of this tile past the context (tail of the last page) get P = 0,
      // but 0 * NaN is NaN: zero their V rows in the stage before P V runs
      // (an unwritten pool row may hold anything).  Thread r owns V row r.
      if (k0 + r >= ctx) {
        unsigned char* vrow = smem + C::OFF_V + (j % NV) * C::KV_BYTES + (r >> 3) * 1024 +
                              (r & 7) * 128;
#pragma unroll
        for (int hf = 0; hf < C::NH; ++hf)
#pragma unroll
          for (int c16 = 0; c16 < 8; ++c16)
            *reinterpret_cast<uint4*>(vrow + hf * (BN * 128) + c16 * 16) = make_uint4(0, 0, 0, 0);
        tc::fence_proxy_async_smem();
      }
      // pass 2: P = exp2(s - m_ref) into the S columns, 32 keys at a time
      // (S re-read from TMEM).  Keys 32c .. 32c + 31 go to columns
      // [32c, 32c + 16) as 16-bit pairs (keys 2i, 2i+1 in column 32c + i),
      // their lo parts to [32c + 16, 32c + 32): every store lands on columns
      // this pass has already read.  Masked keys get s = -inf, so P = 0.
      // (a row with no visible key so far has m_ref = -inf and only masked keys here)
      const float mneg = m_ref == -INFINITY ? 0.f : -m_ref;
      const float2 negm = make_float2(mneg, mneg);
      float2 ls = make_float2(0.f, 0.f);
#pragma unroll
      for (int c = 0; c < BN / 32; ++c) {
        uint32_t u[32];
        tc::tmem_ld32(lane_base + scol + 32 * c, u);
        tc::tmem_wait_ld();
        if (!full) {
#pragma unroll
          for (int i = 0; i < 32; ++i)
            if (32 * c + i >= lim) u[i] = __float_as_uint(-INFINITY);
        }
        uint32_t uh[16], ul[16];
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          const float2 x = add2(make_float2(__uint_as_float(u[2 * i]), __uint_as_float(u[2 * i + 1])), negm);
          const float2 e = make_float2(fast_exp2(x.x), fast_exp2(x.y));
          ls = add2(ls, e);
          p_pair(e.x, e.y, uh[i], ul[i], (T*)nullptr);
        }
        tc::tmem_st16(lane_base + scol + 32 * c, uh);
        if constexpr (C::SPLIT) tc::tmem_st16(lane_base + scol + 32 * c + 16, ul);
      }
      const float lsum = ls.x + ls.y;
      l += lsum;
      tc::tmem_wait_st();
      tc::fence_before_sync();
      mbar_arrive(&p_full[grp]);
      last_j = j;
    }

    // epilogue: merge the two groups' (m, l, O) per row, O / l -> out.  Each
    // warp of a pair writes half of the columns.  (m, l) cross through TMEM
    // columns of this group's (now idle) S buffer.
    const uint32_t xcol = grp ? C::COL_S1 : C::COL_S0;
    const uint32_t xcol_other = grp ? C::COL_S0 : C::COL_S1;
    float mo = -INFINITY, lo_ = 0.f;
    bool have_mine = false, have_other = false;
    if (ok) {
      // all of this row's P V products must be complete: wait both groups' last
      const int lj[2] = {n_tiles >= 1 ? ((n_tiles - 1) & ~1) : -1,
                         n_tiles >= 2 ? (((n_tiles - 2) & ~1) | 1) : -1};
      for (int g = 0; g < 2 && ok; ++g)
        if (lj[g] >= 0 && !warp_wait(&o_ready[g], (lj[g] >> 1) & 1, abort_s)) ok = false;
      have_mine = lj[grp] >= 0;
      have_other = lj[grp ^ 1] >= 0;
      (void)last_j;
    }
    if (ok) {
      tc::fence_after_sync();
      uint32_t x[32];
      x[0] = __float_as_uint(m_ref);
      x[1] = __float_as_uint(l);
#pragma unroll
      for (int i = 2; i < 32; ++i) x[i] = 0;
      tc::tmem_st32(lane_base + xcol, x);
      tc::tmem_wait_st();
      tc::fence_before_sync();
      mbar_arrive(&pair_bar[quad]);
      if (warp_wait(&pair_bar[quad], 0, abort_s)) {
        tc::fence_after_sync();
        uint32_t y[32];
        tc::tmem_ld32(lane_base + xcol_other, y);
        tc::tmem_wait_ld();
        mo = __uint_as_float(y[0]);
        lo_ = __uint_as_float(y[1]);
      } else {
        ok = false;
      }
    }
    constexpr int HD = D / 2;
    float o[HD];
#pragma unroll
    for (int i = 0; i < HD; ++i) o[i] = 0.f;
    if (ok) {
      // this warp's output columns [grp * HD, grp * HD + HD) from both O buffers
      const float mA = grp ? mo : m_ref, lA = grp ? lo_ : l;
      const float mB = grp ? m_ref : mo, lB = grp ? l : lo_;
      const bool hasA = grp ? have_other : have_mine, hasB = grp ? have_mine : have_other;
      const float mm = fmaxf(hasA ? mA : -INFINITY, hasB ? mB : -INFINITY);
      const float wA = (hasA && lA > 0.f) ? fast_exp2(mA - mm) : 0.f;
      const float wB = (hasB && lB > 0.f) ? fast_exp2(mB - mm) : 0.f;
      const float L = lA * wA + lB * wB;
      const float inv = L > 0.f ? 1.f / L : 0.f;
#pragma unroll
      for (int c4 = 0; c4 < HD / 32; ++c4) {
        uint32_t ua[32], ub[32];
        tc::tmem_ld32(lane_base + C::COL_O + grp * HD + 32 * c4, ua);
        tc::tmem_ld32(lane_base + C::COL_O + D + grp * HD + 32 * c4, ub);
        tc::tmem_wait_ld();
#pragma unroll
        for (int i = 0; i < 32; ++i) {
          const float a = wA > 0.f ? __uint_as_float(ua[i]) * wA : 0.f;
          const float bb = wB > 0.f ? __uint_as_float(ub[i]) * wB : 0.f;
          o[32 * c4 + i] = (a + bb) * inv;
        }
      }
    }
    if (row_valid) {
      float* dst = p.out + ((b * p.Sq + qrow) * p.H + h) * D + grp * HD;
#pragma unroll
      for (int i = 0; i < HD; i += 4)
        *reinterpret_cast<float4*>(dst + i) = make_float4(o[i], o[i + 1], o[i + 2], o[i + 3]);
    }
    if (!ok && lane == 0) report(p.dev_status, PA_DEVERR_TIMEOUT);
  } else {
   asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(kOtherRegs));
   if (warp == kMmaWarp) {
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
            // keys 16kk .. 16kk + 15: 8 columns of packed pairs
            tc::mma_ts(tmem + C::COL_O + (j & 1) * D, pcol + (kk >> 1) * 32 + (kk & 1) * 8 + part * 16,
                       tc::smem_desc_sw128(vb + kk * 16 * 128, BN * 128, 1024), idesc_o,
                       (j > 1 || part > 0 || kk > 0) ? 1u : 0u);
          }
        }
        tc::mma_commit(&v_empty[vs]);
        tc::mma_commit(&o_ready[j & 1]);
      }
      if (!ok) report(p.dev_status, PA_DEVERR_TIMEOUT);
    }
  } else if (warp == kTmaWarp) {
    // ------------------------------------------------------------- TMA producer
    // Lane l < 8 * NH loads one 16-row group x 64-column half of the K tile
    // (then of the V tile); the K tile of j runs up to NK tiles ahead, the V
    // tile up to NV.  The sequence's block ids are staged in shared memory,
    // kBtChunk pages per coalesced refill, so no dependent global load sits
    // on the per-tile issue path; a tile's rows serve its K and its V load.
    constexpr int NBOX = 8 * C::NH;
    const int g16 = lane / C::NH;
    const int hf = lane % C::NH;
    const int32_t* bt = p.block_tables + b * p.MB;
    int32_t* bt_s = reinterpret_cast<int32_t*>(smem + C::OFF_BT);
    const int64_t n_pages = (ctx + p.BS - 1) / p.BS;  // <= MB (ctx clamped above)
    int64_t chunk0 = -(int64_t)kBtChunk - 1;         // first page held in bt_s
    // warp-uniform: make pages [pg_lo, pg_hi] resident
    auto stage_pages = [&](int64_t pg_lo, int64_t pg_hi) {
      if (pg_lo >= chunk0 && pg_hi < chunk0 + kBtChunk) return;
      chunk0 = pg_lo;
      int32_t v[kBtChunk / 32];
#pragma unroll
      for (int i = 0; i < kBtChunk / 32; ++i) {
        const int64_t pg = chunk0 + i * 32 + lane;
        v[i] = pg < n_pages ? __ldg(bt + pg) : 0;
      }
      __syncwarp();
#pragma unroll
      for (int i = 0; i < kBtChunk / 32; ++i) bt_s[i * 32 + lane] = v[i];
      __syncwarp();
    };
    // pool row of this lane's 16-token group of tile j (row 0 past the context)
    auto group_row = [&](int j) -> int32_t {
      if (j >= n_tiles) return 0;
      const int64_t t0 = (int64_t)j * BN;
      stage_pages(t0 / p.BS, (t0 + BN - 1) / p.BS);
      const int64_t t = t0 + g16 * 16;  // first token of the group
      if (lane >= NBOX || t >= ctx) return 0;
      const int64_t pg = t / p.BS;
      int64_t blk = bt_s[pg - chunk0];
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
    // K runs NK - NV tiles ahead of V: issue order K0..K(d-1), then (K j+d, V j);
    // rows[i] holds the rows of tile j + i
    constexpr int AHEAD = NK - NV;
    int32_t rows[AHEAD + 1];
    bool ok = true;
#pragma unroll
    for (int i = 0; i < AHEAD; ++i) {
      rows[i] = group_row(i);
      if (ok && i < n_tiles) ok = load(false, i, rows[i]);
    }
    for (int j = 0; j < n_tiles && ok; ++j) {
      const int jk = j + AHEAD;
      rows[AHEAD] = group_row(jk);
      if (jk < n_tiles) ok = load(false, jk, rows[AHEAD]);
      if (ok) ok = load(true, j, rows[0]);
#pragma unroll
      for (int i = 0; i < AHEAD; ++i) rows[i] = rows[i + 1];
    }
    if (!ok && lane == 0) report(p.dev_status, PA_DEVERR_TIMEOUT);
   }
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
