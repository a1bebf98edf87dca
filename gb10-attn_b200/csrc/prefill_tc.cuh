// prefill_tc.cuh -- pieces shared by the tensor-core prefill kernels
// (prefill_tc.cu: one CTA per 128 query rows; prefill_pair.cu: a CTA pair
// sharing one M = 256 MMA): launch parameters, tile constants, the Q / P
// operand packing, the 128-byte swizzle and the warp-uniform bounded wait.
#pragma once

#include <cudaTypedefs.h>

#include "common.cuh"
#include "tcgen05.cuh"

namespace pa {
namespace prefill {

constexpr int BM = 128;  // query rows per CTA
constexpr int BN = 128;  // keys per KV tile
// Warpgroups 0-1: softmax (the 1-SM kernel splits each score tile's columns
// between them; the pair kernel gives each its own chain of query rows);
// warpgroup 2: warp 8 issues the MMAs, warps 9-10 the TMA loads.
// Registers: 384 threads launched at 168 (64512); setmaxnreg gives the
// softmax warpgroups 224 and the rest 56: 256 x 224 + 128 x 56 = 64512.
constexpr int kSoftmaxWarps = 8;
constexpr int kMmaWarp = 8;
constexpr int kTmaWarp = 9;
constexpr int kThreads = 384;
constexpr int kSoftmaxRegs = 224, kOtherRegs = 56;
static_assert(256 * kSoftmaxRegs + 128 * kOtherRegs <= kThreads * 168, "register split");
constexpr uint32_t kTmemCols = 512;
// block ids the TMA warp stages in shared memory per refill (32 tiles at 16-token pages)
constexpr int kBtChunk = 256;

struct Params {
  CUtensorMap tmap_k;  // 3-D [D, HKV, NB*BS] views of the pool, box {64, 1, 16}
  CUtensorMap tmap_v;
  float* out;                    // [B, Sq, H, D]
  const float* q;                // [B, Sq, H, D]
  const char* v_pool;            // [NB, BS, HKV, D] (rows past the context: sanitised copies)
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
  static constexpr uint32_t OFF_XCH = OFF_BT + kBtChunk * 4;      // [2][2][128] fp32
  static constexpr uint32_t SMEM = OFF_XCH + 2048 + 1024;          // + alignment slack
  static_assert(SMEM <= 227 * 1024, "shared memory budget");
  // TMEM columns: S buffers at 0 and 128 (tiles j % 2), O at 256
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

// One lane writes one 16-token group x 64-column half of a V tile (the
// 128-byte-swizzled layout TMA produces) for a group that reaches past the
// context: tokens < ctx are copied from the pool rows `row0 + i` (16-byte
// loads), the rest are zeros, so no P = 0 weight meets a NaN or Inf of an
// unwritten pool row.  `dst` is the group's first row in the stage.
__device__ __forceinline__ void v_group_sanitised(unsigned char* dst, const char* v_pool,
                                                  int64_t row0, int64_t valid, int64_t HKV,
                                                  int64_t kv_h, int hf, int64_t D) {
#pragma unroll 1
  for (int i = 0; i < 16; ++i) {
    const uint4* src = reinterpret_cast<const uint4*>(
        v_pool + (((row0 + i) * HKV + kv_h) * D + hf * 64) * 2);
    unsigned char* drow = dst + (i >> 3) * 1024 + (i & 7) * 128;  // group rows start 8-aligned
#pragma unroll
    for (int c = 0; c < 8; ++c) {
      const uint4 v = i < valid ? __ldg(src + c) : make_uint4(0, 0, 0, 0);
      *reinterpret_cast<uint4*>(drow + ((c ^ (i & 7)) << 4)) = v;
    }
  }
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

// Barriers the softmax warps use (this CTA's shared memory).
struct Bars {
  uint64_t* s_full;    // [2] S of tile j in tensor memory, slot j % 2 (MMA commit)
  uint64_t* p_full;    // [2] P of tile j written by both groups (the leader's in a pair)
  uint64_t* o_ready;   // [2] P V of tile j done, slot j % 2 (MMA commit)
  uint64_t* q_ready;   // Q staged (softmax arrivals; the leader's in a pair)
  uint64_t* pair_bar;  // [4] row max / sum exchange of warps w and w + 4 (64 arrivals)
  float* xch;          // [2][2][128] exchange slots (shared memory)
};

// Warp-uniform bounded wait; CL: acquire at cluster scope (barriers another
// CTA of the pair arrives on or commits to).
template <bool CL>
__device__ __forceinline__ bool warp_wait_t(uint64_t* bar, uint32_t parity, int32_t* abort_flag) {
  int ok = 1;
  if ((threadIdx.x & 31) == 0)
    ok = (CL ? mbar_wait_cl(bar, parity, abort_flag) : mbar_wait(bar, parity, abort_flag)) ? 1 : 0;
  ok = __shfl_sync(0xffffffffu, ok, 0);
  if (ok) (void)(CL ? mbar_wait_cl(bar, parity, abort_flag) : mbar_wait(bar, parity, abort_flag));
  return ok != 0;
}

// Warp-uniform bounded wait on a barrier that hands tensor-memory data on
// (mbar_wait_rx: relaxed, cluster scope).
__device__ __forceinline__ bool warp_wait_rx(uint64_t* bar, uint32_t parity, int32_t* abort_flag) {
  int ok = 1;
  if ((threadIdx.x & 31) == 0) ok = mbar_wait_rx(bar, parity, abort_flag) ? 1 : 0;
  ok = __shfl_sync(0xffffffffu, ok, 0);
  if (ok) (void)mbar_wait_rx(bar, parity, abort_flag);
  return ok != 0;
}

// Arrival on a barrier the MMA issuer waits on: this CTA's own, or in a CTA
// pair the leader's (even CTA) through its cluster address, with release at
// cluster scope.
template <bool PAIR>
__device__ __forceinline__ void arrive_to_leader(uint64_t* bar) {
  if constexpr (PAIR)
    tc::mbar_arrive_cluster(tc::mapa_shared(bar, 0));
  else
    mbar_arrive(bar);
}

// Q rows r0 .. r0 + 15 of the 128-row tile starting at query row q0 (sequence
// b, head h) -> shared memory at qh (and the lo parts at ql for bf16 pools):
// pre-scaled by scale * log2(e), 128-byte swizzled.  One warp; every row's
// global load is issued before the first shared store, so the warp waits on
// global memory once.  Returns true if a scaled element is outside the fp16
// range and Q is kept as one fp16 part.
template <typename T, int D, typename C>
__device__ __forceinline__ bool stage_q(const Params& p, unsigned char* qh, unsigned char* ql,
                                        int64_t b, int64_t h, int64_t q0, int r0, int lane) {
  constexpr int EPT = D / 32;  // elements per lane per row
  constexpr int RPW = 16;
  float x[RPW][EPT];
#pragma unroll
  for (int i = 0; i < RPW; ++i) {
    const int64_t qr = q0 + r0 + i;
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
  bool qover = false;
#pragma unroll
  for (int i = 0; i < RPW; ++i) {
    const int rr = r0 + i;
#pragma unroll
    for (int e = 0; e < EPT; e += 2) {
      const uint32_t off = sw128_offset(rr, lane * EPT + e, BM);
      uint32_t hi, lo;
      const float a = x[i][e] * p.qscale, bq = x[i][e + 1] * p.qscale;
      if constexpr (!C::SPLIT) qover |= !(fabsf(a) < 65520.f && fabsf(bq) < 65520.f);
      split_pair(a, bq, hi, lo, (T*)nullptr);
      *reinterpret_cast<uint32_t*>(qh + off) = hi;
      if constexpr (C::SPLIT) *reinterpret_cast<uint32_t*>(ql + off) = lo;
    }
  }
  return qover;
}

// The softmax role of both tensor-core prefill kernels: warps 0-7 of a CTA,
// 128 query rows (rows q0 .. q0 + 127 of sequence b, head h) against the
// n_tiles KV tiles of 128 keys.  Stages Q (pre-scaled, hi / lo parts) in
// shared memory, turns each S tile of its warpgroup into P in tensor memory,
// and writes O / l to `out` in the epilogue.  Step j of the KV loop holds
// KV tile (j + rot) % n_tiles (the online softmax does not depend on the
// order).  C supplies the shared-memory
// and tensor-memory offsets; PAIR: the CTA is one of a cta_group::2 pair
// whose leader issues the MMAs.
template <typename T, int D, typename C, bool PAIR>
__device__ __forceinline__ void softmax_role(const Params& p, unsigned char* smem, uint32_t tmem,
                                             Bars bars, int32_t* abort_s, int warp, int lane,
                                             int64_t b, int64_t h, int64_t q0, int64_t ctx,
                                             int n_tiles, int rot) {
  uint64_t* s_full = bars.s_full;
  uint64_t* p_full = bars.p_full;
  uint64_t* o_ready = bars.o_ready;
  uint64_t* q_ready = bars.q_ready;
  uint64_t* pair_bar = bars.pair_bar;
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
    const bool qover = stage_q<T, D, C>(p, smem + C::OFF_QH, smem + C::OFF_QL, b, h, q0,
                                        warp * 16, lane);
    if (qover) report(p.dev_status, PA_DEVERR_RANGE);
    tc::fence_proxy_async_smem();
    arrive_to_leader<PAIR>(q_ready);
  }

  // Both warpgroups work on every KV tile: group g = warp / 4 takes columns
  // [64 g, 64 g + 64) of the S tile for the 128 query rows (warps w and w + 4
  // hold the same rows, TMEM lane quadrant w % 4).  Per tile the two halves'
  // row maxima meet through shared memory (xch, two slots, pair_bar[quad]
  // bounded barrier), both groups then share one reference max per row, each
  // writes P of its 64 keys and keeps its half of the row sum; O is one
  // accumulator of which group g rescales columns [g D / 2, (g + 1) D / 2).
  // The MMA issuer computes S of tile j + 1 while tile j's softmax runs.
  const int grp = warp >> 2;
  const uint32_t lane_base = tmem + ((uint32_t)(quad * 32) << 16);
  constexpr int HD = D / 2;  // O columns per group
  const uint32_t ocol = C::COL_O + grp * HD;
  float* xch = bars.xch;     // [2 slots][2 groups][128 rows]
  float m_ref = -INFINITY, l = 0.f;  // l: this group's half of the row sum
  bool ok = true;
  uint32_t xuses = 0;        // phases of pair_bar[quad] used so far
  auto exchange = [&](float mine) -> float {  // the partner half's value of this row
    float* xs = xch + (xuses & 1) * 256;
    xs[grp * 128 + r] = mine;
    mbar_arrive(&pair_bar[quad]);
    if (!warp_wait_t<false>(&pair_bar[quad], xuses & 1, abort_s)) ok = false;
    ++xuses;
    return xs[(grp ^ 1) * 128 + r];
  };
  for (int j = 0; j < n_tiles && ok; ++j) {
    const int sb = j & 1;
    if (!warp_wait_t<PAIR>(&s_full[sb], (j >> 1) & 1, abort_s)) { ok = false; break; }
    tc::fence_after_sync();
    const uint32_t scol = (sb ? C::COL_S1 : C::COL_S0) + 64 * grp;
    // causal rule + context bound (kernels/paged_attn_prefill.cu:62-65):
    // keys k0 + c of this tile are visible when c < lim; this group's
    // columns c = 64 grp + i are visible when i < mlim
    const int jt = j + rot < n_tiles ? j + rot : j + rot - n_tiles;  // physical tile
    const int64_t k0 = (int64_t)jt * BN;
    const int64_t vis = row_valid ? min(q_abs + 1, ctx) - k0 - 64 * grp : 0;
    const int mlim = vis <= 0 ? 0 : (vis >= 64 ? 64 : (int)vis);
    const bool full = __all_sync(0xffffffffu, mlim == 64);
    // This group's 64 scores of the row: two loads issued back to back, one
    // wait; they stay in registers for the exponentials.  Masked keys become
    // -inf (P = 0).
    uint32_t sa[32], sb2[32];
    tc::tmem_ld32(lane_base + scol, sa);
    tc::tmem_ld32(lane_base + scol + 32, sb2);
    tc::tmem_wait_ld();
    if (!full) {
#pragma unroll
      for (int i = 0; i < 32; ++i) {
        if (i >= mlim) sa[i] = __float_as_uint(-INFINITY);
        if (32 + i >= mlim) sb2[i] = __float_as_uint(-INFINITY);
      }
    }
    float m4[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
#pragma unroll
    for (int i = 0; i < 32; ++i) {
      m4[i & 1] = fmaxf(m4[i & 1], __uint_as_float(sa[i]));
      m4[2 + (i & 1)] = fmaxf(m4[2 + (i & 1)], __uint_as_float(sb2[i]));
    }
    const float pm = fmaxf(fmaxf(m4[0], m4[1]), fmaxf(m4[2], m4[3]));
    const float mt = fmaxf(pm, exchange(pm));
    if (!ok) break;
    // The reference max of a row moves only when the row's max grows by more
    // than 2^8 (then O and l are rescaled); the O rescale is done by the
    // whole warp (tcgen05.ld/st are warp-collective), factor 1 for rows that
    // keep their reference.  Both groups reach the same decision per row.
    const bool need = mt > m_ref + 8.f;
    const float factor = need ? fast_exp2(m_ref - mt) : 1.f;  // 0 on a row's first visible tile
    if (__any_sync(0xffffffffu, need) && j >= 1) {
      // the previous tile's P V must have finished
      if (!warp_wait_t<PAIR>(&o_ready[(j - 1) & 1], ((j - 1) >> 1) & 1, abort_s)) { ok = false; break; }
      tc::fence_after_sync();
#pragma unroll
      for (int c4 = 0; c4 < HD / 32; ++c4) {
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
    // (V rows of keys past the context arrive zeroed from the TMA warp.)
    // P = exp2(s - m_ref) into this group's S columns: keys 32c .. 32c + 31
    // go to columns [32c, 32c + 16) as 16-bit pairs (keys 2i, 2i+1 in column
    // 32c + i), their lo parts to [32c + 16, 32c + 32).
    // (a row with no visible key so far has m_ref = -inf and only masked keys here)
    const float mneg = m_ref == -INFINITY ? 0.f : -m_ref;
    const float2 negm = make_float2(mneg, mneg);
    float2 ls = make_float2(0.f, 0.f);
    auto p_store = [&](const uint32_t (&u)[32], uint32_t col) {
      uint32_t uh[16], ul[16];
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        const float2 x = add2(make_float2(__uint_as_float(u[2 * i]), __uint_as_float(u[2 * i + 1])), negm);
        const float2 e = make_float2(fast_exp2(x.x), fast_exp2(x.y));
        ls = add2(ls, e);
        p_pair(e.x, e.y, uh[i], ul[i], (T*)nullptr);
      }
      tc::tmem_st16(lane_base + col, uh);
      if constexpr (C::SPLIT) tc::tmem_st16(lane_base + col + 16, ul);
    };
    p_store(sa, scol);
    p_store(sb2, scol + 32);
    l += ls.x + ls.y;
    tc::tmem_wait_st();
    tc::fence_before_sync();
    arrive_to_leader<PAIR>(&p_full[sb]);
  }

  // epilogue: O / (l_0 + l_1) -> out, group g writing its HD columns
  float o[HD];
#pragma unroll
  for (int i = 0; i < HD; ++i) o[i] = 0.f;
  if (ok && n_tiles > 0 &&
      !warp_wait_t<PAIR>(&o_ready[(n_tiles - 1) & 1], ((n_tiles - 1) >> 1) & 1, abort_s))
    ok = false;
  if (ok) {
    const float L = l + exchange(l);
    if (ok) {
      const float inv = L > 0.f ? 1.f / L : 0.f;
      tc::fence_after_sync();
#pragma unroll
      for (int c4 = 0; c4 < HD / 32; ++c4) {
        uint32_t u[32];
        tc::tmem_ld32(lane_base + ocol + 32 * c4, u);
        tc::tmem_wait_ld();
#pragma unroll
        for (int i = 0; i < 32; ++i) o[32 * c4 + i] = n_tiles > 0 ? __uint_as_float(u[i]) * inv : 0.f;
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
}

// The softmax role of the two-chain CTA-pair prefill (prefill_pair.cu).
// Warpgroup `grp` owns one chain: the 128 query rows q0 .. q0 + 127 of this
// CTA, one thread per row (TMEM lane), the whole 128-key row of each of the
// chain's n_tiles S tiles (S at COL_S0 + 128 grp, O at COL_O + D grp), KV
// tiles in order.  The other warpgroup runs the other chain on other rows, so
// one chain's exponentials overlap the other's MMAs and no row statistic
// crosses warps.  Stages its Q (pre-scaled, hi / lo parts) and writes O / l to
// `out`.  Arrivals go to the leader CTA of the pair.
template <typename T, int D, typename C>
__device__ __forceinline__ void softmax_chain(const Params& p, unsigned char* smem, uint32_t tmem,
                                              uint64_t* s_full, uint64_t* p_full,
                                              uint64_t* o_ready, uint64_t* q_ready,
                                              int32_t* abort_s, int warp, int lane, int grp,
                                              int64_t b, int64_t h, int64_t q0, int64_t ctx,
                                              int n_tiles) {
  const int quad = warp & 3;
  const int r = quad * 32 + lane;  // query row in the tile = TMEM lane
  const int64_t qrow = q0 + r;
  const bool row_valid = qrow < p.Sq;
  const int64_t q_abs = ctx - p.Sq + qrow;  // absolute position of this query
  {
    unsigned char* qh = smem + C::OFF_Q + grp * C::Q_CHAIN;
    unsigned char* ql = qh + C::Q_PART;
    bool qover = stage_q<T, D, C>(p, qh, ql, b, h, q0, quad * 32, lane);
    qover |= stage_q<T, D, C>(p, qh, ql, b, h, q0, quad * 32 + 16, lane);
    if (qover) report(p.dev_status, PA_DEVERR_RANGE);
    tc::fence_proxy_async_smem();
    arrive_to_leader<true>(q_ready);
  }
  const uint32_t lane_base = tmem + ((uint32_t)(quad * 32) << 16);
  const uint32_t scol = C::COL_S0 + 128 * grp;
  const uint32_t ocol = C::COL_O + D * grp;
  float m_ref = -INFINITY, l = 0.f;
  bool ok = true;
  for (int j = 0; j < n_tiles && ok; ++j) {
    if (!warp_wait_rx(&s_full[grp], j & 1, abort_s)) { ok = false; break; }
    tc::fence_after_sync();
    // causal rule + context bound (kernels/paged_attn_prefill.cu:62-65):
    // keys k0 + c of this tile are visible when c < lim
    const int64_t k0 = (int64_t)j * BN;
    const int64_t vis = row_valid ? min(q_abs + 1, ctx) - k0 : 0;
    const int lim = vis <= 0 ? 0 : (vis >= BN ? BN : (int)vis);
    // the row's 128 scores, read from TMEM once (four loads, one wait);
    // masked keys become -inf, so the row max covers the visible keys only
    const bool full = __all_sync(0xffffffffu, lim == BN);
    uint32_t u[BN];
#pragma unroll
    for (int c4 = 0; c4 < BN / 32; ++c4)
      tc::tmem_ld32(lane_base + scol + 32 * c4, *reinterpret_cast<uint32_t(*)[32]>(u + 32 * c4));
    tc::tmem_wait_ld();
#pragma unroll
    for (int c4 = 0; c4 < BN / 32; ++c4) tc::reg_fence(*reinterpret_cast<uint32_t(*)[32]>(u + 32 * c4));
    if (!full) {
#pragma unroll
      for (int i = 0; i < BN; ++i)
        if (i >= lim) u[i] = __float_as_uint(-INFINITY);
    }
    float mt;
    {
      float m4[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
#pragma unroll
      for (int i = 0; i < BN; ++i) m4[i & 3] = fmaxf(m4[i & 3], __uint_as_float(u[i]));
      mt = fmaxf(fmaxf(m4[0], m4[1]), fmaxf(m4[2], m4[3]));
    }
    // The reference max of a row moves only when the row's max grows by more
    // than 2^8 (then O and l are rescaled, factor 1 for rows that keep theirs;
    // tcgen05.ld/st are warp-collective).  O is rescaled after the P stores,
    // once the score registers are free, and before P V is released.
    const bool need = mt > m_ref + 8.f;
    const float factor = need ? fast_exp2(m_ref - mt) : 1.f;  // 0 on a row's first visible tile
    const bool rescale = __any_sync(0xffffffffu, need) && j >= 1;
    if (need) {
      l *= factor;
      m_ref = mt;
    }
    // P = exp2(s - m_ref) into the S columns, 32 keys at a time: keys
    // 32c .. 32c + 31 go to columns [32c, 32c + 16) as 16-bit pairs, their lo
    // parts to [32c + 16, 32c + 32).  (A row with no visible key so far has
    // m_ref = -inf and only masked keys here.)
    const float mneg = m_ref == -INFINITY ? 0.f : -m_ref;
    const float2 negm = make_float2(mneg, mneg);
    float2 ls = make_float2(0.f, 0.f);
#pragma unroll
    for (int c = 0; c < BN / 32; ++c) {
      uint32_t uh[16], ul[16];
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        const float2 x = add2(make_float2(__uint_as_float(u[32 * c + 2 * i]), __uint_as_float(u[32 * c + 2 * i + 1])), negm);
        const float2 e = make_float2(fast_exp2(x.x), fast_exp2(x.y));
        ls = add2(ls, e);
        p_pair(e.x, e.y, uh[i], ul[i], (T*)nullptr);
      }
      tc::tmem_st16(lane_base + scol + 32 * c, uh);
      if constexpr (C::SPLIT) tc::tmem_st16(lane_base + scol + 32 * c + 16, ul);
    }
    l += ls.x + ls.y;
    if (rescale) {
      // the chain's previous P V must have finished
      if (!warp_wait_rx(&o_ready[grp], (j - 1) & 1, abort_s)) { ok = false; break; }
      tc::fence_after_sync();
#pragma unroll
      for (int c4 = 0; c4 < D / 32; ++c4) {
        uint32_t o[32];
        tc::tmem_ld32(lane_base + ocol + 32 * c4, o);
        tc::tmem_wait_ld();
#pragma unroll
        for (int i = 0; i < 32; ++i) o[i] = __float_as_uint(__uint_as_float(o[i]) * factor);
        tc::tmem_st32(lane_base + ocol + 32 * c4, o);
      }
    }
    // every lane's P (and O) stores complete, then one arrival per warp, to
    // the leader's barrier, relaxed: P is tensor-memory data, ordered by
    // tcgen05.wait::st and the fence; no generic write needs releasing (a
    // release at cluster scope here cost ~1-2 thousand cycles per tile and
    // lay on the chain's critical path)
    tc::tmem_wait_st();
    tc::fence_before_sync();
    __syncwarp();
    if (lane == 0) tc::mbar_arrive_cluster_relaxed(tc::mapa_shared(&p_full[grp], 0));
  }

  // epilogue: O / l -> out, 32 columns at a time
  if (ok && n_tiles > 0 && !warp_wait_rx(&o_ready[grp], (n_tiles - 1) & 1, abort_s)) ok = false;
  const bool have = ok && n_tiles > 0;
  const float inv = l > 0.f ? 1.f / l : 0.f;
  if (have) tc::fence_after_sync();
  float* dst = p.out + ((b * p.Sq + qrow) * p.H + h) * D;
#pragma unroll
  for (int c4 = 0; c4 < D / 32; ++c4) {
    uint32_t u[32];
    if (have) {
      tc::tmem_ld32(lane_base + ocol + 32 * c4, u);
      tc::tmem_wait_ld();
    }
    if (row_valid) {
#pragma unroll
      for (int i = 0; i < 32; i += 4)
        *reinterpret_cast<float4*>(dst + 32 * c4 + i) =
            have ? make_float4(__uint_as_float(u[i]) * inv, __uint_as_float(u[i + 1]) * inv,
                               __uint_as_float(u[i + 2]) * inv, __uint_as_float(u[i + 3]) * inv)
                 : make_float4(0.f, 0.f, 0.f, 0.f);
    }
  }
  if (!ok && lane == 0) report(p.dev_status, PA_DEVERR_TIMEOUT);
}

// Host: the CTA-pair kernel for head_dim 128 (prefill_pair.cu).
int launch_pair(const Params& p, int dtype, cudaStream_t s);

// Host: tensor map of one pool tensor as [D, HKV, NB * BS] with a 64 x 1 x 16
// box and 128-byte swizzle (prefill_tc.cu).
int make_map(CUtensorMap* m, const void* base, int dtype, int64_t D, int64_t HKV, int64_t rows);

}  // namespace prefill
}  // namespace pa
