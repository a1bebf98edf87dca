// decode_impl.cuh -- split-KV paged decode for sm_100a.
//
// Replaces paged_attention_split_kernel + merge_splits_kernel of
// gb10-attn kernels/paged_attn_v3.cu:33-166 (and the v1/v2 decode kernels,
// which compute the same function).  Same math: online softmax per piece of
// context, un-normalised partials, log-sum-exp merge (:113-122, :139-165).
// Different machine mapping:
//
//   * Work unit = a tile of kTT = 16 (FP8 pools with QC == 1: 32) consecutive tokens of one sequence for a
//     group of G kv heads ("g-chunk").  The NGC * sum_b ceil(ctx_b / 16) tiles
//     are split into N contiguous ranges, one per CTA (N = SMs x resident CTAs
//     for automatic splitting), so every SM streams about the same number of
//     bytes whatever the context lengths (stream-K style).  The ranges are
//     equal in cost: a sequence start counts as extra tiles (Params::beta).
//     For batches up to kFusedRows rows every CTA builds the plan (tile
//     offsets) in shared memory itself; larger ones use the plan kernel.
//   * One producer warp per CTA issues 1-D bulk (TMA) copies of the token
//     rows [G kv heads x D] of K and V straight from the pages into a ring of
//     shared-memory stages guarded by mbarriers.  A stage is 16 tokens; a row
//     is G*D*sizeof(T) contiguous bytes of a page, landing in this CTA only.
//   * Each consumer warp owns one "slot": one kv head of the g-chunk and QC of
//     the query heads that share it (GQA), so every KV byte is read from HBM
//     once and from shared memory once per slot.  Inside a warp, R lanes
//     hold one token row (lane owns EPL elements, 16-byte shared loads) and
//     the 32/R row groups take different tokens, each keeping its own online
//     softmax state (m, l, acc) in registers; the row groups are merged with
//     shuffles once per segment, not per token.
//   * A sequence whose tiles span several CTAs is merged by the CTA that
//     finishes its piece last (per-(sequence, slot) arrival counter, two
//     levels for long sequences), so no second kernel and no extra partial
//     round trip for unsplit sequences.
//
// Scores are kept in the log2 domain (q pre-scaled by scale*log2(e)) so each
// exponential is one ex2.approx; the reference's __expf is the same
// instruction after a multiply.
#pragma once

#include "common.cuh"

namespace pa {
namespace decode {

constexpr int kTT = 16;            // tokens per pipeline stage (16-bit and wider pools)
constexpr int kGroup = 8;          // pieces merged per step of a split sequence
constexpr int kFusedRows = 1024;   // rows up to which each CTA plans for itself
constexpr int kCountBits = 24;     // arrival count bits of an epoch-tagged counter
constexpr int kPlanScratchBytes = 272;  // scan scratch ahead of the fused plan tables
constexpr float kNegBig = -3.0e38f;  // the reference's "minus infinity" (paged_attn_v3.cu:20)

// FP8 pools with one query head per KV row and warp (QC == 1) use 32-token
// stages: the bytes of a 16-bit pool's 16 tokens, and twice the rows per
// consumer lane for each stage wait (3.72 vs 3.01 TB/s at configs[1]
// geometry).  With several query heads per KV row the consumer work per stage
// already dominates, and 16-token stages measured faster (88.0 vs 108.7 us
// per call at configs[2] geometry).
template <typename T, int QC>
struct Tile {
  static constexpr int TT = (sizeof(T) == 1 && QC == 1) ? 2 * kTT : kTT;
};
inline int tile_tokens(int dtype, int qc) {
  return (dtype_size(dtype) == 1 && qc == 1) ? 2 * kTT : kTT;
}

struct Params {
  float* out;                    // [B, H, D]
  float* lse;                    // [B, H] or null
  const float* q;                // [B, H, D]
  const char* k_cache;           // [NB, BS, HKV, D] bytes
  const char* v_cache;
  const int32_t* block_tables;   // [B, MB]
  const int32_t* context_lens;   // [B]
  int32_t* dev_status;           // nullable
  // Plan tables from the plan kernel, or null: then every CTA builds them in
  // shared memory from context_lens (B <= kFusedRows).
  const int32_t* tile_off;       // [B + 1] tiles before sequence b (per g-chunk)
  const int32_t* cta_seq;        // [N] sequence holding each CTA's first tile
  // Merge arrival counters, tagged with the launch's epoch in the high bits
  // so no launch has to zero them: a value from an earlier launch reads as 0.
  unsigned long long* counters;      // [NGC * B * NS]
  unsigned long long* grp_counters;  // [N * 2 * NS] arrivals per run of kGroup pieces, or null
  unsigned long long epoch;          // this launch's tag (nonzero, < 2^40)
  int32_t arrive_rounds;             // CAS rounds before an arrival gives up
  int32_t* abort_flag;           // holds abort_tag once any pipeline wait timed out
  int32_t abort_tag;
  float empty_fill;              // rows of empty sequences (fused plan)
  // Weighted split (fused plan only): the first tile of every sequence but
  // the first counts as 1 + beta tiles of work, so CTAs that move on to
  // another sequence (a block-table reload, q reload and a published piece)
  // get fewer tiles.  0 with the plan kernel.
  int32_t beta;
  float* partials;               // [N * 2 * NS * QC * (D + 2)]
  int64_t B, H, HKV, NB, MB, BS;
  // Query rows per block-table row: 1 for decode.  For causal prefill row
  // b' = b * qlen + s is query s of sequence b; it reads block_tables[b] and
  // sees keys [0, context_lens[b] - qlen + s] (paged_attn_prefill.cu:62-65).
  int64_t qlen;
  int32_t G, QPK, NS, NGC, N, nstage;
  float qscale;                  // scale * log2(e)
  // FP8 pools: per-KV-head dequantisation scales (null = 1); K's scale folds
  // into q, V's into the softmax weights.  Unused for the other dtypes.
  const float* k_scale;
  const float* v_scale;
  uint32_t row_bytes;            // G * D * sizeof(T)
  int32_t rows_contiguous;       // G == HKV: a page's token rows are adjacent
  int64_t tok_stride;            // HKV * D * sizeof(T): one token row of a page
  int32_t bs_shift;              // log2(BS) when BS is a power of two, else -1
  int64_t blk_stride;            // BS * tok_stride: one page
  // q / out element type (PA_DTYPE_F32 / F16 / BF16: `q` and `out` point at
  // that type; partials and lse stay fp32) and the decode step's new K / V
  // rows ([B, HKV, D] of io_dtype, null: none): the producer that loads a
  // sequence's last tile first writes them at position context_lens[b] - 1.
  int32_t io_dtype;
  const char* k_new;
  const char* v_new;
};

// q / out elements in the call's io type
__device__ __forceinline__ float io_load(int io, const void* base, int64_t i) {
  if (io == PA_DTYPE_BF16) return __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(base)[i]);
  if (io == PA_DTYPE_F16) return __half2float(reinterpret_cast<const __half*>(base)[i]);
  return reinterpret_cast<const float*>(base)[i];
}
__device__ __forceinline__ void io_store(int io, void* base, int64_t i, float x) {
  if (io == PA_DTYPE_BF16)
    reinterpret_cast<__nv_bfloat16*>(base)[i] = __float2bfloat16_rn(x);
  else if (io == PA_DTYPE_F16)
    reinterpret_cast<__half*>(base)[i] = __float2half_rn(x);
  else
    reinterpret_cast<float*>(base)[i] = x;
}
// two adjacent elements (i even): one 8- or 4-byte access
__device__ __forceinline__ float2 io_load2(int io, const void* base, int64_t i) {
  if (io == PA_DTYPE_F32) return *reinterpret_cast<const float2*>(reinterpret_cast<const float*>(base) + i);
  const uint32_t w = *reinterpret_cast<const uint32_t*>(reinterpret_cast<const uint16_t*>(base) + i);
  if (io == PA_DTYPE_BF16) return make_float2(__uint_as_float(w << 16), __uint_as_float(w & 0xffff0000u));
  const __half2 h = *reinterpret_cast<const __half2*>(&w);
  return __half22float2(h);
}
__device__ __forceinline__ void io_store2(int io, void* base, int64_t i, float2 x) {
  if (io == PA_DTYPE_F32) {
    *reinterpret_cast<float2*>(reinterpret_cast<float*>(base) + i) = x;
  } else if (io == PA_DTYPE_BF16) {
    const __nv_bfloat162 h = __floats2bfloat162_rn(x.x, x.y);
    *reinterpret_cast<__nv_bfloat162*>(reinterpret_cast<__nv_bfloat16*>(base) + i) = h;
  } else {
    const __half2 h = __floats2half2_rn(x.x, x.y);
    *reinterpret_cast<__half2*>(reinterpret_cast<__half*>(base) + i) = h;
  }
}
// a pool element from fp32, rounded to nearest even (the writer's rule)
template <typename T> __device__ __forceinline__ T pool_from_f32(float x);
template <> __device__ __forceinline__ float pool_from_f32<float>(float x) { return x; }
template <> __device__ __forceinline__ double pool_from_f32<double>(float x) { return (double)x; }
template <> __device__ __forceinline__ __half pool_from_f32<__half>(float x) { return __float2half_rn(x); }
template <> __device__ __forceinline__ __nv_bfloat16 pool_from_f32<__nv_bfloat16>(float x) {
  return __float2bfloat16_rn(x);
}
template <> __device__ __forceinline__ __nv_fp8_e4m3 pool_from_f32<__nv_fp8_e4m3>(float x) {
  __nv_fp8_e4m3 r;
  r.__x = __nv_cvt_float_to_fp8(x, __NV_SATFINITE, __NV_E4M3);
  return r;
}


struct __align__(16) StageHeader {
  int32_t b, gc, tok0, nvalid;
  int32_t flags, seq_k, pad1, pad2;  // seq_k: ordinal among the non-empty sequences
  int64_t gt, seq_t0, seq_t1, pad3;
};
constexpr int kFirst = 1, kLast = 2, kEnd = 4, kCtaLast = 8;

// Lane geometry for element type T and head_dim D (TT tokens per stage).
template <typename T, int D, int TT = kTT>
struct Geo {
  static constexpr int VEC = Chunk<T>::N;                 // elements per 16 B
  static constexpr int CH = D / VEC;                      // 16 B chunks per row
  static constexpr int R = CH <= 8 ? CH : (CH / 2 > 32 ? 32 : CH / 2);  // lanes per row
  static constexpr int NCH = CH / R;                      // chunks per lane
  static constexpr int EPL = NCH * VEC;                   // elements per lane
  static constexpr int NRG = 32 / R;                      // row groups per warp
  static constexpr int TPR = TT / NRG;                    // tokens per row group per stage
  static_assert(D % VEC == 0 && CH % R == 0 && 32 % R == 0 && NRG <= TT, "geometry");
};

// CTA shape of a (T, D, QC) instantiation, by the per-lane register state
// S = QC * EPL floats of q (and as many of acc):
//  * kLight (S <= 8; <= 16 for FP8; <= 4 for 4/8-byte types): consumer warps
//    0..NS-1 (up to 16) plus the producer warp NS; (NS + 1) * 32 threads.
//  * kWs16 (S <= 32): warp-specialised.  Warpgroup 0 is the producer (warp 0
//    issues copies, warps 1-3 retire) and hands registers back with
//    setmaxnreg.dec; warpgroups 1-4 are up to 16 consumer warps.  640 threads
//    launched at 96 registers (20 warps, 5 per SM sub-partition) = 61440; after
//    the split 128 x 40 + 512 x 104 = 58368.
//  * kWs8 (larger S): warpgroup 0 producer, warpgroups 1-2 = 8 consumer warps.
//    384 threads x 168 registers = 64512; after the split 128 x 56 + 256 x 224
//    = 64512.
// setmaxnreg.inc draws on the registers the CTA was launched with, so each
// split stays inside its launch total (checked below).
enum CtaKind { kLight = 0, kWs16 = 1, kWs8 = 2 };

template <typename T, int D, int QC>
struct Limits {
  static constexpr int S = QC * Geo<T, D>::EPL;
  // FP8 rows put 16 elements in a lane at D = 64: still a light CTA (measured
  // 3.28 TB/s at configs[1] geometry, against 2.67 TB/s as a kWs16 CTA)
  static constexpr int kLightS = sizeof(T) == 1 ? 16 : 8;
  static constexpr int KIND = (sizeof(T) <= 2 ? (S <= kLightS ? kLight : (S <= 32 ? kWs16 : kWs8))
                                              : (S <= 4 ? kLight : (S <= 16 ? kWs16 : kWs8)));
  static constexpr bool WS = KIND != kLight;
  static constexpr int MAXW = KIND == kWs8 ? 8 : 16;
  static constexpr int THREADS = KIND == kWs8 ? 384 : (KIND == kWs16 ? 640 : 544);
  static constexpr int PROD_REGS = KIND == kWs8 ? 56 : 40;
  static constexpr int CONS_REGS = KIND == kWs8 ? 224 : 104;
};
static_assert(128 * 56 + 256 * 224 <= 384 * 168, "kWs8 register split exceeds launch");
static_assert(128 * 40 + 512 * 104 <= 640 * 96, "kWs16 register split exceeds launch");

__host__ __device__ __forceinline__ int64_t cta_lo(int64_t c, int64_t T_all, int64_t N) {
  return T_all >= N ? (c * T_all + N - 1) / N : (c < T_all ? c : T_all);
}
// CTA whose range holds global tile t < T_all: the largest c with cta_lo(c) <= t.
__host__ __device__ __forceinline__ int64_t cta_of(int64_t t, int64_t T_all, int64_t N) {
  return T_all >= N ? t * N / T_all : t;
}

// One arrival on an epoch-tagged counter (value = epoch << kCountBits |
// count); returns the arrivals of this launch before it.  A value left by an
// earlier launch (another epoch) counts as zero, so counters are never reset.
// Gives up after `rounds` failed compare-and-swap rounds and returns -1: the
// arrival is not counted, so no warp completes that merge, and the caller
// writes NaN rows and reports PA_DEVERR_MERGE instead.
__device__ __forceinline__ int epoch_arrive(unsigned long long* counter, unsigned long long epoch,
                                            int rounds) {
  unsigned long long v = *reinterpret_cast<volatile unsigned long long*>(counter);
  for (int it = 0; it < rounds; ++it) {  // lock-free: one CAS wins per round
    const bool same = (v >> kCountBits) == epoch;
    const unsigned long long nv = same ? v + 1 : ((epoch << kCountBits) | 1ull);
    const unsigned long long prev = atomicCAS(counter, v, nv);
    if (prev == v) return same ? (int)(v & ((1ull << kCountBits) - 1)) : 0;
    v = prev;
  }
  return -1;  // never settled: the arrival is not counted
}

// The plan of one launch built by every CTA in shared memory (B <= kFusedRows
// rows; scratch = 33 64-bit words): ne_s[b] = non-empty rows before b;
// tile_off_s[b] = tiles of rows 0..b-1, ntok_s[b] = keys row b reads
// (the plan kernel's rule: a query row s of qlen sees context - qlen + s + 1
// keys, clamped to the block table).  CTA b % gridDim fills the output rows of
// empty sequences (the reference's v3 yields NaN there, paged_attn_v3.cu:160-165).
template <int D, int TT>
__device__ __forceinline__ void fused_plan(const Params& p, int io, int32_t* tile_off_s, int32_t* ntok_s,
                                           int32_t* ne_s, long long* scratch) {
  // one scan carries both counts: tiles in the high bits, non-empty rows in
  // the low 16 (rows <= kFusedRows < 2^16)
  long long* warp_tot = scratch;     // [32]
  long long& carry_s = scratch[32];
  const int tid = threadIdx.x, lane = tid & 31, wid = tid >> 5, nw = blockDim.x >> 5;
  const int64_t max_ctx = p.MB * p.BS;
  if (tid == 0) carry_s = 0;
  __syncthreads();
  for (int64_t base = 0; base < p.B; base += blockDim.x) {
    const int64_t b = base + tid;
    int32_t tiles = 0;
    if (b < p.B) {
      const int64_t sq = b / p.qlen;
      const int64_t c = p.context_lens[sq];
      if (c > max_ctx && b == sq * p.qlen && blockIdx.x == 0) report(p.dev_status, PA_DEVERR_CONTEXT);
      int64_t n = c - p.qlen + (b - sq * p.qlen) + 1;
      if (n > max_ctx) n = max_ctx;
      if (n <= 0) {
        n = 0;
        if (b % gridDim.x == blockIdx.x) {
          for (int64_t i = 0; i < p.H * D; ++i) io_store(io, p.out, b * p.H * D + i, p.empty_fill);
          if (p.lse)
            for (int64_t h = 0; h < p.H; ++h) p.lse[b * p.H + h] = -INFINITY;
        }
      }
      ntok_s[b] = (int32_t)n;
      tiles = (int32_t)((n + TT - 1) / TT);
    }
    const long long mine = ((long long)tiles << 16) | (tiles > 0 ? 1 : 0);
    long long x = mine;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const long long y = __shfl_up_sync(0xffffffffu, x, o);
      if (lane >= o) x += y;
    }
    if (lane == 31) warp_tot[wid] = x;
    __syncthreads();
    if (wid == 0) {
      long long w = lane < nw ? warp_tot[lane] : 0;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const long long y = __shfl_up_sync(0xffffffffu, w, o);
        if (lane >= o) w += y;
      }
      if (lane < nw) warp_tot[lane] = w;  // inclusive over warps
    }
    __syncthreads();
    const long long carry = carry_s;
    if (b < p.B) {
      const long long excl = carry + (wid ? warp_tot[wid - 1] : 0) + x - mine;
      tile_off_s[b] = (int32_t)(excl >> 16);
      ne_s[b] = (int32_t)(excl & 0xffff);
    }
    __syncthreads();
    if (tid == 0) carry_s = carry + warp_tot[nw - 1];
    __syncthreads();
  }
  if (tid == 0) {
    tile_off_s[p.B] = (int32_t)(carry_s >> 16);
    ne_s[p.B] = (int32_t)(carry_s & 0xffff);
  }
  __syncthreads();
}

// Log-sum-exp merge of the partial states at ptr(c0), ptr(c0 + stride), ...
// (count of them; layout [QC][D] un-normalised O, then QC maxima, then QC
// sums).  One warp.  The result is a fixed function of the states: they are
// folded in state order with the online rule (fold_state, every operation
// pinned by fmaf / __fmul_rn), so whichever warp merges a sequence (the last
// to arrive, which varies from launch to launch) writes the same bits.
// Every lane ends with the merged maxima mg, sums lg and elements lane + 32k
// of O in o[k].
template <int QC, int D>
__device__ __forceinline__ void fold_state(float (&o)[QC * D / 32], float (&mg)[QC],
                                           float (&lg)[QC], const float (&ms)[QC],
                                           const float (&ls)[QC], const float (&os)[QC * D / 32]) {
  constexpr int PER = QC * D / 32;
  float a[QC], b[QC];
#pragma unroll
  for (int j = 0; j < QC; ++j) {
    const float mn = fmaxf(mg[j], ms[j]);
    a[j] = fast_exp2(mg[j] - mn);
    b[j] = fast_exp2(ms[j] - mn);
    lg[j] = fmaf(ls[j], b[j], __fmul_rn(lg[j], a[j]));
    mg[j] = mn;
  }
#pragma unroll
  for (int q = 0; q < PER; ++q)
    o[q] = fmaf(os[q], b[(32 * q) / D], __fmul_rn(o[q], a[(32 * q) / D]));
}

template <int QC, int D, typename PtrFn>
__device__ __forceinline__ void load_state(PtrFn ptr, int64_t c, int lane, float (&ms)[QC],
                                           float (&ls)[QC], float (&os)[QC * D / 32]) {
  const float* pc = ptr(c);
#pragma unroll
  for (int j = 0; j < QC; ++j) {
    ms[j] = __ldcg(pc + QC * D + j);
    ls[j] = __ldcg(pc + QC * D + QC + j);
  }
#pragma unroll
  for (int q = 0; q < QC * D / 32; ++q) os[q] = __ldcg(pc + lane + 32 * q);
}

// One state at a time (few registers: usable inside the consumer loop).
template <int QC, int D, typename PtrFn>
__device__ __forceinline__ void merge_pieces(PtrFn ptr, int64_t c0, int64_t stride, int64_t count,
                                             int lane, float (&o)[QC * D / 32], float (&mg)[QC],
                                             float (&lg)[QC]) {
  constexpr int PER = QC * D / 32;
#pragma unroll
  for (int j = 0; j < QC; ++j) { mg[j] = kNegBig; lg[j] = 0.f; }
#pragma unroll
  for (int k = 0; k < PER; ++k) o[k] = 0.f;
#pragma unroll 2
  for (int64_t k = 0; k < count; ++k) {
    float ms[QC], ls[QC], os[PER];
    load_state<QC, D>(ptr, c0 + k * stride, lane, ms, ls, os);
    fold_state<QC, D>(o, mg, lg, ms, ls, os);
  }
}

// The same merge with U states' loads in flight together (~24 registers per
// state per lane: runs where the consumer's q and accumulator registers are
// no longer live).  Same fold, same order: bit-identical to merge_pieces.
template <int QC, int D, int U, typename PtrFn>
__device__ __forceinline__ void merge_pieces_wide(PtrFn ptr, int64_t c0, int64_t stride,
                                                  int64_t count, int lane, float (&o)[QC * D / 32],
                                                  float (&mg)[QC], float (&lg)[QC]) {
  constexpr int PER = QC * D / 32;
#pragma unroll
  for (int j = 0; j < QC; ++j) { mg[j] = kNegBig; lg[j] = 0.f; }
#pragma unroll
  for (int k = 0; k < PER; ++k) o[k] = 0.f;
  for (int64_t k0 = 0; k0 < count; k0 += U) {
    float ms[U][QC], ls[U][QC], os[U][PER];
#pragma unroll
    for (int u = 0; u < U; ++u)
      if (k0 + u < count) load_state<QC, D>(ptr, c0 + (k0 + u) * stride, lane, ms[u], ls[u], os[u]);
#pragma unroll
    for (int u = 0; u < U; ++u)
      if (k0 + u < count) fold_state<QC, D>(o, mg, lg, ms[u], ls[u], os[u]);
  }
}

// STEP: the decode-step instantiation (q / out of p.io_dtype, the K / V
// append); the plain one reads fp32 q and writes fp32 out with no branch.
template <typename T, int D, int QC, bool STEP>
__global__ void __launch_bounds__(Limits<T, D, QC>::THREADS, 1)
    decode_kernel(const __grid_constant__ Params p) {
  const int io = STEP ? p.io_dtype : (int)PA_DTYPE_F32;
  constexpr int TT = Tile<T, QC>::TT;
  using G_ = Geo<T, D, TT>;
  constexpr int VEC = G_::VEC, R = G_::R, NCH = G_::NCH, EPL = G_::EPL;
  constexpr int NRG = G_::NRG, TPR = G_::TPR;

  extern __shared__ __align__(128) unsigned char smem[];
  const int nstage = p.nstage;
  const uint32_t stage_bytes = 2u * TT * p.row_bytes;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + (size_t)nstage * stage_bytes);
  uint64_t* empty = full + nstage;
  StageHeader* hdr = reinterpret_cast<StageHeader*>(empty + nstage);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int NS = p.NS;
  constexpr bool WS = Limits<T, D, QC>::WS;

  if (threadIdx.x == 0) {
    for (int s = 0; s < nstage; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], NS);
    }
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  __syncthreads();
  // Everything above overlaps the previous kernel on the stream (the plan
  // kernel, or the previous call); its results are read below.  The next
  // kernel may launch now: it waits for this grid to complete before it
  // touches memory.
  pdl_wait();
  pdl_trigger();

  // Plan tables: the plan kernel's (global) or, for small batches, built here
  // by the whole CTA in shared memory -- no plan kernel on the stream and no
  // global round trips when the producer moves to the next sequence.
  const int32_t* tile_off = p.tile_off;
  const int32_t* ntok_s = nullptr;
  const int32_t* ne_s = nullptr;
  if (tile_off == nullptr) {
    unsigned char* plan_base = reinterpret_cast<unsigned char*>(hdr + nstage);
    int32_t* to_s = reinterpret_cast<int32_t*>(plan_base + kPlanScratchBytes);
    int32_t* nt_s = to_s + p.B + 1;
    int32_t* nz_s = nt_s + p.B;
    fused_plan<D, TT>(p, io, to_s, nt_s, nz_s, reinterpret_cast<long long*>(plan_base));
    tile_off = to_s;
    ntok_s = nt_s;
    ne_s = nz_s;
  }

  const int64_t Tpg = tile_off[p.B];  // tiles per g-chunk
  const int64_t T_all = Tpg * p.NGC;
  const int64_t cta = blockIdx.x;
  // Weighted stream-K split.  Tile t of the k-th non-empty sequence costs
  // from t + beta * k on, C is the total; CTA c owns the tiles whose cost
  // lies in [ceil(c C / N), ceil((c+1) C / N)).  beta is used only while
  // every CTA's share (>= 2 beta + 2) outweighs the jump at a sequence start,
  // so no CTA is left without tiles.
  const int64_t Kseq = ne_s ? (int64_t)p.NGC * ne_s[p.B] : 0;
  const int64_t beta = (ne_s && p.beta > 0 && T_all >= p.N &&
                        T_all + (int64_t)p.beta * (Kseq - 1) >= (int64_t)p.N * (2 * p.beta + 2))
                           ? p.beta : 0;
  const int64_t Ccost = T_all + beta * (Kseq > 0 ? Kseq - 1 : 0);
  // CTA owning tile t of the sequence with ordinal k
  auto owner = [&](int64_t t, int64_t k) -> int64_t {
    return T_all >= p.N ? (t + beta * k) * p.N / Ccost : t;
  };

  if constexpr (WS) {
    if (warp < 4) {
      asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(Limits<T, D, QC>::PROD_REGS));
      if (warp != 0) return;
    } else {
      asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(Limits<T, D, QC>::CONS_REGS));
      if (warp - 4 >= NS) return;
    }
  }
  const bool is_producer = WS ? (warp == 0) : (warp == NS);

  if (is_producer) {
    // ------------------------------------------------------------------ producer
    // This CTA's tiles [lo, hi).  Weighted split: the first non-empty
    // sequence whose last tile's cost reaches each bound, found by the 32
    // lanes over 32 sequences at a time.
    int64_t lo, hi, lo_seq = -1;
    if (beta == 0) {
      lo = cta_lo(cta, T_all, p.N);
      hi = cta_lo(cta + 1, T_all, p.N);
    } else {
      const int64_t t_lo = (cta * Ccost + p.N - 1) / p.N;
      const int64_t t_hi = cta + 1 >= p.N ? Ccost : ((cta + 1) * Ccost + p.N - 1) / p.N;
      const int Bi = (int)p.B, S = p.NGC * Bi, Kr = ne_s[p.B];
      int s_lo = -1, s_hi = -1;
      for (int base = 0; base < S && (s_lo < 0 || s_hi < 0); base += 32) {
        const int sq = base + lane;
        long long cl = -1;  // empty rows never qualify
        if (sq < S) {
          const int g = sq / Bi, bb = sq - g * Bi;
          if (tile_off[bb + 1] > tile_off[bb])
            cl = (long long)g * Tpg + tile_off[bb + 1] - 1 + beta * ((long long)g * Kr + ne_s[bb]);
        }
        const unsigned m_lo = __ballot_sync(0xffffffffu, cl >= t_lo);
        const unsigned m_hi = __ballot_sync(0xffffffffu, cl >= t_hi);
        if (s_lo < 0 && m_lo) s_lo = base + __ffs(m_lo) - 1;
        if (s_hi < 0 && m_hi) s_hi = base + __ffs(m_hi) - 1;
      }
      // first tile whose cost reaches t: within sequence sq, or its first tile
      auto tile_at = [&](int sq, int64_t t) -> int64_t {
        const int g = sq / Bi, bb = sq - g * Bi;
        const int64_t start = (int64_t)g * Tpg + tile_off[bb];
        const int64_t x = t - beta * ((int64_t)g * Kr + ne_s[bb]);
        return x > start ? x : start;
      };
      lo = s_lo >= 0 ? tile_at(s_lo, t_lo) : T_all;
      hi = (cta + 1 >= p.N || s_hi < 0) ? T_all : tile_at(s_hi, t_hi);
      lo_seq = s_lo;
    }
    int stage = 0;
    uint32_t phase = 0;
    bool ok = true;
    if (lo < hi) {
      int64_t gt = lo;
      int gc = (int)(lo / Tpg);
      int64_t r = lo - (int64_t)gc * Tpg;
      int b;
      if (lo_seq >= 0) {  // weighted split: the search found it
        b = (int)(lo_seq % p.B);
      } else if (p.cta_seq) {
        b = p.cta_seq[cta];
      } else {  // upper_bound(tile_off[0..B], r) - 1
        int64_t a = 0, z = p.B + 1;
        while (a < z) {
          const int64_t mid = (a + z) >> 1;
          if (tile_off[mid] <= r) a = mid + 1;
          else z = mid;
        }
        b = (int)(a - 1);
      }
      int64_t s0 = tile_off[b], s1 = tile_off[b + 1];
      const int64_t max_ctx = p.MB * p.BS;
      auto seq_len = [&](int bb) -> int64_t {
        if (ntok_s) return ntok_s[bb];
        const int64_t sq = bb / p.qlen;
        int64_t n = (int64_t)p.context_lens[sq] - p.qlen + (bb - sq * p.qlen) + 1;
        if (n > max_ctx) n = max_ctx;
        return n < 0 ? 0 : n;
      };
      int64_t n_tok = seq_len(b);
      // ordinal of the sequence among the non-empty ones (the weighted
      // split's cost of its tiles; carried to the consumers' merges)
      auto ordinal = [&](int g, int bb) -> int32_t {
        return ne_s ? (int32_t)((int64_t)g * ne_s[p.B] + ne_s[bb]) : 0;
      };
      int32_t seq_k = ordinal(gc, b);
      const int32_t* bt = p.block_tables + (int64_t)(b / p.qlen) * p.MB;
      auto bt_load = [&](int64_t idx) -> int32_t {
        return (idx >= 0 && idx < p.MB) ? __ldg(bt + idx) : 0;
      };
      int64_t win_base = -1;
      int32_t win_cur = 0, win_next = 0;
      int nx_b = 0, nx_gc = 0;           // the next sequence of this CTA's range
      int32_t nx_cur = 0, nx_next = 0;   // its first block-table window
      const int64_t gbytes = (int64_t)p.G * D * (int64_t)sizeof(T);
      const int64_t qes = io == PA_DTYPE_F32 ? 4 : 2;  // bytes per q element
      const uint32_t qbytes = (uint32_t)(p.G * p.QPK * D * qes);

      while (gt < hi) {
        const int64_t t_in_seq = r - s0;
        const int64_t tok0 = t_in_seq * TT;
        const int nvalid = (int)(n_tok - tok0 < TT ? n_tok - tok0 : TT);
        // block-table window: lane l holds bt[win_base + l] (cur) and
        // bt[win_base + 32 + l] (next); `next` is loaded a window ahead.
        // page of a token: a shift, or a 32-bit division (every token index
        // is below 2^31, MB * BS being checked on the host)
        auto page_of = [&](int64_t tok) -> int64_t {
          return p.bs_shift >= 0 ? (tok >> p.bs_shift)
                                 : (int64_t)((uint32_t)tok / (uint32_t)p.BS);
        };
        const int64_t pg_lo = page_of(tok0);
        if (win_base < 0 || pg_lo >= win_base + 32) {
          if (win_base >= 0 && pg_lo < win_base + 64) {
            win_base += 32;
            win_cur = win_next;
          } else {
            win_base = pg_lo;
            win_cur = bt_load(win_base + lane);
          }
          win_next = bt_load(win_base + 32 + lane);
        }
        if (!mbar_wait(&empty[stage], phase ^ 1, p.abort_flag, p.abort_tag)) { ok = false; break; }

        // lane = (row % 16, K|V); TT / 16 rows per lane
        constexpr int RPL = TT / 16;
        const int kv = lane >> 4;
        int64_t blk_r[RPL], pg_r[RPL];
        bool bad = false;
#pragma unroll
        for (int hh = 0; hh < RPL; ++hh) {
          const int row = (lane & 15) + 16 * hh;
          const int64_t pg = page_of(tok0 + row);
          pg_r[hh] = pg;
          const int idx = (int)(pg - win_base);
          const int32_t a = __shfl_sync(0xffffffffu, win_cur, idx & 31);
          const int32_t c = __shfl_sync(0xffffffffu, win_next, idx & 31);
          blk_r[hh] = idx < 32 ? a : c;
          if (row < nvalid && (blk_r[hh] < 0 || blk_r[hh] >= p.NB)) { bad = true; blk_r[hh] = 0; }
        }
        if (__any_sync(0xffffffffu, bad) && lane == 0) report(p.dev_status, PA_DEVERR_BLOCK_ID);

        if (lane == 0) {
          StageHeader& h = hdr[stage];
          const bool first = (gt == lo) || (t_in_seq == 0);
          h.b = b;
          h.gc = gc;
          h.tok0 = (int32_t)tok0;
          h.nvalid = nvalid;
          h.flags = (first ? kFirst : 0) | ((gt + 1 == hi || r + 1 == s1) ? kLast : 0) |
                    (gt + 1 == hi ? kCtaLast : 0);
          h.seq_k = seq_k;
          h.gt = gt;
          h.seq_t0 = (int64_t)gc * Tpg + s0;
          h.seq_t1 = (int64_t)gc * Tpg + s1;
          if (first)
            prefetch_l2(reinterpret_cast<const char*>(p.q) +
                            ((int64_t)b * p.H + (int64_t)gc * p.G * p.QPK) * D * qes,
                        qbytes);
          mbar_arrive_expect_tx(&full[stage], (uint32_t)nvalid * 2u * p.row_bytes);
        }
        // Decode step with append: the sequence's new K / V row (this g-chunk's
        // heads) goes to position context_lens[b] - 1, the last row of this
        // tile, before the tile is copied; only this CTA reads that row.
        if (STEP && p.k_new != nullptr && r + 1 == s1) {
          const int64_t cb = p.context_lens[b];
          if (cb > 0 && cb <= max_ctx) {
            const int64_t pos = cb - 1;
            const int64_t pg = page_of(pos);
            const int idx = (int)(pg - win_base);
            const int32_t a0 = __shfl_sync(0xffffffffu, win_cur, idx & 31);
            const int32_t a1 = __shfl_sync(0xffffffffu, win_next, idx & 31);
            const int64_t blk = idx < 32 ? a0 : a1;
            if (blk >= 0 && blk < p.NB) {
              const int64_t roff = blk * p.blk_stride + (pos - pg * p.BS) * p.tok_stride + (int64_t)gc * gbytes;
              T* kd = reinterpret_cast<T*>(const_cast<char*>(p.k_cache) + roff);
              T* vd = reinterpret_cast<T*>(const_cast<char*>(p.v_cache) + roff);
              const int64_t src0 = ((int64_t)b * p.HKV + (int64_t)gc * p.G) * D;
              for (int64_t e = lane; e < (int64_t)p.G * D; e += 32) {
                kd[e] = pool_from_f32<T>(io_load(io, p.k_new, src0 + e));
                vd[e] = pool_from_f32<T>(io_load(io, p.v_new, src0 + e));
              }
              // the generic-proxy stores before the bulk copies that read them
              asm volatile("fence.proxy.async.global;" ::: "memory");
            }
          }
        }
        __syncwarp();
#pragma unroll
        for (int hh = 0; hh < RPL; ++hh) {
          const int row = (lane & 15) + 16 * hh;
          if (row >= nvalid) continue;
          const int64_t off = tok0 + row - pg_r[hh] * p.BS;
          const char* src = (kv ? p.v_cache : p.k_cache) + blk_r[hh] * p.blk_stride +
                            off * p.tok_stride + (int64_t)gc * gbytes;
          unsigned char* dst = smem + (size_t)stage * stage_bytes +
                               (size_t)(kv * TT + row) * p.row_bytes;
          if (p.rows_contiguous) {
            // The g-chunk spans every KV head, so the tile's rows that share a
            // page are one contiguous run of bytes: one bulk copy per run,
            // issued by the run's first row (one K + one V copy per tile when
            // the tile size divides block_size).
            if (row == 0 || off == 0) {
              const int64_t run = min((int64_t)(nvalid - row), p.BS - off);
              bulk_g2s(dst, src, (uint32_t)run * p.row_bytes, &full[stage]);
            }
          } else {
            bulk_g2s(dst, src, p.row_bytes, &full[stage]);
          }
        }

        // On a sequence's last tile (when the range goes on): find the next
        // sequence, start loading its first block-table window and warm its q
        // in L2 now, so the switch does not wait on global memory.
        if (r + 1 == s1 && gt + 1 < hi) {
          nx_gc = gc;
          nx_b = b;
          if (r + 1 == Tpg) { ++nx_gc; nx_b = 0; }
          else ++nx_b;
          while (tile_off[nx_b + 1] == tile_off[nx_b]) ++nx_b;  // skip empty sequences
          const int32_t* nbt = p.block_tables + (int64_t)(nx_b / p.qlen) * p.MB;
          nx_cur = lane < p.MB ? __ldg(nbt + lane) : 0;
          nx_next = 32 + lane < p.MB ? __ldg(nbt + 32 + lane) : 0;
          if (lane == 0)
            prefetch_l2(reinterpret_cast<const char*>(p.q) +
                            ((int64_t)nx_b * p.H + (int64_t)nx_gc * p.G * p.QPK) * D * qes,
                        qbytes);
        }
        ++gt;
        ++r;
        if (++stage == nstage) { stage = 0; phase ^= 1; }
        if (gt < hi && r == s1) {
          if (r == Tpg) r = 0;
          gc = nx_gc;
          b = nx_b;
          s0 = tile_off[b];
          s1 = tile_off[b + 1];
          n_tok = seq_len(b);
          seq_k = ordinal(gc, b);
          bt = p.block_tables + (int64_t)(b / p.qlen) * p.MB;
          win_base = 0;  // the new sequence starts at its first page
          win_cur = nx_cur;
          win_next = nx_next;
        }
      }
    }
    if (ok && mbar_wait(&empty[stage], phase ^ 1, p.abort_flag, p.abort_tag)) {
      if (lane == 0) {
        hdr[stage].flags = kEnd;
        mbar_arrive(&full[stage]);
      }
    } else if (lane == 0) {
      // The consumers then give up on their own bounded full-barrier wait.
      // Copies already issued complete within microseconds, long before any
      // 1 s wait expires, so no copy is in flight when the CTA retires.
      report(p.dev_status, PA_DEVERR_TIMEOUT);
    }
    return;
  }

  // -------------------------------------------------------------------- consumers
  const int slot = WS ? warp - 4 : warp;
  const int slots_per_g = p.QPK / QC;
  const int g_local = slot / slots_per_g;
  const int hq0 = (slot % slots_per_g) * QC;
  const int rg = lane / R, li = lane % R;

  float qf[QC][EPL];
  float acc[QC][EPL];
  float m[QC], l[QC];
#pragma unroll
  for (int j = 0; j < QC; ++j) {
    m[j] = kNegBig;
    l[j] = 0.f;
#pragma unroll
    for (int e = 0; e < EPL; ++e) { acc[j][e] = 0.f; qf[j][e] = 0.f; }
  }

  // Arrival of a written piece of a split sequence (row pb, g-chunk pgc,
  // first head phead0, global tiles [t0, t1)); the last arriver merges.  Up to
  // kGroup pieces merge in one step.  Longer sequences merge in two levels so
  // no single warp reads every piece at the kernel's tail: the last arriver of
  // each run of kGroup consecutive pieces folds them into the run's first
  // slot, and the last run to finish merges the run results.
  const int64_t pstride = (int64_t)QC * (D + 2);
  // `wide`: called after the consumer loop, where the wide merge fits in the
  // registers (inside the loop the q and accumulator state is live).
  auto publish = [&](int pb, int pgc, int64_t phead0, int64_t t0, int64_t t1, int64_t k, bool wide) {
    const int64_t first = owner(t0, k);
    const int64_t last = owner(t1 - 1, k);
    const int64_t npieces = last - first + 1;
    // A CTA's first segment sits in partial slot 0, a later one in slot 1:
    // only the first CTA of a sequence can hold it as a later segment.
    // (tile t0 - 1 is the last tile of the previous non-empty sequence)
    const bool first_late = t0 > 0 && owner(t0 - 1, k - 1) == first;
    auto piece = [&](int64_t c) -> float* {
      const int o2 = (c == first && first_late) ? 1 : 0;
      return p.partials + ((c * 2 + o2) * NS + slot) * pstride;
    };
    auto arrive = [&](unsigned long long* counter) -> int {
      __threadfence();
      __syncwarp();
      int old = 0;
      if (lane == 0) old = epoch_arrive(counter, p.epoch, p.arrive_rounds);
      return __shfl_sync(0xffffffffu, old, 0);
    };
    // An arrival that never registered leaves its merge incomplete for every
    // warp, so this warp owns the rows: NaN, and the error bit.
    auto give_up = [&]() {
      constexpr int PERG = QC * D / 32;
#pragma unroll
      for (int k = 0; k < PERG; ++k) {
        const int j = (32 * k) / D;
        const int e = (lane + 32 * k) - j * D;
        io_store(io, p.out, ((int64_t)pb * p.H + phead0 + j) * D + e, __int_as_float(0x7fc00000));
      }
      if (p.lse && lane < QC) p.lse[(int64_t)pb * p.H + phead0 + lane] = __int_as_float(0x7fc00000);
      if (lane == 0) report(p.dev_status, PA_DEVERR_MERGE);
    };
    constexpr int PER = QC * D / 32;
    float o[PER], mg[QC], lg[QC];
    int64_t n_top = npieces, top_stride = 1;
    bool go = true;
    if (npieces > kGroup && p.grp_counters) {
      const int64_t g0 = first + ((cta - first) / kGroup) * kGroup;
      const int64_t g1 = g0 + kGroup - 1 < last ? g0 + kGroup - 1 : last;
      const int o2 = (g0 == first && first_late) ? 1 : 0;
      const int got = arrive(&p.grp_counters[(g0 * 2 + o2) * NS + slot]);
      if (got < 0) {
        give_up();
        return;
      }
      go = got == (int)(g1 - g0);
      if (go) {
        __threadfence();
        if (wide) merge_pieces_wide<QC, D, 4>(piece, g0, 1, g1 - g0 + 1, lane, o, mg, lg);
        else merge_pieces<QC, D>(piece, g0, 1, g1 - g0 + 1, lane, o, mg, lg);
        float* dst = piece(g0);  // read above; now holds the run's merged state
#pragma unroll
        for (int k = 0; k < PER; ++k) dst[lane + 32 * k] = o[k];
#pragma unroll
        for (int j = 0; j < QC; ++j)
          if (lane == j) {
            dst[QC * D + j] = mg[j];
            dst[QC * D + QC + j] = lg[j];
          }
      }
      n_top = (npieces + kGroup - 1) / kGroup;
      top_stride = kGroup;
    }
    if (!go) return;
    const int got_top = arrive(&p.counters[((int64_t)pgc * p.B + pb) * NS + slot]);
    if (got_top < 0) {
      give_up();
      return;
    }
    if (got_top == (int)(n_top - 1)) {
      __threadfence();
      if (wide) merge_pieces_wide<QC, D, 4>(piece, first, top_stride, n_top, lane, o, mg, lg);
      else merge_pieces<QC, D>(piece, first, top_stride, n_top, lane, o, mg, lg);
#pragma unroll
      for (int k = 0; k < PER; ++k) {
        const int j = (32 * k) / D;
        const int e = (lane + 32 * k) - j * D;
        io_store(io, p.out, ((int64_t)pb * p.H + phead0 + j) * D + e, o[k] / lg[j]);
      }
      if (p.lse && lane < QC) {
#pragma unroll
        for (int j = 0; j < QC; ++j)
          if (lane == j) p.lse[(int64_t)pb * p.H + phead0 + j] = (mg[j] + __log2f(lg[j])) * kLn2;
      }
    }
  };

  bool pend = false;  // the CTA's final split piece, published after the loop
  int pend_b = 0, pend_gc = 0;
  int64_t pend_head0 = 0, pend_t0 = 0, pend_t1 = 0, pend_k = 0;

  int stage = 0;
  uint32_t phase = 0;
  int seg_count = 0;
  int64_t seg_gt0 = 0;
  int b = 0, gc = 0;
  int64_t head0 = 0;
  float vsc = 1.f;  // FP8 pools: V's dequantisation scale for this KV head

  while (true) {
    if (!mbar_wait(&full[stage], phase, p.abort_flag, p.abort_tag)) {
      if (lane == 0) report(p.dev_status, PA_DEVERR_TIMEOUT);
      break;
    }
    const StageHeader h = hdr[stage];
    if (h.flags & kEnd) {
      if (pend) publish(pend_b, pend_gc, pend_head0, pend_t0, pend_t1, pend_k, true);
      break;
    }

    if (h.flags & kFirst) {
      b = h.b;
      gc = h.gc;
      seg_gt0 = h.gt;
      head0 = ((int64_t)gc * p.G + g_local) * p.QPK + hq0;
      const int64_t q0 = ((int64_t)b * p.H + head0) * D;  // element offset in q
      float qs = p.qscale;
      if constexpr (sizeof(T) == 1) {
        const int64_t kvh = (int64_t)gc * p.G + g_local;
        if (p.k_scale) qs *= p.k_scale[kvh];
        vsc = p.v_scale ? p.v_scale[kvh] : 1.f;
      }
#pragma unroll
      for (int j = 0; j < QC; ++j) {
#pragma unroll
        for (int c = 0; c < NCH; ++c) {
          const int64_t src = q0 + (int64_t)j * D + (c * R + li) * VEC;
#pragma unroll
          for (int v = 0; v < VEC; v += 2) {
            const float2 x = io_load2(io, p.q, src + v);
            qf[j][c * VEC + v] = x.x * qs;
            qf[j][c * VEC + v + 1] = x.y * qs;
          }
        }
        m[j] = kNegBig;
        l[j] = 0.f;
#pragma unroll
        for (int e = 0; e < EPL; ++e) acc[j][e] = 0.f;
      }
    }

    const unsigned char* kbase =
        smem + (size_t)stage * stage_bytes + (size_t)g_local * D * sizeof(T);
    const unsigned char* vbase = kbase + (size_t)TT * p.row_bytes;
    const int nvalid = h.nvalid;

    // scores of this row group's tokens for the QC heads (packed pairs:
    // even and odd elements accumulate separately, summed at the end)
    float s[TPR][QC];
#pragma unroll
    for (int i = 0; i < TPR; ++i) {
      const int t = rg + i * NRG;
      float2 sp[QC];
#pragma unroll
      for (int j = 0; j < QC; ++j) sp[j] = make_float2(0.f, 0.f);
      const unsigned char* kr = kbase + (size_t)t * p.row_bytes;
#pragma unroll
      for (int c = 0; c < NCH; ++c) {
        float kf[VEC];
        Chunk<T>::cvt(lds128(kr + (size_t)(c * R + li) * 16), kf);
#pragma unroll
        for (int v = 0; v < VEC; v += 2)
#pragma unroll
          for (int j = 0; j < QC; ++j)  // independent chains back to back
            sp[j] = fma2(make_float2(qf[j][c * VEC + v], qf[j][c * VEC + v + 1]),
                         make_float2(kf[v], kf[v + 1]), sp[j]);
      }
#pragma unroll
      for (int j = 0; j < QC; ++j) s[i][j] = sp[j].x + sp[j].y;
    }
#pragma unroll
    for (int off = R / 2; off >= 1; off >>= 1)
#pragma unroll
      for (int i = 0; i < TPR; ++i)
#pragma unroll
        for (int j = 0; j < QC; ++j) s[i][j] += __shfl_xor_sync(0xffffffffu, s[i][j], off);

    // Online softmax with a lazy reference max: m[j] only moves when the
    // stage's max exceeds it by more than 2^8 (then acc and l are rescaled),
    // so weights stay below 2^8 and the usual stage rescales nothing.  Any
    // reference gives the same result: out = acc / l and lse = m + log2(l)
    // are taken against the same m.
    float mt[QC];
    bool need[QC], need_any = false;
#pragma unroll
    for (int j = 0; j < QC; ++j) {
      mt[j] = kNegBig;
#pragma unroll
      for (int i = 0; i < TPR; ++i)
        if (rg + i * NRG < nvalid) mt[j] = fmaxf(mt[j], s[i][j]);
      need[j] = mt[j] > m[j] + 8.f;
      need_any |= need[j];
    }
    if (__any_sync(0xffffffffu, need_any)) {  // one vote for all heads
#pragma unroll
      for (int j = 0; j < QC; ++j) {
        const float corr = need[j] ? fast_exp2(m[j] - mt[j]) : 1.f;  // 0 on the first stage
#pragma unroll
        for (int e = 0; e < EPL; ++e) acc[j][e] *= corr;
        l[j] *= corr;
        if (need[j]) m[j] = mt[j];
      }
    }
#pragma unroll
    for (int j = 0; j < QC; ++j) {
      float lsum = 0.f;
#pragma unroll
      for (int i = 0; i < TPR; ++i) {
        const float pv = (rg + i * NRG < nvalid) ? fast_exp2(s[i][j] - m[j]) : 0.f;
        // FP8: the weight that multiplies the raw V row carries V's scale;
        // the denominator does not
        s[i][j] = sizeof(T) == 1 ? pv * vsc : pv;
        lsum += pv;
      }
      l[j] += lsum;
    }
    // P V, branch-free: a token past nvalid reads the last valid row (finite
    // data) with weight 0, so the V loads can be issued ahead of the softmax
#pragma unroll
    for (int i = 0; i < TPR; ++i) {
      const int t = rg + i * NRG;
      {
        const unsigned char* vr = vbase + (size_t)(t < nvalid ? t : nvalid - 1) * p.row_bytes;
#pragma unroll
        for (int c = 0; c < NCH; ++c) {
          float vf[VEC];
          Chunk<T>::cvt(lds128(vr + (size_t)(c * R + li) * 16), vf);
#pragma unroll
          for (int j = 0; j < QC; ++j) {
            const float2 pp = make_float2(s[i][j], s[i][j]);
#pragma unroll
            for (int v = 0; v < VEC; v += 2) {
              const float2 a = fma2(pp, make_float2(vf[v], vf[v + 1]),
                                    make_float2(acc[j][c * VEC + v], acc[j][c * VEC + v + 1]));
              acc[j][c * VEC + v] = a.x;
              acc[j][c * VEC + v + 1] = a.y;
            }
          }
        }
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[stage]);
    if (++stage == nstage) { stage = 0; phase ^= 1; }

    if (!(h.flags & kLast)) continue;

    // ---------------------------------------------------------- segment end
    // merge the row groups of this warp
#pragma unroll
    for (int off = R; off < 32; off <<= 1) {
#pragma unroll
      for (int j = 0; j < QC; ++j) {
        const float mo = __shfl_xor_sync(0xffffffffu, m[j], off);
        const float lo_ = __shfl_xor_sync(0xffffffffu, l[j], off);
        const float mn = fmaxf(m[j], mo);
        const float wa = fast_exp2(m[j] - mn), wb = fast_exp2(mo - mn);
        l[j] = l[j] * wa + lo_ * wb;
#pragma unroll
        for (int e = 0; e < EPL; ++e) {
          const float ao = __shfl_xor_sync(0xffffffffu, acc[j][e], off);
          acc[j][e] = acc[j][e] * wa + ao * wb;
        }
        m[j] = mn;
      }
    }

    const bool split = (h.seq_t0 < seg_gt0) || (h.seq_t1 > h.gt + 1);
    if (!split) {
      if (rg == 0) {
#pragma unroll
        for (int j = 0; j < QC; ++j) {
          const float inv = 1.f / l[j];
          const int64_t o = ((int64_t)b * p.H + head0 + j) * D;  // element offset in out
#pragma unroll
          for (int c = 0; c < NCH; ++c) {
#pragma unroll
            for (int v = 0; v < VEC; v += 2) {
              float2 y;
              y.x = acc[j][c * VEC + v] * inv;
              y.y = acc[j][c * VEC + v + 1] * inv;
              io_store2(io, p.out, o + (c * R + li) * VEC + v, y);
            }
          }
          if (p.lse && li == 0) p.lse[(int64_t)b * p.H + head0 + j] = (m[j] + __log2f(l[j])) * kLn2;
        }
      }
    } else {
      // Piece of a sequence split over CTAs first..last: write the partial
      // state and publish it at once (published at the kernel's end instead,
      // the arrivals of CTAs that move on to another sequence lengthen the
      // tail more than they stall the pipeline here).
      const int ord = seg_count == 0 ? 0 : 1;
      float* mine = p.partials + ((cta * 2 + ord) * NS + slot) * pstride;
      if (rg == 0) {
#pragma unroll
        for (int j = 0; j < QC; ++j) {
#pragma unroll
          for (int c = 0; c < NCH; ++c)
#pragma unroll
            for (int v = 0; v < VEC; ++v) mine[j * D + (c * R + li) * VEC + v] = acc[j][c * VEC + v];
          if (li == 0) {
            mine[QC * D + j] = m[j];
            mine[QC * D + QC + j] = l[j];
          }
        }
      }
      // The CTA's final segment is published once the loop is left (the
      // next stage is the end marker), with the wide merge.
      if (h.flags & kCtaLast) {
        pend = true;
        pend_b = b;
        pend_gc = gc;
        pend_head0 = head0;
        pend_t0 = h.seq_t0;
        pend_t1 = h.seq_t1;
        pend_k = h.seq_k;
      } else {
        publish(b, gc, head0, h.seq_t0, h.seq_t1, h.seq_k, false);
      }
    }
    ++seg_count;
  }
}

}  // namespace decode

// Kernel pointer for an instantiation (nullptr if not instantiated).
const void* decode_kernel_ptr(int dtype, int D, int QC, bool step);
int decode_max_warps(int dtype, int D, int QC);
int decode_elems_per_lane(int dtype, int D);

}  // namespace pa

namespace pa {
namespace decode {

template <typename T, int D, int QC, bool STEP>
const void* kernel_if_fits() {
  if constexpr (QC * Geo<T, D>::EPL <= (sizeof(T) <= 2 ? 64 : (sizeof(T) == 4 ? 32 : 16))) {
    return reinterpret_cast<const void*>(&decode_kernel<T, D, QC, STEP>);
  } else {
    return nullptr;
  }
}

template <typename T, int D, bool STEP>
const void* pick_qc(int QC) {
  switch (QC) {
    case 1: return kernel_if_fits<T, D, 1, STEP>();
    case 2: return kernel_if_fits<T, D, 2, STEP>();
    case 4: return kernel_if_fits<T, D, 4, STEP>();
    case 8: return kernel_if_fits<T, D, 8, STEP>();
    default: return nullptr;
  }
}

template <typename T, bool STEP>
const void* pick_kernel(int D, int QC) {
  switch (D) {
    case 32: return pick_qc<T, 32, STEP>(QC);
    case 64: return pick_qc<T, 64, STEP>(QC);
    case 128: return pick_qc<T, 128, STEP>(QC);
    case 256: return pick_qc<T, 256, STEP>(QC);
    default: return nullptr;
  }
}

}  // namespace decode
}  // namespace pa
