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

#include "decode_host.h"
#include "prefill_tc.cuh"

namespace pa {
namespace prefill {
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
  uint64_t* s_full = v_empty + NV;       // [2] S of tile j in TMEM (slot j % 2)
  uint64_t* p_full = s_full + 2;         // [2] P of tile j written (both softmax warpgroups)
  uint64_t* o_ready = p_full + 2;        // [2] P V of tile j done
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
      mbar_init(&p_full[s], kSoftmaxWarps * 32);  // both warpgroups per tile
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
    softmax_role<T, D, C, false>(p, smem, tmem,
                                 Bars{s_full, p_full, o_ready, q_ready, pair_bar,
                                      reinterpret_cast<float*>(smem + C::OFF_XCH)},
                                 abort_s, warp, lane, b, h, q0, ctx, n_tiles, 0);
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
            tc::mma_ts(tmem + C::COL_O, pcol + (kk >> 1) * 32 + (kk & 1) * 8 + part * 16,
                       tc::smem_desc_sw128(vb + kk * 16 * 128, BN * 128, 1024), idesc_o,
                       (j > 0 || part > 0 || kk > 0) ? 1u : 0u);
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
    // A K group past the context loads whatever row it is given (its scores
    // are masked); a V group that reaches past the context is written by its
    // lane instead (v_group_sanitised) before the stage's arrival, so its
    // rows past the context are zeros.
    auto load = [&](bool is_v, int j, int32_t row) -> bool {
      const int st = is_v ? j % NV : j % NK;
      const int n = is_v ? NV : NK;
      uint64_t* empty = is_v ? &v_empty[st] : &k_empty[st];
      uint64_t* full = is_v ? &v_full[st] : &k_full[st];
      if (!warp_wait(empty, ((j / n) & 1) ^ 1, abort_s)) return false;
      unsigned char* dst = smem + (is_v ? C::OFF_V : C::OFF_K) + st * C::KV_BYTES +
                           hf * (BN * 128) + g16 * 16 * 128;
      const int64_t valid = ctx - ((int64_t)j * BN + g16 * 16);  // tokens of the group < ctx
      const bool manual = is_v && lane < NBOX && valid < 16;
      if (manual) {
        v_group_sanitised(dst, p.v_pool, row, valid, p.HKV, kv_h, hf, D);
        tc::fence_proxy_async_smem();
      }
      const uint32_t boxes = __popc(__ballot_sync(0xffffffffu, lane < NBOX && !manual));
      __syncwarp();
      if (lane == 0) mbar_arrive_expect_tx(full, boxes * 16u * 128u);
      __syncwarp();
      if (lane < NBOX && !manual)
        tc::tma_load_3d(dst, is_v ? &p.tmap_v : &p.tmap_k, hf * 64, (int32_t)kv_h, row, full);
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

int make_map(CUtensorMap* m, const void* base, int dtype, int64_t D, int64_t HKV,
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
  p.v_pool = static_cast<const char*>(v);
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
  // head_dim 128: CTA pairs sharing each K/V tile (prefill_pair.cu)
  if (D == 128) return launch_pair(p, dtype, s);
  const int64_t grid = (int64_t)p.n_qtiles * B * H;
  if (grid <= 0) return PA_OK;
  if (grid > (int64_t(1) << 31) - 1) return PA_ERR_TOO_LARGE;
  // head_dim 64 (head_dim 128 went to the pair kernel above)
  return dtype == PA_DTYPE_BF16 ? launch_typed<__nv_bfloat16, 64>(p, grid, s)
                                : launch_typed<__half, 64>(p, grid, s);
}

}  // namespace prefill
}  // namespace pa
