// prefill_pair.cu -- causal paged prefill for head_dim 128 on CTA pairs
// sharing one tensor-core MMA (tcgen05 cta_group::2), two chains per CTA.
//
// Same algorithm as prefill_tc.cu (S = Q K^T in tensor memory, P written over
// S and used as the A operand of P V, the causal rule of gb10-attn
// kernels/paged_attn_prefill.cu:62-65), laid out for two SMs and two
// independent row chains:
//
//   * A cluster of two CTAs takes 512 consecutive query rows of one (sequence,
//     head) as two chains of 256: chain c = rows 256 c .. 256 c + 255, of which
//     the even CTA ("leader") holds rows 0-127 and the odd CTA rows 128-255.
//     Each CTA keeps its two 128-row Q tiles, S tiles and O accumulators in its
//     own shared and tensor memory (TMEM: S0, S1, O0, O1 = 512 columns).
//   * The leader's MMA warp issues M = 256 MMAs for both CTAs, alternating the
//     chains: P V of chain c on tile j, then S of chain c on tile j + 1, so one
//     chain's MMAs run while the other chain's softmax works.  The B operand is
//     split between the CTAs by its N dimension: for S = Q K^T each CTA holds 64
//     of a tile's 128 keys, for O += P V one 64-column half of V; each K and V
//     tile serves all 512 rows.
//   * Softmax: warpgroup c of each CTA owns chain c (one thread per row, the
//     whole 128-key row; prefill_tc.cuh softmax_chain).
//   * Loads: warp 9 K, warp 10 V, plain tiled TMA into the CTA's own shared
//     memory (no cluster broadcast); the odd CTA's bytes count on the leader's
//     barriers through the pair form of the load.  The leader's commits arrive
//     on both CTAs' barriers; the odd CTA's softmax threads arrive on the
//     leader's q_ready and p_full barriers through their cluster addresses.
//
// Every wait is bounded (PA_DEVERR_TIMEOUT), and both CTAs meet at a cluster
// barrier before freeing the pair's tensor memory, so neither leaves while
// the other may still touch its shared or tensor memory.
#include <algorithm>
#include <mutex>
#include <vector>

#include "prefill_tc.cuh"

namespace pa {
namespace prefill {

namespace {

template <typename T>
struct PairCfg {
  static constexpr int D = 128;
  static constexpr bool SPLIT = Fmt<T>::split;
  static constexpr uint32_t Q_PART = BM * D * 2;        // one Q part: 2 halves x 128 rows x 128 B
  static constexpr uint32_t Q_CHAIN = Q_PART * (SPLIT ? 2 : 1);
  static constexpr int KROWS = BN / 2;                  // keys of a K tile per CTA
  static constexpr uint32_t K_BYTES = KROWS * D * 2;    // 2 halves x 64 rows x 128 B
  static constexpr uint32_t V_BYTES = BN * 64 * 2;      // 128 rows x 128 B (one half)
  static constexpr uint32_t GROUP_BYTES = 16 * 128;     // one TMA box: 16 rows x 128 B
  // each K / V tile serves both chains, so the rings turn at half the rate
  static constexpr int NK = SPLIT ? 3 : 5;
  static constexpr int NV = SPLIT ? 2 : 4;
  static constexpr uint32_t OFF_Q = 0;                  // [chain][hi, lo]
  static constexpr uint32_t OFF_K = 2 * Q_CHAIN;
  static constexpr uint32_t OFF_V = OFF_K + NK * K_BYTES;
  static constexpr uint32_t OFF_BAR = OFF_V + NV * V_BYTES;
  // K and V full / empty rings, per-chain s_full / p_full / o_ready, q_ready;
  // then the TMEM address and the abort flag
  static constexpr uint32_t N_BARS = 2 * NK + 2 * NV + 2 * 3 + 1;
  static constexpr uint32_t OFF_BT = OFF_BAR + ((N_BARS * 8 + 8 + 15) / 16) * 16;
  // two block-id chunks: one per loading warp (K, V)
  static constexpr uint32_t SMEM = OFF_BT + 2 * kBtChunk * 4 + 1024;  // + alignment slack
  static_assert(SMEM <= 227 * 1024, "shared memory budget");
  // TMEM columns: S of chain c at 128 c, O of chain c at 256 + D c
  static constexpr uint32_t COL_S0 = 0, COL_O = 256;
};

constexpr uint16_t kBoth = 0x3;  // CTA mask of the pair for commits

}  // namespace

// Grid: 2 CTAs per 512 query rows of one (sequence, head), clusters of 2.
template <typename T>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kThreads, 1)
    prefill_pair_kernel(const __grid_constant__ Params p) {
  using C = PairCfg<T>;
  constexpr int D = C::D, NK = C::NK, NV = C::NV;
  extern __shared__ unsigned char smem_raw[];
  unsigned char* smem = smem_raw + ((1024 - (smem_u32(smem_raw) & 1023)) & 1023);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + C::OFF_BAR);
  uint64_t* k_full = bars;            // [NK] leader: both CTAs' K halves landed
  uint64_t* k_empty = k_full + NK;    // [NK] both chains' S = Q K^T done with the stage
  uint64_t* v_full = k_empty + NK;    // [NV] leader: both V halves landed / written
  uint64_t* v_empty = v_full + NV;    // [NV] both chains' P V done with the stage
  uint64_t* s_full = v_empty + NV;    // [2] chain c: S tile in tensor memory (both CTAs)
  uint64_t* p_full = s_full + 2;      // [2] leader, chain c: P written in both CTAs
  uint64_t* o_ready = p_full + 2;     // [2] chain c: P V of its latest tile done (both CTAs)
  uint64_t* q_ready = o_ready + 2;    // leader: Q of both chains of both CTAs staged
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(q_ready + 1);
  int32_t* abort_s = reinterpret_cast<int32_t*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t rank = tc::cluster_ctarank();  // 0: leader

  // Consecutive pairs take the 512-row items of one (sequence, head),
  // longest first, so the pairs resident together share its K/V in L2.
  const int64_t c = blockIdx.x >> 1;
  const int n_items = (p.n_qtiles + 3) / 4;
  const int it = n_items - 1 - (int)(c % n_items);
  const int64_t bh = c / n_items;
  const int64_t b = bh / p.H, h = bh % p.H;
  const int64_t kv_h = h / (p.H / p.HKV);
  const int64_t item0 = (int64_t)it * 4 * BM;  // the item's first query row

  if (threadIdx.x == 0) {
    for (int s = 0; s < NK; ++s) {
      mbar_init(&k_full[s], 1);
      mbar_init(&k_empty[s], 1);
    }
    for (int s = 0; s < NV; ++s) {
      mbar_init(&v_full[s], 2);  // the leader's expect_tx + the odd CTA's arrival
      mbar_init(&v_empty[s], 1);
    }
    for (int s = 0; s < 2; ++s) {
      mbar_init(&s_full[s], 1);
      mbar_init(&p_full[s], 2 * 4);  // chain s: one arrival per warp of its warpgroup, both CTAs
      mbar_init(&o_ready[s], 1);
    }
    mbar_init(q_ready, 2 * kSoftmaxWarps * 32);
    *abort_s = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == kMmaWarp) {
    tc::tmem_alloc_pair(tmem_slot, kTmemCols);
    tc::tmem_relinquish_pair();
  }
  tc::fence_before_sync();
  // both CTAs' barriers exist before any arrival crosses the pair
  tc::cluster_sync();
  tc::fence_after_sync();
  const uint32_t tmem = *tmem_slot;

  int64_t ctx = p.context_lens[b];
  const int64_t max_ctx = p.MB * p.BS;
  if (ctx > max_ctx) {
    if (threadIdx.x == 0 && rank == 0) report(p.dev_status, PA_DEVERR_CONTEXT);
    ctx = max_ctx;
  }
  // KV tiles chain k needs: keys [0, min(ctx, ctx - Sq + its last row + 1))
  int ntile[2];
#pragma unroll
  for (int k = 0; k < 2; ++k) {
    const int64_t first = item0 + 2 * BM * k;
    const int64_t last = min(first + 2 * BM, p.Sq) - 1;
    const int64_t key_end = min(ctx, ctx - p.Sq + last + 1);
    ntile[k] = (first < p.Sq && key_end > 0) ? (int)((key_end + BN - 1) / BN) : 0;
  }
  const int n_tiles = max(ntile[0], ntile[1]);  // tiles loaded
  // the chain that uses tile j last (its S / P V releases the K / V stage)
  auto last_user = [&](int j) { return j < ntile[1] ? 1 : 0; };
  auto phys = [&](int j) { return j; };

  if (warp < kSoftmaxWarps) {
    asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(kSoftmaxRegs));
    const int grp = warp >> 2;
    softmax_chain<T, D, C>(p, smem, tmem, s_full, p_full, o_ready, q_ready, abort_s, warp, lane,
                           grp, b, h, item0 + 2 * BM * grp + (int64_t)rank * BM, ctx, ntile[grp]);
  } else {
   asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(kOtherRegs));
   if (warp == kMmaWarp) {
    // ------------------------------------------------- MMA issuer (leader only)
    if (rank == 0 && lane == 0 && n_tiles > 0) {
      constexpr uint32_t idesc_s = tc::idesc_f16(Fmt<T>::id, 2 * BM, BN, false);
      constexpr uint32_t idesc_o = tc::idesc_f16(Fmt<T>::id, 2 * BM, D, true);
      bool ok = mbar_wait_cl(q_ready, 0, abort_s);
      tc::fence_after_sync();
      int k_seen = -1, v_seen = -1;  // latest K / V tile waited for
      auto issue_s = [&](int k, int jj) -> bool {
        const int st = jj % NK;
        if (jj > k_seen) {
          if (!mbar_wait_cl(&k_full[st], (jj / NK) & 1, abort_s)) return false;
          tc::fence_after_sync();
          k_seen = jj;
        }
        // descriptors: base + (byte offset >> 4) in the start-address field
        // (shared-memory offsets stay below 2^18 bytes, so no carry)
        const uint64_t kd = tc::smem_desc_sw128(smem_u32(smem + C::OFF_K + st * C::K_BYTES), 16, 1024);
        const uint64_t qd0 = tc::smem_desc_sw128(smem_u32(smem + C::OFF_Q + k * C::Q_CHAIN), 16, 1024);
        const uint32_t dcol = tmem + C::COL_S0 + 128 * k;
#pragma unroll 1
        for (int part = 0; part < (C::SPLIT ? 2 : 1); ++part) {
          const uint64_t qd = qd0 + (uint64_t)((part * C::Q_PART) >> 4);
#pragma unroll
          for (int kk = 0; kk < D / 16; ++kk) {
            const uint32_t koff = (kk >> 2) * (C::KROWS * 128) + (kk & 3) * 32;
            const uint32_t qoff = (kk >> 2) * (BM * 128) + (kk & 3) * 32;
            tc::mma_ss_pair(dcol, qd + (qoff >> 4), kd + (koff >> 4), idesc_s, (part | kk) != 0);
          }
        }
        tc::mma_commit_pair(&s_full[k], kBoth);
        if (last_user(jj) == k) tc::mma_commit_pair(&k_empty[st], kBoth);
        return true;
      };
      for (int k = 0; k < 2 && ok; ++k)
        if (ntile[k] > 0) ok = issue_s(k, 0);
      for (int j = 0; j < n_tiles && ok; ++j) {
        for (int k = 0; k < 2 && ok; ++k) {
          if (j >= ntile[k]) continue;
          if (!mbar_wait_rx(&p_full[k], j & 1, abort_s)) { ok = false; break; }
          const int vs = j % NV;
          if (j > v_seen) {
            if (!mbar_wait_cl(&v_full[vs], (j / NV) & 1, abort_s)) { ok = false; break; }
            v_seen = j;
          }
          tc::fence_after_sync();
          const uint64_t vd = tc::smem_desc_sw128(smem_u32(smem + C::OFF_V + vs * C::V_BYTES),
                                                  BN * 128, 1024);
          const uint32_t pcol = tmem + C::COL_S0 + 128 * k;
#pragma unroll 1
          for (int part = 0; part < (C::SPLIT ? 2 : 1); ++part) {
#pragma unroll
            for (int kk = 0; kk < BN / 16; ++kk) {
              // keys 16kk .. 16kk + 15: 8 columns of packed pairs
              tc::mma_ts_pair(tmem + C::COL_O + D * k,
                              pcol + (kk >> 1) * 32 + (kk & 1) * 8 + part * 16,
                              vd + (uint64_t)((kk * 16 * 128) >> 4), idesc_o,
                              (j > 0 || part > 0 || kk > 0) ? 1u : 0u);
            }
          }
          tc::mma_commit_pair(&o_ready[k], kBoth);
          if (last_user(j) == k) tc::mma_commit_pair(&v_empty[vs], kBoth);
          // the chain's next S overwrites its P: issued after its P V, in order
          if (j + 1 < ntile[k]) ok = issue_s(k, j + 1);
        }
      }
      if (!ok) report(p.dev_status, PA_DEVERR_TIMEOUT);
    }
   } else if (warp == kTmaWarp || warp == kTmaWarp + 1) {
    // ------------------------------------- TMA producers (both CTAs): K and V
    // Warp 9 loads K, warp 10 loads V, each issuing its own copies (one warp
    // issuing both measured half the load rate the MMAs need).
    // K: lane l < 8 loads 16 keys (group l >> 1 of this CTA's 64) x half l & 1;
    // V: lane l < 8 loads 16 keys (group l of the tile's 128) x this CTA's
    // half.  The block ids are staged in shared memory as in prefill_tc.cu,
    // one chunk per warp.
    const bool is_v = warp != kTmaWarp;
    const int32_t* bt = p.block_tables + b * p.MB;
    int32_t* bt_s = reinterpret_cast<int32_t*>(smem + C::OFF_BT) + (is_v ? kBtChunk : 0);
    const int64_t n_pages = (ctx + p.BS - 1) / p.BS;
    int64_t chunk0 = -(int64_t)kBtChunk - 1;
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
    // pool row of the 16-token group at offset `toff` in tile j (0 past the context)
    auto group_row = [&](int j, int toff) -> int32_t {
      const int64_t t0 = (int64_t)phys(j) * BN;
      stage_pages(t0 / p.BS, (t0 + BN - 1) / p.BS);
      const int64_t t = t0 + toff;
      if (lane >= 8 || t >= ctx) return 0;
      const int64_t pg = t / p.BS;
      int64_t blk = bt_s[pg - chunk0];
      if (blk < 0 || blk >= p.NB) {
        report(p.dev_status, PA_DEVERR_BLOCK_ID);
        blk = 0;
      }
      return (int32_t)(blk * p.BS + (t - pg * p.BS));
    };
    const int kg = lane >> 1, khf = lane & 1;
    auto load_k = [&](int j) -> bool {
      const int st = j % NK;
      const int32_t row = group_row(j, (int)rank * C::KROWS + kg * 16);
      if (!warp_wait_t<true>(&k_empty[st], ((j / NK) & 1) ^ 1, abort_s)) return false;
      if (lane == 0 && rank == 0) mbar_arrive_expect_tx(&k_full[st], 2 * C::K_BYTES);
      __syncwarp();
      if (lane < 8) {
        unsigned char* dst = smem + C::OFF_K + st * C::K_BYTES + khf * (C::KROWS * 128) +
                             kg * C::GROUP_BYTES;
        tc::tma_load_3d_pair(dst, &p.tmap_k, khf * 64, (int32_t)kv_h, row,
                             tc::mapa_shared(&k_full[st], 0));
      }
      return true;
    };
    // A V group that reaches past the context is written by its lane
    // (v_group_sanitised: rows past the context are zeros) before the arrival.
    auto load_v = [&](int j) -> bool {
      const int st = j % NV;
      const int32_t row = group_row(j, lane * 16);
      if (!warp_wait_t<true>(&v_empty[st], ((j / NV) & 1) ^ 1, abort_s)) return false;
      unsigned char* dst = smem + C::OFF_V + st * C::V_BYTES + lane * C::GROUP_BYTES;
      const int64_t valid = ctx - ((int64_t)phys(j) * BN + lane * 16);
      const bool manual = lane < 8 && valid < 16;
      if (manual) {
        v_group_sanitised(dst, p.v_pool, row, valid, p.HKV, kv_h, (int)rank, D);
        tc::fence_proxy_async_smem();
      }
      const uint32_t boxes = __popc(__ballot_sync(0xffffffffu, lane < 8 && !manual));
      __syncwarp();
      if (lane == 0) {
        if (rank == 0)
          mbar_arrive_expect_tx(&v_full[st], 2 * boxes * C::GROUP_BYTES);
        else
          tc::mbar_arrive_cluster(tc::mapa_shared(&v_full[st], 0));
      }
      __syncwarp();
      if (lane < 8 && !manual)
        tc::tma_load_3d_pair(dst, &p.tmap_v, (int32_t)rank * 64, (int32_t)kv_h, row,
                             tc::mapa_shared(&v_full[st], 0));
      return true;
    };
    bool ok = true;
    for (int j = 0; j < n_tiles && ok; ++j) ok = is_v ? load_v(j) : load_k(j);
    if (!ok && lane == 0) report(p.dev_status, PA_DEVERR_TIMEOUT);
   }
  }

  // Both CTAs meet before the pair's tensor memory is freed: after this no
  // MMA, load or arrival of either CTA touches the other's memory.
  tc::fence_before_sync();
  tc::cluster_sync();
  if (warp == kMmaWarp) {
    tc::fence_after_sync();
    tc::tmem_dealloc_pair(tmem, kTmemCols);
  }
}

template <typename T>
static int launch_pair_typed(const Params& p, int64_t grid, cudaStream_t s) {
  using C = PairCfg<T>;
  auto kern = prefill_pair_kernel<T>;
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

// Launches the pair kernel for a head_dim 128 fp16 / bf16 pool (the caller
// built `p` and checked eligibility); one cluster of two CTAs per 512 query
// rows of each (sequence, head).
int launch_pair(const Params& p, int dtype, cudaStream_t s) {
  const int64_t n_items = (p.n_qtiles + 3) / 4;
  const int64_t grid = 2 * n_items * p.B * p.H;
  if (grid <= 0) return PA_OK;
  if (grid > (int64_t(1) << 31) - 1) return PA_ERR_TOO_LARGE;
  return dtype == PA_DTYPE_BF16 ? launch_pair_typed<__nv_bfloat16>(p, grid, s)
                                : launch_pair_typed<__half>(p, grid, s);
}

}  // namespace prefill
}  // namespace pa
