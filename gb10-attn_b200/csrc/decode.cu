// decode.cu -- host side of the split-KV decode: configuration choice, the
// plan kernel (per-call work split), launch of the persistent decode kernel
// with programmatic dependent launch, and the decode entry points of the C ABI
// (pa_paged_attention, _v2, _v3, _v3_fp8, pa_choose_num_splits,
// pa_decode_workspace_size, pa_merge_states, pa_validate_block_tables).
#include <algorithm>
#include <atomic>
#include <chrono>
#include <limits>
#include <mutex>
#include <vector>

#include "decode_host.h"
#include "decode_impl.cuh"

namespace pa {

const void* decode_kernel_ptr_f16(int D, int QC, bool step);
const void* decode_kernel_ptr_bf16(int D, int QC, bool step);
const void* decode_kernel_ptr_f32(int D, int QC, bool step);
const void* decode_kernel_ptr_f64(int D, int QC, bool step);
const void* decode_kernel_ptr_e4m3(int D, int QC, bool step);

const void* decode_kernel_ptr(int dtype, int D, int QC, bool step) {
  switch (dtype) {
    case PA_DTYPE_F16: return decode_kernel_ptr_f16(D, QC, step);
    case PA_DTYPE_BF16: return decode_kernel_ptr_bf16(D, QC, step);
    case PA_DTYPE_F32: return decode_kernel_ptr_f32(D, QC, step);
    case PA_DTYPE_F64: return decode_kernel_ptr_f64(D, QC, step);
    case PA_DTYPE_E4M3: return decode_kernel_ptr_e4m3(D, QC, step);
    default: return nullptr;
  }
}

// Lane geometry mirrored on the host (must match decode::Geo / Limits).
int decode_elems_per_lane(int dtype, int D) {
  const int vec = 16 / dtype_size(dtype);
  const int ch = D / vec;
  const int r = ch <= 8 ? ch : std::min(ch / 2, 32);
  return (ch / r) * vec;
}
// Host mirrors of decode::Limits and of the QC cap in decode::kernel_if_fits.
// Returns the CTA kind (decode::CtaKind) of an instantiation.
static int decode_kind(int dtype, int D, int QC) {
  const int s = QC * decode_elems_per_lane(dtype, D);
  if (dtype_size(dtype) <= 2) return s <= (dtype_size(dtype) == 1 ? 16 : 8) ? 0 : (s <= 32 ? 1 : 2);
  return s <= 4 ? 0 : (s <= 16 ? 1 : 2);
}
static int decode_qc_cap(int dtype) {
  return dtype_size(dtype) <= 2 ? 64 : (dtype_size(dtype) == 4 ? 32 : 16);
}
int decode_max_warps(int dtype, int D, int QC) { return decode_kind(dtype, D, QC) == 2 ? 8 : 16; }

namespace decode {

constexpr int kPlanThreads = 1024;
constexpr uint32_t kStageCap = 64 * 1024;   // bytes of K+V per stage
constexpr uint32_t kRingBudget = 200 * 1024;  // bytes of stages per CTA

struct Config {
  int QC, G, NS, NGC, nstage, threads, N;
  int tt;  // tokens per tile (decode::Tile)
  int64_t n_grp;  // run counters for two-level merges (0: single-level merges)
  bool fused;     // plan built by each CTA (no plan kernel)
  uint32_t row_bytes;
  size_t smem;
  const void* kernel;
  // workspace layout (byte offsets)
  size_t off_abort, off_tile, off_cta, off_cnt, off_part, total;
};

static size_t align256(size_t x) { return (x + 255) & ~size_t(255); }
constexpr int64_t kMaxRunCounters = int64_t(1) << 20;  // 8 MB of workspace at most
// Extra tiles a sequence start costs in the weighted split: moving to another
// sequence reloads the block-table window and q and publishes a piece,
// measured at ~4-6 us on the CTAs that do it; 6 tiles measured best on the
// config-2 shape (4 and 8 within 1 %).
constexpr int kStartTiles = 6;

// Launch epoch: tags the merge counters and the abort flag of one launch, so
// no kernel has to zero them.  40 bits, never 0; starts from the clock so two
// processes sharing a workspace layout do not replay each other's tags.
// CAS rounds before a merge arrival gives up (pa_set_merge_arrive_rounds).
constexpr int kArriveRounds = 1 << 20;
static std::atomic<int> g_arrive_rounds{kArriveRounds};

static void next_epoch(unsigned long long* epoch, int32_t* abort_tag) {
  static std::atomic<unsigned long long> ctr{
      (unsigned long long)std::chrono::steady_clock::now().time_since_epoch().count() * 2654435761ull};
  unsigned long long e = ctr.fetch_add(1) & ((1ull << (64 - kCountBits)) - 1);
  if (e == 0) e = 1;
  *epoch = e;
  *abort_tag = (int32_t)(1 + e % 0x7ffffffeull);
}

struct PlanParams {
  const int32_t* context_lens;
  int32_t* tile_off;   // [B + 1]
  int32_t* cta_seq;    // [N]
  float* out;          // rows of empty sequences are filled with empty_fill
  float* lse;
  int32_t* dev_status;
  int64_t B, H, D, max_ctx, qlen;
  int32_t NGC, N;
  int32_t tt;  // tokens per tile
  float empty_fill;
  int32_t io_dtype;  // element type of out
};

// One CTA: tile counts -> exclusive scan -> tile_off; the sequence holding
// each CTA's first tile; NaN rows for empty
// sequences (the reference's v3 yields NaN there, paged_attn_v3.cu:160-165).
__global__ void __launch_bounds__(kPlanThreads) plan_kernel(const __grid_constant__ PlanParams pp) {
  // Launched with programmatic stream serialisation: let the decode kernel
  // start launching at once, and wait for the previous kernel on the stream
  // (which may still use this workspace or write context_lens) before
  // touching memory.
  pdl_trigger();
  pdl_wait();
  __shared__ int32_t warp_tot[kPlanThreads / 32];
  __shared__ int32_t carry_s;
  const int tid = threadIdx.x, lane = tid & 31, wid = tid >> 5;
  if (tid == 0) carry_s = 0;
  __syncthreads();
  for (int64_t base = 0; base < pp.B; base += kPlanThreads) {
    const int64_t b = base + tid;
    int32_t tiles = 0;
    if (b < pp.B) {
      const int64_t sq = b / pp.qlen;
      const int64_t c = pp.context_lens[sq];
      if (c > pp.max_ctx && b == sq * pp.qlen) report(pp.dev_status, PA_DEVERR_CONTEXT);
      int64_t n = c - pp.qlen + (b - sq * pp.qlen) + 1;
      if (n > pp.max_ctx) n = pp.max_ctx;
      if (n <= 0) {
        n = 0;
        for (int64_t i = 0; i < pp.H * pp.D; ++i) io_store(pp.io_dtype, pp.out, b * pp.H * pp.D + i, pp.empty_fill);
        if (pp.lse)
          for (int64_t h = 0; h < pp.H; ++h) pp.lse[b * pp.H + h] = -INFINITY;
      }
      tiles = (int32_t)((n + pp.tt - 1) / pp.tt);
    }
    int32_t x = tiles;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int32_t y = __shfl_up_sync(0xffffffffu, x, o);
      if (lane >= o) x += y;
    }
    if (lane == 31) warp_tot[wid] = x;
    __syncthreads();
    if (wid == 0) {
      int32_t w = warp_tot[lane];
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int32_t y = __shfl_up_sync(0xffffffffu, w, o);
        if (lane >= o) w += y;
      }
      warp_tot[lane] = w;  // inclusive over warps
    }
    __syncthreads();
    const int32_t carry = carry_s;
    const int32_t excl = carry + (wid ? warp_tot[wid - 1] : 0) + x - tiles;
    if (b < pp.B) pp.tile_off[b] = excl;
    __syncthreads();
    if (tid == kPlanThreads - 1) carry_s = carry + warp_tot[kPlanThreads / 32 - 1];
    __syncthreads();
  }
  if (tid == 0) pp.tile_off[pp.B] = carry_s;
  __syncthreads();
  const int64_t Tpg = carry_s;
  const int64_t T_all = Tpg * pp.NGC;
  for (int64_t c = tid; c < pp.N; c += kPlanThreads) {
    const int64_t lo = cta_lo(c, T_all, pp.N);
    int32_t seq = 0;
    if (lo < T_all) {
      const int64_t r = lo % Tpg;
      // upper_bound(tile_off[0..B], r) - 1
      int64_t a = 0, z = pp.B + 1;
      while (a < z) {
        const int64_t mid = (a + z) >> 1;
        if (pp.tile_off[mid] <= r) a = mid + 1;
        else z = mid;
      }
      seq = (int32_t)(a - 1);
    }
    pp.cta_seq[c] = seq;
  }
}

static std::mutex g_mu;

// Opt a kernel into the large dynamic shared-memory carve-out, once per
// (device, kernel).  Caller holds g_mu.
static int ensure_smem_attr_locked(int dev, const void* kernel) {
  static std::vector<std::pair<int, const void*>> done;
  for (auto& a : done)
    if (a.first == dev && a.second == kernel) return PA_OK;
  cudaError_t e =
      cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024);
  if (e != cudaSuccess) return cuda_status(e);
  done.push_back({dev, kernel});
  return PA_OK;
}

static int ensure_smem_attr(const void* kernel) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_status(e);
  std::lock_guard<std::mutex> lk(g_mu);
  return ensure_smem_attr_locked(dev, kernel);
}

// Blocks per SM for (kernel, threads, smem); sets the dynamic smem limit once
// per (device, kernel).
static int occupancy(const void* kernel, int threads, size_t smem, int* blocks) {
  struct Key {
    int dev;
    const void* k;
    int threads;
    size_t smem;
    int blocks;
  };
  static std::vector<Key> cache;
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_status(e);
  std::lock_guard<std::mutex> lk(g_mu);
  for (const Key& k : cache)
    if (k.dev == dev && k.k == kernel && k.threads == threads && k.smem == smem) {
      *blocks = k.blocks;
      return PA_OK;
    }
  int st = ensure_smem_attr_locked(dev, kernel);
  if (st) return st;
  int nb = 0;
  e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&nb, kernel, threads, smem);
  if (e != cudaSuccess) return cuda_status(e);
  if (nb < 1) nb = 1;
  cache.push_back({dev, kernel, threads, smem, nb});
  *blocks = nb;
  return PA_OK;
}

static int check_args(const DecodeArgs& a) {
  if (a.B < 0 || a.H <= 0 || a.HKV <= 0 || a.D <= 0 || a.BS <= 0 || a.NB < 0 || a.MB < 0)
    return PA_ERR_INVALID_ARGUMENT;
  if (a.H % a.HKV != 0) return PA_ERR_NUM_HEADS;
  if (a.D != 32 && a.D != 64 && a.D != 128 && a.D != 256) return PA_ERR_HEAD_DIM;
  if (dtype_size(a.dtype) == 0) return PA_ERR_DTYPE;
  if (a.qlen < 1) return PA_ERR_INVALID_ARGUMENT;
  if (a.io_dtype != PA_DTYPE_F32 && a.io_dtype != PA_DTYPE_F16 && a.io_dtype != PA_DTYPE_BF16)
    return PA_ERR_DTYPE;
  // the step's append: decode only, both rows or neither, a pool it writes
  // without scales (FP8 pools take pa_append_kv)
  if ((a.k_new == nullptr) != (a.v_new == nullptr) || (a.k_new && a.qlen != 1))
    return PA_ERR_INVALID_ARGUMENT;
  if (a.k_new && a.dtype == PA_DTYPE_E4M3) return PA_ERR_DTYPE;
  if (a.B * a.qlen > (int64_t(1) << 30) || a.MB * a.BS > (int64_t(1) << 31) - 2 * kTT)
    return PA_ERR_TOO_LARGE;
  return PA_OK;
}

// Chooses the instantiation and the per-call geometry; fills the workspace
// layout.  Needs the current device (SM count, occupancy).
static int configure(const DecodeArgs& a, Config* c) {
  const int elt = dtype_size(a.dtype);
  const int QPK = (int)(a.H / a.HKV);
  const int epl = decode_elems_per_lane(a.dtype, (int)a.D);
  // Query heads per consumer warp: the largest group whose state fits (each
  // KV row is then read from shared memory by the fewest warps).  Measured on
  // config 3: 8 warps x 4 heads and 16 warps x 2 heads run at the same speed.
  auto pick_g = [&](int qc) {
    const int maxw = decode_max_warps(a.dtype, (int)a.D, qc);
    const int tq = tile_tokens(a.dtype, qc);
    for (int g = (int)std::min<int64_t>(a.HKV, 64); g >= 1; --g) {
      if (a.HKV % g) continue;
      if (g * (QPK / qc) > maxw) continue;
      if (2u * tq * (uint32_t)(g * a.D * elt) > kStageCap) continue;
      return g;
    }
    return 0;
  };
  int QC = 1, G = 0, best_ns = -1;
  for (int qc : {8, 4, 2, 1}) {
    if (QPK % qc || qc * epl > decode_qc_cap(a.dtype)) continue;
    const int g = pick_g(qc);
    if (g == 0) continue;
    best_ns = g * (QPK / qc);
    QC = qc;
    G = g;
    break;
  }
  (void)best_ns;
  if (G == 0) return PA_ERR_TOO_LARGE;  // QPK / QC beyond one CTA
  const int maxw = decode_max_warps(a.dtype, (int)a.D, QC);
  const int tt = tile_tokens(a.dtype, QC);
  c->tt = tt;
  c->QC = QC;
  c->G = G;
  c->NS = G * (QPK / QC);
  if (c->NS > maxw) return PA_ERR_TOO_LARGE;  // QPK / QC beyond one CTA
  c->NGC = (int)(a.HKV / G);
  c->row_bytes = (uint32_t)(G * a.D * elt);
  const uint32_t stage_bytes = 2u * tt * c->row_bytes;
  c->nstage = (int)std::max<uint32_t>(2, std::min<uint32_t>(8, kRingBudget / stage_bytes));
  // must match decode::Limits
  {
    const int kind = decode_kind(a.dtype, (int)a.D, QC);
    c->threads = kind == 2 ? 384 : (kind == 1 ? 640 : (c->NS + 1) * 32);
  }
  c->smem = (size_t)c->nstage * stage_bytes + (size_t)c->nstage * (16 + sizeof(StageHeader));
  // the decode-step instantiation only when the call needs it
  const bool step = a.io_dtype != PA_DTYPE_F32 || a.k_new != nullptr;
  c->kernel = decode_kernel_ptr(a.dtype, (int)a.D, QC, step);
  if (!c->kernel) return PA_ERR_HEAD_DIM;

  const int64_t rows = a.B * a.qlen;
  const int64_t max_tiles = (a.MB * a.BS + tt - 1) / tt;
  const int64_t t_upper = std::max<int64_t>(1, (int64_t)c->NGC * rows * max_tiles);
  int64_t N;
  if (a.num_splits <= 0) {
    int sms = 0, per_sm = 1;
    int st = device_sm_count(&sms);
    if (st) return st;
    st = occupancy(c->kernel, c->threads, c->smem, &per_sm);
    if (st) return st;
    N = (int64_t)sms * per_sm;
  } else {
    N = rows * c->NGC * std::min<int64_t>(a.num_splits, 1 << 16);
  }
  N = std::max<int64_t>(1, std::min<int64_t>(N, t_upper));
  // keeps c * T_all (CTA range arithmetic) far inside int64
  if (N > (int64_t(1) << 24) || t_upper > (int64_t(1) << 36)) return PA_ERR_TOO_LARGE;
  c->N = (int)N;

  // Small batches: every CTA builds the plan in shared memory (no plan
  // kernel, tables beside the stage headers).
  c->fused = rows <= kFusedRows;
  // (scan scratch, then tile offsets, key counts, non-empty prefix)
  if (c->fused) c->smem += kPlanScratchBytes + sizeof(int32_t) * (size_t)(3 * rows + 2);

  size_t off = 0;
  c->off_abort = off;
  off = align256(off + sizeof(int32_t));
  c->off_tile = off;
  if (!c->fused) off = align256(off + sizeof(int32_t) * (size_t)(rows + 1));
  c->off_cta = off;
  if (!c->fused) off = align256(off + sizeof(int32_t) * (size_t)N);
  c->off_cnt = off;
  // epoch-tagged merge counters per (g-chunk, row, slot), then per (CTA,
  // slot) run counters for two-level merges (bounded workspace)
  c->n_grp = (N * 2 * c->NS <= kMaxRunCounters) ? N * 2 * c->NS : 0;
  off = align256(off + sizeof(unsigned long long) * ((size_t)c->NGC * rows * c->NS + (size_t)c->n_grp));
  c->off_part = off;
  off = align256(off + sizeof(float) * (size_t)N * 2 * c->NS * QC * (a.D + 2));
  c->total = off;
  return PA_OK;
}

int launch(const DecodeArgs& a, void* ws, size_t ws_bytes, cudaStream_t stream) {
  int st = check_args(a);
  if (st) return st;
  if (a.B == 0) return PA_OK;
  if (!a.out || !a.q || !a.k_cache || !a.v_cache || !a.block_tables || !a.context_lens)
    return PA_ERR_INVALID_ARGUMENT;
  if (!aligned16(a.k_cache) || !aligned16(a.v_cache) || !aligned16(a.q) || !aligned16(a.out))
    return PA_ERR_ALIGNMENT;
  Config c;
  st = configure(a, &c);
  if (st) return st;
  if (!ws || ws_bytes < c.total || !aligned16(ws)) return PA_ERR_WORKSPACE;
  st = ensure_smem_attr(c.kernel);
  if (st) return st;

  char* w = static_cast<char*>(ws);
  PlanParams pp;
  pp.context_lens = a.context_lens;
  pp.tile_off = reinterpret_cast<int32_t*>(w + c.off_tile);
  pp.cta_seq = reinterpret_cast<int32_t*>(w + c.off_cta);
  pp.out = a.out;
  pp.lse = a.lse;
  pp.dev_status = a.dev_status;
  pp.B = a.B * a.qlen;
  pp.H = a.H;
  pp.D = a.D;
  pp.max_ctx = a.MB * a.BS;
  pp.qlen = a.qlen;
  pp.NGC = c.NGC;
  pp.N = c.N;
  pp.empty_fill = a.empty_fill;
  pp.tt = c.tt;
  pp.io_dtype = a.io_dtype;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cudaError_t e;
  if (!c.fused) {
    cudaLaunchConfig_t pcfg = {};
    pcfg.gridDim = dim3(1);
    pcfg.blockDim = dim3(kPlanThreads);
    pcfg.stream = stream;
    pcfg.attrs = attr;
    pcfg.numAttrs = 1;
    e = cudaLaunchKernelEx(&pcfg, plan_kernel, pp);
    if (e != cudaSuccess) return cuda_status(e);
  }

  Params p;
  p.out = a.out;
  p.lse = a.lse;
  p.q = a.q;
  p.k_cache = static_cast<const char*>(a.k_cache);
  p.v_cache = static_cast<const char*>(a.v_cache);
  p.block_tables = a.block_tables;
  p.context_lens = a.context_lens;
  p.dev_status = a.dev_status;
  p.tile_off = c.fused ? nullptr : pp.tile_off;
  p.cta_seq = c.fused ? nullptr : pp.cta_seq;
  p.counters = reinterpret_cast<unsigned long long*>(w + c.off_cnt);
  p.grp_counters = c.n_grp ? p.counters + (int64_t)c.NGC * pp.B * c.NS : nullptr;
  p.abort_flag = reinterpret_cast<int32_t*>(w + c.off_abort);
  next_epoch(&p.epoch, &p.abort_tag);
  p.arrive_rounds = g_arrive_rounds.load(std::memory_order_relaxed);
  p.empty_fill = a.empty_fill;
  // the start cost is in 16-token tiles: fewer of the larger FP8 tiles
  p.beta = c.fused ? kStartTiles * kTT / c.tt : 0;
  p.partials = reinterpret_cast<float*>(w + c.off_part);
  p.B = a.B * a.qlen;
  p.qlen = a.qlen;
  p.H = a.H;
  p.HKV = a.HKV;
  p.NB = a.NB;
  p.MB = a.MB;
  p.BS = a.BS;
  p.G = c.G;
  p.QPK = (int32_t)(a.H / a.HKV);
  p.NS = c.NS;
  p.NGC = c.NGC;
  p.N = c.N;
  p.nstage = c.nstage;
  p.qscale = (float)a.scale * kLog2e;
  p.k_scale = a.k_scale;
  p.v_scale = a.v_scale;
  p.row_bytes = c.row_bytes;
  p.rows_contiguous = (c.G == a.HKV) ? 1 : 0;
  const int elt = dtype_size(a.dtype);
  p.tok_stride = a.HKV * a.D * elt;
  p.bs_shift = -1;
  if ((a.BS & (a.BS - 1)) == 0)
    for (int sh = 0; sh < 32; ++sh)
      if ((int64_t(1) << sh) == a.BS) p.bs_shift = sh;
  p.blk_stride = a.BS * p.tok_stride;
  p.io_dtype = a.io_dtype;
  p.k_new = static_cast<const char*>(a.k_new);
  p.v_new = static_cast<const char*>(a.v_new);

  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)c.N);
  cfg.blockDim = dim3((unsigned)c.threads);
  cfg.dynamicSmemBytes = c.smem;
  cfg.stream = stream;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  void* args[] = {&p};
  e = cudaLaunchKernelExC(&cfg, c.kernel, args);
  if (e != cudaSuccess) return cuda_status(e);
  return PA_OK;
}

int workspace_bytes(const DecodeArgs& a, size_t* bytes) {
  int st = check_args(a);
  if (st) return st;
  if (a.B == 0) {
    *bytes = 0;
    return PA_OK;
  }
  Config c;
  st = configure(a, &c);
  if (st) return st;
  *bytes = c.total;
  return PA_OK;
}

// ---------------------------------------------------------------------------
// cross-device state merge and block-table validation
// ---------------------------------------------------------------------------

__global__ void merge_states_kernel(float* __restrict__ out, float* __restrict__ lse_out,
                                    const float* __restrict__ outs,
                                    const float* __restrict__ lses, int64_t parts,
                                    int64_t rows, int64_t D) {
  const int64_t warps = (int64_t)gridDim.x * (blockDim.x >> 5);
  const int lane = threadIdx.x & 31;
  for (int64_t row = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); row < rows;
       row += warps) {
    float mx = -INFINITY;
    for (int64_t r = 0; r < parts; ++r) mx = fmaxf(mx, lses[r * rows + row]);
    float den = 0.f;
    for (int64_t r = 0; r < parts; ++r) {
      const float lr = lses[r * rows + row];
      den += (lr == -INFINITY) ? 0.f : __expf(lr - mx);
    }
    for (int64_t d = lane; d < D; d += 32) {
      float num = 0.f;
      for (int64_t r = 0; r < parts; ++r) {
        const float lr = lses[r * rows + row];
        if (lr != -INFINITY) num += __expf(lr - mx) * outs[(r * rows + row) * D + d];
      }
      out[row * D + d] = num / den;  // den == 0 (all parts empty) -> NaN
    }
    if (lse_out && lane == 0) lse_out[row] = (den > 0.f) ? mx + __logf(den) : -INFINITY;
  }
}

__global__ void validate_kernel(const int32_t* __restrict__ bt, const int32_t* __restrict__ ctx,
                                int64_t B, int64_t MB, int64_t BS, int64_t NB,
                                int32_t* __restrict__ counts) {
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < B * MB; i += stride) {
    const int64_t b = i / MB, m = i % MB;
    const int64_t n = ctx[b];
    if (m == 0 && n > MB * BS) atomicAdd(&counts[1], 1);
    const int64_t used = n <= 0 ? 0 : ((n < MB * BS ? n : MB * BS) + BS - 1) / BS;
    if (m < used) {
      const int32_t v = bt[i];
      if (v < 0 || v >= NB) atomicAdd(&counts[0], 1);
    }
  }
}

}  // namespace decode
}  // namespace pa

// ---------------------------------------------------------------------------
// C ABI
// ---------------------------------------------------------------------------

using pa::decode::DecodeArgs;

extern "C" int pa_set_merge_arrive_rounds(int rounds) {
  return pa::decode::g_arrive_rounds.exchange(rounds < 0 ? pa::decode::kArriveRounds : rounds);
}

extern "C" int64_t pa_choose_num_splits(int64_t num_seqs, int64_t num_heads,
                                        int64_t max_context) {
  int sms = 0;
  if (pa::device_sm_count(&sms) != PA_OK) return -1;
  // kernels/paged_attn_v3.cu:181-189
  const int64_t have = std::max<int64_t>(num_seqs * num_heads, 1);
  const int64_t by_chain = std::max<int64_t>(max_context / 32, 1);
  const int64_t to_fill = std::max<int64_t>(((int64_t)sms * 8 + have - 1) / have, 1);
  const int64_t s = std::max(by_chain, to_fill);
  return std::max<int64_t>(1, std::min<int64_t>(s, 64));
}

extern "C" int pa_decode_workspace_size(int64_t num_seqs, int64_t num_heads,
                                        int64_t num_kv_heads, int64_t head_dim, int kv_dtype,
                                        int64_t block_size, int64_t max_blocks,
                                        int64_t num_splits, size_t* bytes) {
  if (!bytes) return PA_ERR_INVALID_ARGUMENT;
  DecodeArgs a = {};
  a.dtype = kv_dtype;
  a.B = num_seqs;
  a.H = num_heads;
  a.HKV = num_kv_heads;
  a.D = head_dim;
  a.BS = block_size;
  a.NB = 1;
  a.MB = max_blocks;
  a.num_splits = num_splits;
  return pa::decode::workspace_bytes(a, bytes);
}

static int decode_entry(float* out, float* lse, const float* q, const void* k, const void* v,
                        int dt, const int32_t* bt, const int32_t* ctx, int64_t B, int64_t H,
                        int64_t HKV, int64_t D, int64_t BS, int64_t NB, int64_t MB,
                        double scale, int64_t num_splits, void* ws, size_t ws_bytes,
                        int32_t* dev_status, void* stream, const float* k_scale = nullptr,
                        const float* v_scale = nullptr) {
  DecodeArgs a;
  a.k_scale = k_scale;
  a.v_scale = v_scale;
  a.out = out;
  a.lse = lse;
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
  a.num_splits = num_splits;
  a.dev_status = dev_status;
  a.qlen = 1;
  a.empty_fill = std::numeric_limits<float>::quiet_NaN();  // as the reference's v3
  return pa::decode::launch(a, ws, ws_bytes, static_cast<cudaStream_t>(stream));
}

extern "C" int pa_paged_attention_v3(float* out, float* lse, const float* q, const void* k_cache,
                                     const void* v_cache, int kv_dtype,
                                     const int32_t* block_tables, const int32_t* context_lens,
                                     int64_t num_seqs, int64_t num_heads, int64_t num_kv_heads,
                                     int64_t head_dim, int64_t block_size, int64_t num_blocks,
                                     int64_t max_blocks, double scale, int64_t num_splits,
                                     void* workspace, size_t workspace_bytes,
                                     int32_t* dev_status, void* stream) {
  return decode_entry(out, lse, q, k_cache, v_cache, kv_dtype, block_tables, context_lens,
                      num_seqs, num_heads, num_kv_heads, head_dim, block_size, num_blocks,
                      max_blocks, scale, num_splits, workspace, workspace_bytes, dev_status,
                      stream);
}

// One layer of a decode step (an addition): q / out in io_dtype, and when
// k_new / v_new are given, sequence b's new K / V row written at position
// context_lens[b] - 1 of its pages inside the same launch, before the tile
// that holds it is read.
extern "C" int pa_decode_layer_step(void* out, float* lse, const void* q, int io_dtype,
                                    void* k_cache, void* v_cache, int kv_dtype,
                                    const void* k_new, const void* v_new,
                                    const int32_t* block_tables, const int32_t* context_lens,
                                    int64_t num_seqs, int64_t num_heads, int64_t num_kv_heads,
                                    int64_t head_dim, int64_t block_size, int64_t num_blocks,
                                    int64_t max_blocks, double scale, int64_t num_splits,
                                    void* workspace, size_t workspace_bytes, int32_t* dev_status,
                                    void* stream) {
  DecodeArgs a;
  a.out = static_cast<float*>(out);
  a.lse = lse;
  a.q = static_cast<const float*>(q);
  a.k_cache = k_cache;
  a.v_cache = v_cache;
  a.dtype = kv_dtype;
  a.block_tables = block_tables;
  a.context_lens = context_lens;
  a.B = num_seqs;
  a.H = num_heads;
  a.HKV = num_kv_heads;
  a.D = head_dim;
  a.BS = block_size;
  a.NB = num_blocks;
  a.MB = max_blocks;
  a.scale = scale;
  a.num_splits = num_splits;
  a.dev_status = dev_status;
  a.qlen = 1;
  a.empty_fill = std::numeric_limits<float>::quiet_NaN();  // as pa_paged_attention_v3
  a.io_dtype = io_dtype;
  a.k_new = k_new;
  a.v_new = v_new;
  return pa::decode::launch(a, workspace, workspace_bytes, static_cast<cudaStream_t>(stream));
}

extern "C" int pa_paged_attention_v3_fp8(float* out, float* lse, const float* q,
                                         const void* k_cache, const void* v_cache,
                                         const float* k_scale, const float* v_scale,
                                         int kv_dtype, const int32_t* block_tables,
                                         const int32_t* context_lens, int64_t num_seqs,
                                         int64_t num_heads, int64_t num_kv_heads,
                                         int64_t head_dim, int64_t block_size,
                                         int64_t num_blocks, int64_t max_blocks, double scale,
                                         int64_t num_splits, void* workspace,
                                         size_t workspace_bytes, int32_t* dev_status,
                                         void* stream) {
  if (kv_dtype != PA_DTYPE_E4M3) return PA_ERR_DTYPE;
  return decode_entry(out, lse, q, k_cache, v_cache, kv_dtype, block_tables, context_lens,
                      num_seqs, num_heads, num_kv_heads, head_dim, block_size, num_blocks,
                      max_blocks, scale, num_splits, workspace, workspace_bytes, dev_status,
                      stream, k_scale, v_scale);
}

extern "C" int pa_paged_attention(float* out, const float* q, const void* k_cache,
                                  const void* v_cache, int kv_dtype, const int32_t* block_tables,
                                  const int32_t* context_lens, int64_t num_seqs,
                                  int64_t num_heads, int64_t num_kv_heads, int64_t head_dim,
                                  int64_t block_size, int64_t num_blocks, int64_t max_blocks,
                                  double scale, void* workspace, size_t workspace_bytes,
                                  int32_t* dev_status, void* stream) {
  return decode_entry(out, nullptr, q, k_cache, v_cache, kv_dtype, block_tables, context_lens,
                      num_seqs, num_heads, num_kv_heads, head_dim, block_size, num_blocks,
                      max_blocks, scale, 0, workspace, workspace_bytes, dev_status, stream);
}

extern "C" int pa_paged_attention_v2(float* out, const float* q, const void* k_cache,
                                     const void* v_cache, int kv_dtype,
                                     const int32_t* block_tables, const int32_t* context_lens,
                                     int64_t num_seqs, int64_t num_heads, int64_t num_kv_heads,
                                     int64_t head_dim, int64_t block_size, int64_t num_blocks,
                                     int64_t max_blocks, double scale, void* workspace,
                                     size_t workspace_bytes, int32_t* dev_status,
                                     void* stream) {
  return decode_entry(out, nullptr, q, k_cache, v_cache, kv_dtype, block_tables, context_lens,
                      num_seqs, num_heads, num_kv_heads, head_dim, block_size, num_blocks,
                      max_blocks, scale, 0, workspace, workspace_bytes, dev_status, stream);
}

extern "C" int pa_merge_states(float* out, float* lse_out, const float* outs, const float* lses,
                               int64_t num_parts, int64_t rows, int64_t head_dim, void* stream) {
  if (num_parts < 1 || rows < 0 || head_dim <= 0 || !out || !outs || !lses)
    return PA_ERR_INVALID_ARGUMENT;
  if (rows == 0) return PA_OK;
  const int threads = 256;
  const int64_t blocks = std::min<int64_t>((rows + 7) / 8, 65535);
  pa::decode::merge_states_kernel<<<(unsigned)blocks, threads, 0,
                                     static_cast<cudaStream_t>(stream)>>>(
      out, lse_out, outs, lses, num_parts, rows, head_dim);
  return pa::cuda_status(cudaGetLastError());
}

extern "C" int pa_validate_block_tables(const int32_t* block_tables, const int32_t* context_lens,
                                        int64_t num_seqs, int64_t max_blocks,
                                        int64_t block_size, int64_t num_blocks, int32_t* counts,
                                        void* stream) {
  if (num_seqs < 0 || max_blocks < 0 || block_size <= 0 || !counts) return PA_ERR_INVALID_ARGUMENT;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  cudaError_t e = cudaMemsetAsync(counts, 0, 2 * sizeof(int32_t), s);
  if (e != cudaSuccess) return pa::cuda_status(e);
  if (num_seqs == 0 || max_blocks == 0) return PA_OK;
  if (!block_tables || !context_lens) return PA_ERR_INVALID_ARGUMENT;
  const int64_t n = num_seqs * max_blocks;
  const int64_t blocks = std::min<int64_t>((n + 255) / 256, 4096);
  pa::decode::validate_kernel<<<(unsigned)blocks, 256, 0, s>>>(
      block_tables, context_lens, num_seqs, max_blocks, block_size, num_blocks, counts);
  return pa::cuda_status(cudaGetLastError());
}
