// peer_merge.cu -- the cross-GPU step of the sequence-sharded decode, on peer
// memory instead of a collective.
//
// Every rank of a job owns one exchange buffer in its own HBM, mapped into
// every other rank's address space (CUDA IPC, pa_ipc_*):
//
//   [slot 0][slot 1][flags: world x u32]
//   slot = out [rows, D] fp32 | pad to 256 B | lse [rows] fp32 | pad to 256 B
//
// A step with epoch e (1, 2, 3, ... the same sequence on every rank):
//   1. the rank's decode writes its normalised partial (out, lse) of its own
//      token range into slot e & 1 of its OWN buffer (plain local stores);
//   2. pa_merge_peer_partials, one small launch (a programmatic dependent of
//      the decode, so its launch overlaps the decode's tail): every CTA stores
//      e into flags[rank] of every peer's buffer (st.release.sys over NVLink), waits,
//      bounded, until its own flags[p] >= e for every p (ld.acquire.sys, local),
//      reads every rank's slot e & 1 with plain peer loads, and merges the rows
//      with the log-sum-exp rule of kernels/paged_attn_v3.cu:139-165 (the
//      reference's merge_splits_kernel, here over ranks instead of splits).
//
// Reuse is safe with two slots: a rank writes slot e & 1 again at step e + 2
// only after its merge of step e + 1 has seen every peer's flag e + 1, and a
// peer raises that flag only after its own merge of step e (the last reader
// of that slot) has finished, in stream order.  A peer is at most one epoch
// ahead, so the flags compare with >= (serial-number arithmetic), not ==.
//
// No TMA of any form reads peer memory: peer data move only through ordinary
// ld.global (non-caching, .cv) loads.  Every wait gives up after 1 s, writes
// NaN rows and reports PA_DEVERR_TIMEOUT.
#include <math.h>
#include <string.h>

#include <algorithm>

#include "common.cuh"

namespace pa {
namespace peer {

constexpr int kMaxWorld = 32;  // one lane per rank in the lse reduction
constexpr size_t kAlign = 256;

__host__ __device__ inline size_t round_up(size_t x, size_t a) { return (x + a - 1) / a * a; }

struct Layout {
  size_t lse_offset, slot_bytes, flags_offset, total_bytes;
};

inline Layout layout(int64_t rows, int64_t D) {
  Layout l;
  l.lse_offset = round_up((size_t)rows * (size_t)D * sizeof(float), kAlign);
  l.slot_bytes = round_up(l.lse_offset + (size_t)rows * sizeof(float), kAlign);
  l.flags_offset = 2 * l.slot_bytes;
  l.total_bytes = l.flags_offset + round_up(kMaxWorld * sizeof(uint32_t), kAlign);
  return l;
}

__device__ __forceinline__ void st_release_sys(uint32_t* p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ bool reached(uint32_t flag, uint32_t epoch) {
  return (int32_t)(flag - epoch) >= 0;
}

__global__ void __launch_bounds__(256)
    merge_peers_kernel(float* __restrict__ out, float* __restrict__ lse_out,
                       const unsigned long long* __restrict__ bases, int world, int rank,
                       int64_t rows, int D, int64_t lse_offset, int64_t slot_bytes,
                       int64_t flags_offset, uint32_t epoch, int32_t* dev_status) {
  __shared__ int s_fail;
  __shared__ const char* s_slot[kMaxWorld];
  __shared__ float s_w[8][kMaxWorld];  // per warp: the current row's rank weights
  const int t = threadIdx.x;
  if (t == 0) s_fail = 0;
  // Launched as a programmatic dependent of the decode that wrote this rank's
  // partial: the launch overlaps that kernel's tail, and nothing below runs
  // before it has completed and its stores are visible.  The next kernel on
  // the stream may launch now (it waits for this grid before touching memory).
  pdl_wait();
  pdl_trigger();
  if (t < world) {
    // 1. tell rank t that this rank's partial of `epoch` is in place.  The
    //    decode that wrote it finished before this launch (stream order); the
    //    system-scope fence orders those stores before the flag for a reader
    //    on another GPU.
    char* peer = reinterpret_cast<char*>(bases[t]);
    __threadfence_system();
    st_release_sys(reinterpret_cast<uint32_t*>(peer + flags_offset) + rank, epoch);
    s_slot[t] = peer + (int64_t)(epoch & 1u) * slot_bytes;
  }
  __syncthreads();
  if (t < world) {
    // 2. wait for rank t's flag in this rank's own buffer (a local load).
    const uint32_t* mine =
        reinterpret_cast<const uint32_t*>(reinterpret_cast<const char*>(bases[rank]) +
                                          flags_offset) + t;
    if (!reached(ld_acquire_sys(mine), epoch)) {
      const uint64_t t0 = globaltimer_ns();
      for (;;) {
        __nanosleep(100);
        if (reached(ld_acquire_sys(mine), epoch)) break;
        if (globaltimer_ns() - t0 > kWaitLimitNs) {
          s_fail = 1;
          break;
        }
      }
    }
  }
  __syncthreads();
  const bool fail = s_fail != 0;
  if (fail && t == 0) report(dev_status, PA_DEVERR_TIMEOUT);

  // 3. one warp per row: weights from the ranks' lse (one lane per rank, kept
  //    in shared memory so the column loops below, where lanes may drop out,
  //    need no shuffle), then every lane folds its columns over the ranks in
  //    rank order, so every rank computes bit-identical rows.
  const int lane = t & 31, warp = t >> 5, nw = blockDim.x >> 5;
  float* w_s = s_w[warp];
  for (int64_t row = (int64_t)blockIdx.x * nw + warp; row < rows;
       row += (int64_t)gridDim.x * nw) {
    if (fail) {
      for (int d = lane; d < D; d += 32) out[row * D + d] = NAN;
      if (lse_out && lane == 0) lse_out[row] = NAN;
      continue;
    }
    float l = -INFINITY;
    if (lane < world)
      l = __ldcv(reinterpret_cast<const float*>(s_slot[lane] + lse_offset) + row);
    float mx = l;
#pragma unroll
    for (int o = 16; o; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    const float w = (l == -INFINITY) ? 0.f : __expf(l - mx);
    __syncwarp();  // every lane is done with the previous row's weights
    w_s[lane] = w;
    __syncwarp();
    // the denominator in rank order, the same on every lane and every rank
    float den = 0.f;
    for (int r = 0; r < world; ++r) den += w_s[r];
    const float inv = 1.f / den;  // den == 0 (every range empty) -> inf -> NaN rows
    if ((D & 3) == 0) {
      for (int d4 = lane; d4 < (D >> 2); d4 += 32) {
        float4 num = make_float4(0.f, 0.f, 0.f, 0.f);
        for (int r = 0; r < world; ++r) {
          const float wr = w_s[r];
          if (wr == 0.f) continue;
          const float4 v = __ldcv(reinterpret_cast<const float4*>(s_slot[r]) + row * (D >> 2) + d4);
          num.x += wr * v.x;
          num.y += wr * v.y;
          num.z += wr * v.z;
          num.w += wr * v.w;
        }
        float4 res;
        res.x = den > 0.f ? num.x * inv : NAN;
        res.y = den > 0.f ? num.y * inv : NAN;
        res.z = den > 0.f ? num.z * inv : NAN;
        res.w = den > 0.f ? num.w * inv : NAN;
        reinterpret_cast<float4*>(out)[row * (D >> 2) + d4] = res;
      }
    } else {
      for (int d = lane; d < D; d += 32) {
        float num = 0.f;
        for (int r = 0; r < world; ++r) {
          const float wr = w_s[r];
          if (wr == 0.f) continue;
          num += wr * __ldcv(reinterpret_cast<const float*>(s_slot[r]) + row * D + d);
        }
        out[row * D + d] = den > 0.f ? num * inv : NAN;
      }
    }
    if (lse_out && lane == 0) lse_out[row] = (den > 0.f) ? mx + __logf(den) : -INFINITY;
  }
}

}  // namespace peer
}  // namespace pa

// ---------------------------------------------------------------------------
// C ABI
// ---------------------------------------------------------------------------

extern "C" int pa_peer_exchange_layout(int64_t rows, int64_t head_dim, size_t* lse_offset,
                                       size_t* slot_bytes, size_t* flags_offset,
                                       size_t* total_bytes) {
  if (rows < 0 || head_dim <= 0 || !lse_offset || !slot_bytes || !flags_offset || !total_bytes)
    return PA_ERR_INVALID_ARGUMENT;
  const pa::peer::Layout l = pa::peer::layout(rows, head_dim);
  *lse_offset = l.lse_offset;
  *slot_bytes = l.slot_bytes;
  *flags_offset = l.flags_offset;
  *total_bytes = l.total_bytes;
  return PA_OK;
}

extern "C" int pa_ipc_alloc(size_t bytes, void** dev_ptr, void* handle) {
  if (bytes == 0 || !dev_ptr || !handle) return PA_ERR_INVALID_ARGUMENT;
  static_assert(sizeof(cudaIpcMemHandle_t) == PA_IPC_HANDLE_BYTES, "IPC handle size");
  void* p = nullptr;
  cudaError_t e = cudaMalloc(&p, bytes);
  if (e != cudaSuccess) return pa::cuda_status(e);
  // zeroed before any peer can see it: flags start below every epoch
  e = cudaMemset(p, 0, bytes);
  if (e == cudaSuccess) e = cudaDeviceSynchronize();
  cudaIpcMemHandle_t h;
  if (e == cudaSuccess) e = cudaIpcGetMemHandle(&h, p);
  if (e != cudaSuccess) {
    cudaFree(p);
    return pa::cuda_status(e);
  }
  memcpy(handle, &h, sizeof(h));
  *dev_ptr = p;
  return PA_OK;
}

extern "C" int pa_ipc_open(const void* handle, void** dev_ptr) {
  if (!handle || !dev_ptr) return PA_ERR_INVALID_ARGUMENT;
  cudaIpcMemHandle_t h;
  memcpy(&h, handle, sizeof(h));
  void* p = nullptr;
  const cudaError_t e = cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess);
  if (e != cudaSuccess) return pa::cuda_status(e);
  *dev_ptr = p;
  return PA_OK;
}

extern "C" int pa_ipc_close(void* dev_ptr) {
  if (!dev_ptr) return PA_ERR_INVALID_ARGUMENT;
  return pa::cuda_status(cudaIpcCloseMemHandle(dev_ptr));
}

extern "C" int pa_ipc_free(void* dev_ptr) {
  if (!dev_ptr) return PA_ERR_INVALID_ARGUMENT;
  return pa::cuda_status(cudaFree(dev_ptr));
}

extern "C" int pa_merge_peer_partials(float* out, float* lse_out, const uint64_t* peer_bases,
                                      int64_t world, int64_t rank, int64_t rows,
                                      int64_t head_dim, uint32_t epoch, int32_t* dev_status,
                                      void* stream) {
  if (world < 1 || world > pa::peer::kMaxWorld || rank < 0 || rank >= world || rows < 0 ||
      head_dim <= 0 || head_dim > (1 << 20) || !out || !peer_bases)
    return PA_ERR_INVALID_ARGUMENT;
  if (((head_dim & 3) == 0) && !pa::aligned16(out)) return PA_ERR_ALIGNMENT;
  if (rows == 0) return PA_OK;
  const pa::peer::Layout l = pa::peer::layout(rows, head_dim);
  const int threads = 256;
  const int64_t blocks = std::min<int64_t>((rows + 7) / 8, 1184);
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)blocks);
  cfg.blockDim = dim3(threads);
  cfg.stream = static_cast<cudaStream_t>(stream);
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return pa::cuda_status(cudaLaunchKernelEx(
      &cfg, pa::peer::merge_peers_kernel, out, lse_out,
      reinterpret_cast<const unsigned long long*>(peer_bases), (int)world, (int)rank, rows,
      (int)head_dim, (int64_t)l.lse_offset, (int64_t)l.slot_bytes, (int64_t)l.flags_offset,
      epoch, dev_status));
}
