// common.cuh -- sm_100a building blocks shared by the paged-attention kernels:
// mbarrier pipeline primitives, 1-D bulk (TMA) copies, bounded waits, dtype
// conversion of 16-byte chunks, and the host-side launch helpers.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_fp8.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/pa_b200.h"

namespace pa {

// ---------------------------------------------------------------------------
// dtype traits
// ---------------------------------------------------------------------------

template <typename T> struct DTypeId;
template <> struct DTypeId<float> { static constexpr int value = PA_DTYPE_F32; };
template <> struct DTypeId<__half> { static constexpr int value = PA_DTYPE_F16; };
template <> struct DTypeId<__nv_bfloat16> { static constexpr int value = PA_DTYPE_BF16; };
template <> struct DTypeId<double> { static constexpr int value = PA_DTYPE_F64; };
template <> struct DTypeId<__nv_fp8_e4m3> { static constexpr int value = PA_DTYPE_E4M3; };

inline int dtype_size(int dt) {
  switch (dt) {
    case PA_DTYPE_F32: return 4;
    case PA_DTYPE_F16: return 2;
    case PA_DTYPE_BF16: return 2;
    case PA_DTYPE_F64: return 8;
    case PA_DTYPE_E4M3: return 1;
    default: return 0;
  }
}

// Convert one 16-byte chunk (16 / sizeof(T) elements) to fp32.
template <typename T> struct Chunk;

template <> struct Chunk<__half> {
  static constexpr int N = 8;
  static __device__ __forceinline__ void cvt(const uint4& u, float* f) {
    const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      __half2 h = *reinterpret_cast<const __half2*>(&w[i]);
      float2 p = __half22float2(h);
      f[2 * i] = p.x;
      f[2 * i + 1] = p.y;
    }
  }
};

template <> struct Chunk<__nv_bfloat16> {
  static constexpr int N = 8;
  // bf16 -> fp32 is exact: the bf16 bits are the high half of the fp32.
  static __device__ __forceinline__ void cvt(const uint4& u, float* f) {
    const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      f[2 * i] = __uint_as_float(w[i] << 16);
      f[2 * i + 1] = __uint_as_float(w[i] & 0xffff0000u);
    }
  }
};

template <> struct Chunk<__nv_fp8_e4m3> {
  static constexpr int N = 16;
  // e4m3 -> fp16 is exact (every e4m3 value is an fp16 value), then fp16 -> fp32.
  static __device__ __forceinline__ void cvt(const uint4& u, float* f) {
    const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const __half2_raw lo =
          __nv_cvt_fp8x2_to_halfraw2((__nv_fp8x2_storage_t)(w[i] & 0xffffu), __NV_E4M3);
      const __half2_raw hi =
          __nv_cvt_fp8x2_to_halfraw2((__nv_fp8x2_storage_t)(w[i] >> 16), __NV_E4M3);
      const float2 a = __half22float2(*reinterpret_cast<const __half2*>(&lo));
      const float2 b = __half22float2(*reinterpret_cast<const __half2*>(&hi));
      f[4 * i] = a.x;
      f[4 * i + 1] = a.y;
      f[4 * i + 2] = b.x;
      f[4 * i + 3] = b.y;
    }
  }
};

template <> struct Chunk<float> {
  static constexpr int N = 4;
  static __device__ __forceinline__ void cvt(const uint4& u, float* f) {
    f[0] = __uint_as_float(u.x);
    f[1] = __uint_as_float(u.y);
    f[2] = __uint_as_float(u.z);
    f[3] = __uint_as_float(u.w);
  }
};

template <> struct Chunk<double> {
  static constexpr int N = 2;
  static __device__ __forceinline__ void cvt(const uint4& u, float* f) {
    const double d0 = __hiloint2double((int)u.y, (int)u.x);
    const double d1 = __hiloint2double((int)u.w, (int)u.z);
    f[0] = (float)d0;
    f[1] = (float)d1;
  }
};

// ---------------------------------------------------------------------------
// PTX wrappers
// ---------------------------------------------------------------------------

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count)
               : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.release.cta.shared::cta.b64 _, [%0], %1;" ::"r"(
                   smem_u32(bar)),
               "r"(bytes)
               : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.release.cta.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar))
               : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.acquire.cta.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// try_wait that lets the hardware suspend the thread (up to `hint_ns`) until
// the phase completes, instead of returning at once: waiting warps then do
// not take issue slots from the warps doing the work.
__device__ __forceinline__ bool mbar_try_wait_sleep(uint64_t* bar, uint32_t parity,
                                                    uint32_t hint_ns) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.acquire.cta.shared::cta.b64 p, [%1], %2, %3;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity), "r"(hint_ns)
      : "memory");
  return ok != 0;
}

__device__ __forceinline__ uint64_t globaltimer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// Every pipeline wait in this library is bounded: after kWaitLimitNs of
// wall time the wait gives up, returns false and the caller reports
// PA_DEVERR_TIMEOUT instead of hanging the GPU.
constexpr uint64_t kWaitLimitNs = 1000ull * 1000ull * 1000ull;  // 1 s

// `abort_flag` (global, per launch) makes every CTA give up as soon as one
// wait anywhere in the grid has timed out, so a failure costs ~1 s in total.
// The flag holds `abort_tag` once a wait has given up; a launch that does not
// zero the flag first passes a tag of its own, so a stale value left by an
// earlier launch reads as "no abort".
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity,
                                          int32_t* abort_flag = nullptr, int32_t abort_tag = 1) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = globaltimer_ns();
  for (uint32_t it = 1;; ++it) {
    if (mbar_try_wait_sleep(bar, parity, 100000u)) return true;
    if ((it & 7) == 0) {
      if (abort_flag && *reinterpret_cast<volatile int32_t*>(abort_flag) == abort_tag) return false;
      if (globaltimer_ns() - t0 > kWaitLimitNs) {
        if (abort_flag) atomicExch(abort_flag, abort_tag);
        return false;
      }
    }
  }
}

// The same bounded wait with acquire at cluster scope: for barriers that
// threads of another CTA of the cluster arrive on (their release.cluster
// arrivals then order their earlier writes before this thread's later reads).
__device__ __forceinline__ bool mbar_try_wait_cl(uint64_t* bar, uint32_t parity, uint32_t hint_ns) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2, %3;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity), "r"(hint_ns)
      : "memory");
  return ok != 0;
}

// try_wait with relaxed semantics at cluster scope: for barriers that only
// hand tensor-memory data between threads and the tensor core (an MMA's
// commit, or threads' tcgen05.st + tcgen05.wait::st); the tcgen05 fences on
// both sides order that data, and an acquire at cluster scope would add
// nothing but its cost.
__device__ __forceinline__ bool mbar_try_wait_rx(uint64_t* bar, uint32_t parity, uint32_t hint_ns) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.relaxed.cluster.shared::cta.b64 p, [%1], %2, %3;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity), "r"(hint_ns)
      : "memory");
  return ok != 0;
}

// The bounded wait on such a barrier.
__device__ __forceinline__ bool mbar_wait_rx(uint64_t* bar, uint32_t parity, int32_t* abort_flag,
                                             int32_t abort_tag = 1) {
  if (mbar_try_wait_rx(bar, parity, 0u)) return true;
  const uint64_t t0 = globaltimer_ns();
  for (uint32_t it = 1;; ++it) {
    if (mbar_try_wait_rx(bar, parity, 100000u)) return true;
    if ((it & 7) == 0) {
      if (abort_flag && *reinterpret_cast<volatile int32_t*>(abort_flag) == abort_tag) return false;
      if (globaltimer_ns() - t0 > kWaitLimitNs) {
        if (abort_flag) atomicExch(abort_flag, abort_tag);
        return false;
      }
    }
  }
}

__device__ __forceinline__ bool mbar_wait_cl(uint64_t* bar, uint32_t parity, int32_t* abort_flag,
                                             int32_t abort_tag = 1) {
  if (mbar_try_wait_cl(bar, parity, 0u)) return true;
  const uint64_t t0 = globaltimer_ns();
  for (uint32_t it = 1;; ++it) {
    if (mbar_try_wait_cl(bar, parity, 100000u)) return true;
    if ((it & 7) == 0) {
      if (abort_flag && *reinterpret_cast<volatile int32_t*>(abort_flag) == abort_tag) return false;
      if (globaltimer_ns() - t0 > kWaitLimitNs) {
        if (abort_flag) atomicExch(abort_flag, abort_tag);
        return false;
      }
    }
  }
}

// 1-D bulk async copy global -> shared (TMA engine), completing on `bar`.
// dst, src and bytes must be multiples of 16; dst is this CTA's own shared memory.
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes,
                                         uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

__device__ __forceinline__ void prefetch_l2(const void* src, uint32_t bytes) {
  asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(src), "r"(bytes) : "memory");
}

__device__ __forceinline__ uint4 lds128(const void* p) {
  uint4 v;
  asm volatile("ld.shared.v4.u32 {%0, %1, %2, %3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "r"(smem_u32(p)));
  return v;
}

__device__ __forceinline__ float fast_exp2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// Packed fp32 pair arithmetic (sm_100 add / fma .f32x2, round to nearest, no
// flush): one issue slot does the work of two scalar instructions.
__device__ __forceinline__ float2 add2(float2 a, float2 b) {
  float2 r;
  asm("{.reg .b64 pa, pb, pd;\n\tmov.b64 pa, {%2, %3};\n\tmov.b64 pb, {%4, %5};\n\t"
      "add.rn.f32x2 pd, pa, pb;\n\tmov.b64 {%0, %1}, pd;}"
      : "=f"(r.x), "=f"(r.y) : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y));
  return r;
}
__device__ __forceinline__ float2 fma2(float2 a, float2 b, float2 c) {
  float2 r;
  asm("{.reg .b64 pa, pb, pc, pd;\n\tmov.b64 pa, {%2, %3};\n\tmov.b64 pb, {%4, %5};\n\t"
      "mov.b64 pc, {%6, %7};\n\tfma.rn.f32x2 pd, pa, pb, pc;\n\tmov.b64 {%0, %1}, pd;}"
      : "=f"(r.x), "=f"(r.y)
      : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y), "f"(c.x), "f"(c.y));
  return r;
}

__device__ __forceinline__ void report(int32_t* dev_status, int bits) {
  if (dev_status) atomicOr(dev_status, bits);
}

// Programmatic dependent launch controls (no-ops when launched without PDL).
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// ---------------------------------------------------------------------------
// host helpers
// ---------------------------------------------------------------------------

void set_last_cuda_error(cudaError_t e);
int cuda_status(cudaError_t e);  // PA_OK or PA_ERR_CUDA (records e)
int device_sm_count(int* sms);   // current device; PA_OK / PA_ERR_NO_DEVICE

inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

constexpr float kLog2e = 1.4426950408889634f;
constexpr float kLn2 = 0.6931471805599453f;

}  // namespace pa
