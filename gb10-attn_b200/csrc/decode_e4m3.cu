// decode_e4m3.cu -- split-KV decode kernels for an FP8 E4M3 KV pool (one
// translation unit per dtype so the instantiations compile in parallel).
#include "decode_impl.cuh"

namespace pa {
const void* decode_kernel_ptr_e4m3(int D, int QC, bool step) {
  return step ? decode::pick_kernel<__nv_fp8_e4m3, true>(D, QC) : decode::pick_kernel<__nv_fp8_e4m3, false>(D, QC);
}
}  // namespace pa
