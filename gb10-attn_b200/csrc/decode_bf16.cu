// decode_bf16.cu -- split-KV decode kernels for a __nv_bfloat16 KV pool (one translation
// unit per dtype so the instantiations compile in parallel).
#include "decode_impl.cuh"

namespace pa {
const void* decode_kernel_ptr_bf16(int D, int QC, bool step) {
  return step ? decode::pick_kernel<__nv_bfloat16, true>(D, QC) : decode::pick_kernel<__nv_bfloat16, false>(D, QC);
}
}  // namespace pa
