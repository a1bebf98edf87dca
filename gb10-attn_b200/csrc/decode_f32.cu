// decode_f32.cu -- split-KV decode kernels for a float KV pool (one translation
// unit per dtype so the instantiations compile in parallel).
#include "decode_impl.cuh"

namespace pa {
const void* decode_kernel_ptr_f32(int D, int QC, bool step) {
  return step ? decode::pick_kernel<float, true>(D, QC) : decode::pick_kernel<float, false>(D, QC);
}
}  // namespace pa
