// decode_f64.cu -- split-KV decode kernels for a double KV pool (one translation
// unit per dtype so the instantiations compile in parallel).
#include "decode_impl.cuh"

namespace pa {
const void* decode_kernel_ptr_f64(int D, int QC, bool step) {
  return step ? decode::pick_kernel<double, true>(D, QC) : decode::pick_kernel<double, false>(D, QC);
}
}  // namespace pa
