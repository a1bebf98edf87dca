// decode_f16.cu -- split-KV decode kernels for a __half KV pool (one translation
// unit per dtype so the instantiations compile in parallel).
#include "decode_impl.cuh"

namespace pa {
const void* decode_kernel_ptr_f16(int D, int QC, bool step) {
  return step ? decode::pick_kernel<__half, true>(D, QC) : decode::pick_kernel<__half, false>(D, QC);
}
}  // namespace pa
