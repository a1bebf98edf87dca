// decode_f32.cu -- split-KV decode kernels for a float KV pool (one translation
// unit per dtype so the instantiations compile in parallel).
#include "decode_impl.cuh"

namespace pa {
const void* decode_kernel_ptr_f32(int D, int QC) { return decode::pick_kernel<float>(D, QC); }
}  // namespace pa
