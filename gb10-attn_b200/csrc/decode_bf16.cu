// decode_bf16.cu -- split-KV decode kernels for a __nv_bfloat16 KV pool (one translation
// unit per dtype so the instantiations compile in parallel).
#include "decode_impl.cuh"

namespace pa {
const void* decode_kernel_ptr_bf16(int D, int QC) { return decode::pick_kernel<__nv_bfloat16>(D, QC); }
}  // namespace pa
