// decode_host.h -- host interface of the split-KV decode launcher, shared by
// the decode entry points (decode.cu) and the CUDA-core prefill path
// (prefill.cu), which runs the same kernel with one pseudo-sequence per query
// row.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

namespace pa {
namespace decode {

struct DecodeArgs {
  float* out;
  float* lse;
  const float* q;
  const void* k_cache;
  const void* v_cache;
  int dtype;
  const int32_t* block_tables;
  const int32_t* context_lens;
  int64_t B, H, HKV, D, BS, NB, MB;
  double scale;
  int64_t num_splits;
  int32_t* dev_status;
  int64_t qlen = 1;        // query rows per sequence (causal prefill: Sq)
  float empty_fill = 0.f;  // value of rows that see no key
  const float* k_scale = nullptr;  // FP8 pools: [HKV] dequantisation scales (null = 1)
  const float* v_scale = nullptr;
  // element type of q and out (PA_DTYPE_F32 / F16 / BF16; `q` and `out` point
  // at that type), and the decode step's new K / V rows ([B, HKV, D] of
  // io_dtype, null: none), written at position context_lens[b] - 1 first
  int io_dtype = 0;
  const void* k_new = nullptr;
  const void* v_new = nullptr;
};

int launch(const DecodeArgs& a, void* ws, size_t ws_bytes, cudaStream_t stream);
int workspace_bytes(const DecodeArgs& a, size_t* bytes);

}  // namespace decode
}  // namespace pa
