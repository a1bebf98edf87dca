// ref_arm_shim.cpp -- C entry points over the reference's own scalar CPU
// lane (gb10-attn arm_cpu/src/scalar.cpp, compiled from the reference
// sources by oracle/build_ref.py).  TEST INFRASTRUCTURE ONLY: used to pin
// oracle/pa_oracle.c's pao_scores / pao_softmax bit-for-bit.
#include <cstdint>

#include "gb10_arm/attention.hpp"

extern "C" void ref_attention_scores(const float* query, const float* keys, float* scores,
                                     int64_t tokens, int64_t head_dim) {
  gb10::arm::attention_scores(query, keys, scores, (std::size_t)tokens, (std::size_t)head_dim,
                              gb10::arm::dot_scalar);
}

extern "C" void ref_softmax_inplace(float* scores, int64_t n) {
  gb10::arm::softmax_inplace(scores, (std::size_t)n);
}
