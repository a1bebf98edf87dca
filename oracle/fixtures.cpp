// fixtures.cpp -- seeded inputs of the reference's own self-tests, regenerated
// with the same C++ <random> engines and distributions so the oracle and the
// B200 kernels can be run on exactly the reference's fixtures.
// TEST INFRASTRUCTURE ONLY (compiled into oracle/_build/libpa_oracle.so).
#include <cstdint>
#include <random>

extern "C" {

// rocm/hip/paged_attn_v1_hip.cpp:151-164: B=2, H=4, HKV=2, D=32, BS=16, MB=4,
// NB=8, ctx=48; std::mt19937(7), uniform_real_distribution<float>(-0.25,
// 0.25) drawn for q, then k, then v; bt[b][m] = (b*MB + m) % NB.
// q: B*H*D, k/v: NB*BS*HKV*D, bt: B*MB, ctx: B.
void pao_fixture_hip_selftest(float* q, float* k, float* v, int32_t* bt, int32_t* ctx) {
  const int B = 2, H = 4, HKV = 2, D = 32, BS = 16, MB = 4, NB = 8, NCTX = 48;
  std::mt19937 rng(7);
  std::uniform_real_distribution<float> dist(-0.25f, 0.25f);
  for (int i = 0; i < B * H * D; ++i) q[i] = dist(rng);
  for (int i = 0; i < NB * BS * HKV * D; ++i) k[i] = dist(rng);
  for (int i = 0; i < NB * BS * HKV * D; ++i) v[i] = dist(rng);
  for (int b = 0; b < B; ++b)
    for (int m = 0; m < MB; ++m) bt[b * MB + m] = (b * MB + m) % NB;
  for (int b = 0; b < B; ++b) ctx[b] = NCTX;
}

// arm_cpu/src/bench.cpp:56-63: std::mt19937(2026), uniform(-0.25, 0.25),
// query [dim] then keys [tokens * dim].
void pao_fixture_arm_bench(float* query, float* keys, int64_t tokens, int64_t dim) {
  std::mt19937 rng(2026);
  std::uniform_real_distribution<float> dist(-0.25f, 0.25f);
  for (int64_t i = 0; i < dim; ++i) query[i] = dist(rng);
  for (int64_t i = 0; i < tokens * dim; ++i) keys[i] = dist(rng);
}

}  // extern "C"
