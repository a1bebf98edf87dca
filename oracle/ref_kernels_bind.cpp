// ref_kernels_bind.cpp -- Python binding of the reference's own CUDA kernels
// (gb10-attn kernels/*.cu, compiled unchanged for sm_100a by
// oracle/build_ref.py), equivalent to the module hetero-serve builds with
// load_inline(functions=[...]) (kernels/paged_attn_v3.h:5-7).  TEST
// INFRASTRUCTURE ONLY: tests and tests/golden/make_golden.py use it to pin the
// oracle and the B200 kernels against the reference's outputs on a GPU.
#include <torch/extension.h>

#include "paged_attn_prefill.h"
#include "paged_attn_v1.h"
#include "paged_attn_v2.h"
#include "paged_attn_v3.h"
#include "paged_attn_wmma.h"

PYBIND11_MODULE(gb10_ref_kernels, m) {
  m.def("paged_attention", &paged_attention);
  m.def("paged_attention_v2", &paged_attention_v2);
  m.def("paged_attention_v3", &paged_attention_v3);
  m.def("choose_num_splits", &choose_num_splits);
  m.def("paged_attention_prefill", &paged_attention_prefill);
  m.def("paged_attention_prefill_wmma", &paged_attention_prefill_wmma);
}
