// torch_shim.cpp -- the reference's C++ operator API on top of libpa_b200.so.
//
// gb10-attn's kernels are consumed as torch extension functions built by
// hetero-serve with torch.utils.cpp_extension.load_inline(functions=[...])
// (kernels/paged_attn_v1.h:5-7 and siblings).  This file exports the same
// functions with the same signatures, argument meaning and TORCH_CHECK
// messages, so a caller swaps the module and nothing else:
//
//   paged_attention(q, k_cache, v_cache, block_tables, context_lens, scale)
//       kernels/paged_attn_v1.h:13-15
//   paged_attention_v2(...)                       kernels/paged_attn_v2.h:13-15
//   paged_attention_v3(..., scale, num_splits)    kernels/paged_attn_v3.h:13-16
//   choose_num_splits(num_seqs, num_heads, max_context)  paged_attn_v3.h:17
//   paged_attention_prefill(...)                  kernels/paged_attn_prefill.h:13-15
//   paged_attention_prefill_wmma(...)             kernels/paged_attn_wmma.h:13-15
//
// plus the pool writer and helpers the reference keeps in Python
// (write_kv, validate_block_tables, paged_attention_v3_lse, merge_states), and
// the FP8-pool additions (paged_attention_v3_fp8, write_kv_scaled) and the
// many-sequence writer (write_kv_batch) and one layer of a decode step
// (decode_layer_step: q / out in bf16 or fp16, the K/V append fused in).
//
// Differences, all supersets: bf16 pools are accepted (the reference's
// AT_DISPATCH_FLOATING_TYPES_AND_HALF has fp32/fp64/fp16 only); launches go to
// the current torch stream (the reference uses the legacy default stream,
// which is torch's default current stream); a device guard selects q's device.
// Scratch comes from torch's caching allocator, as the reference's
// torch::empty partial buffers did (paged_attn_v3.cu:220-224).
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#include "pa_b200.h"

namespace {

int pool_dtype(const torch::Tensor& t, const char* op) {
  switch (t.scalar_type()) {
    case torch::kFloat: return PA_DTYPE_F32;
    case torch::kHalf: return PA_DTYPE_F16;
    case torch::kBFloat16: return PA_DTYPE_BF16;
    case torch::kDouble: return PA_DTYPE_F64;
    case torch::kFloat8_e4m3fn: return PA_DTYPE_E4M3;
    default:
      TORCH_CHECK(false, "\"", op, "\" not implemented for '", toString(t.scalar_type()), "'");
  }
  return -1;
}

void check_status(int st, const char* op) {
  if (st == PA_OK) return;
  if (st == PA_ERR_CUDA) {
    TORCH_CHECK(false, op, ": CUDA error: ",
                cudaGetErrorString(static_cast<cudaError_t>(pa_last_cuda_error())));
  }
  TORCH_CHECK(false, op, ": ", pa_strerror(st));
}

void* stream_ptr() { return static_cast<void*>(at::cuda::getCurrentCUDAStream().stream()); }

torch::Tensor workspace(size_t bytes, const torch::Tensor& like) {
  return torch::empty({static_cast<int64_t>(bytes > 0 ? bytes : 1)},
                      like.options().dtype(torch::kUInt8));
}

struct DecodeInputs {
  torch::Tensor q, k, v, bt, ctx;
  int64_t B, H, D, BS, HKV, MB, NB;
  int dtype;
};

// The reference's argument handling (paged_attn_v3.cu:201-216): contiguous
// q/k/v, block tables and context lengths converted to int32.
DecodeInputs prepare(torch::Tensor q, torch::Tensor k_cache, torch::Tensor v_cache,
                     torch::Tensor block_tables, torch::Tensor context_lens, const char* op,
                     int q_dims) {
  DecodeInputs in;
  TORCH_CHECK(q.is_cuda(), "q must be on CUDA");
  TORCH_CHECK(k_cache.is_cuda() && v_cache.is_cuda(), "kv cache must be on CUDA");
  TORCH_CHECK(q.dim() == q_dims, q_dims == 3 ? "q must be [B, H, D]" : "q must be [B, S, H, D]");
  TORCH_CHECK(k_cache.dim() == 4, "k_cache must be [NB, BS, H, D]");
  TORCH_CHECK(v_cache.sizes() == k_cache.sizes(), "v_cache must match k_cache");
  TORCH_CHECK(v_cache.scalar_type() == k_cache.scalar_type(), "v_cache dtype must match k_cache");
  TORCH_CHECK(q.scalar_type() == torch::kFloat, "expected scalar type Float but found ",
              toString(q.scalar_type()));
  in.q = q.contiguous();
  in.k = k_cache.contiguous();
  in.v = v_cache.contiguous();
  in.bt = block_tables.to(q.device(), torch::kInt32).contiguous();
  in.ctx = context_lens.to(q.device(), torch::kInt32).contiguous();
  TORCH_CHECK(in.bt.dim() == 2, "block_tables must be [B, MB]");
  in.dtype = pool_dtype(in.k, op);
  in.B = q.size(0);
  in.H = q.size(q_dims - 2);
  in.D = q.size(q_dims - 1);
  in.BS = in.k.size(1);
  in.HKV = in.k.size(2);
  in.NB = in.k.size(0);
  in.MB = in.bt.size(1);
  TORCH_CHECK(in.k.size(3) == in.D, "k_cache head_dim must match q");
  TORCH_CHECK(in.ctx.numel() >= in.B, "context_lens must have B entries");
  TORCH_CHECK(in.bt.size(0) >= in.B, "block_tables must have B rows");
  return in;
}

void decode_checks(const DecodeInputs& in) {
  TORCH_CHECK(in.H % in.HKV == 0, "n_head must be divisible by n_kv_head");
  TORCH_CHECK(in.D % 32 == 0, "head_dim must be a multiple of the warp size");
  TORCH_CHECK(in.D == 32 || in.D == 64 || in.D == 128 || in.D == 256, "unsupported head_dim ",
              in.D);
}

std::tuple<torch::Tensor, torch::Tensor> decode_impl(torch::Tensor q, torch::Tensor k_cache,
                                                     torch::Tensor v_cache,
                                                     torch::Tensor block_tables,
                                                     torch::Tensor context_lens, double scale,
                                                     int64_t num_splits, int which,
                                                     bool want_lse) {
  static const char* names[] = {"paged_attention", "paged_attention_v2", "paged_attention_v3"};
  const char* op = names[which];
  DecodeInputs in = prepare(q, k_cache, v_cache, block_tables, context_lens, op, 3);
  decode_checks(in);
  const c10::cuda::CUDAGuard guard(in.q.device());
  auto fopts = in.q.options().dtype(torch::kFloat32);
  torch::Tensor out = torch::empty({in.B, in.H, in.D}, fopts);
  torch::Tensor lse = want_lse ? torch::empty({in.B, in.H}, fopts) : torch::Tensor();
  if (in.B == 0) return {out, lse};
  const int64_t splits = which == 2 ? num_splits : 0;
  size_t ws_bytes = 0;
  check_status(pa_decode_workspace_size(in.B, in.H, in.HKV, in.D, in.dtype, in.BS, in.MB, splits,
                                        &ws_bytes),
               op);
  torch::Tensor ws = workspace(ws_bytes, in.q);
  int st;
  if (which == 2 || want_lse) {
    st = pa_paged_attention_v3(out.data_ptr<float>(), want_lse ? lse.data_ptr<float>() : nullptr,
                               in.q.data_ptr<float>(), in.k.data_ptr(), in.v.data_ptr(), in.dtype,
                               in.bt.data_ptr<int32_t>(), in.ctx.data_ptr<int32_t>(), in.B, in.H,
                               in.HKV, in.D, in.BS, in.NB, in.MB, scale, splits, ws.data_ptr(),
                               ws_bytes, nullptr, stream_ptr());
  } else if (which == 1) {
    st = pa_paged_attention_v2(out.data_ptr<float>(), in.q.data_ptr<float>(), in.k.data_ptr(),
                               in.v.data_ptr(), in.dtype, in.bt.data_ptr<int32_t>(),
                               in.ctx.data_ptr<int32_t>(), in.B, in.H, in.HKV, in.D, in.BS,
                               in.NB, in.MB, scale, ws.data_ptr(), ws_bytes, nullptr,
                               stream_ptr());
  } else {
    st = pa_paged_attention(out.data_ptr<float>(), in.q.data_ptr<float>(), in.k.data_ptr(),
                            in.v.data_ptr(), in.dtype, in.bt.data_ptr<int32_t>(),
                            in.ctx.data_ptr<int32_t>(), in.B, in.H, in.HKV, in.D, in.BS, in.NB,
                            in.MB, scale, ws.data_ptr(), ws_bytes, nullptr, stream_ptr());
  }
  check_status(st, op);
  return {out, lse};
}

}  // namespace

torch::Tensor paged_attention(torch::Tensor q, torch::Tensor k_cache, torch::Tensor v_cache,
                              torch::Tensor block_tables, torch::Tensor context_lens,
                              double scale) {
  return std::get<0>(
      decode_impl(q, k_cache, v_cache, block_tables, context_lens, scale, 0, 0, false));
}

torch::Tensor paged_attention_v2(torch::Tensor q, torch::Tensor k_cache, torch::Tensor v_cache,
                                 torch::Tensor block_tables, torch::Tensor context_lens,
                                 double scale) {
  return std::get<0>(
      decode_impl(q, k_cache, v_cache, block_tables, context_lens, scale, 0, 1, false));
}

torch::Tensor paged_attention_v3(torch::Tensor q, torch::Tensor k_cache, torch::Tensor v_cache,
                                 torch::Tensor block_tables, torch::Tensor context_lens,
                                 double scale, int64_t num_splits) {
  return std::get<0>(decode_impl(q, k_cache, v_cache, block_tables, context_lens, scale,
                                 num_splits, 2, false));
}

// (out, lse) of a decode; lse[b, h] = ln sum_j exp(scale * q.k_j).  Used by the
// sequence-sharded multi-GPU decode before the cross-device merge.
std::tuple<torch::Tensor, torch::Tensor> paged_attention_v3_lse(
    torch::Tensor q, torch::Tensor k_cache, torch::Tensor v_cache, torch::Tensor block_tables,
    torch::Tensor context_lens, double scale, int64_t num_splits) {
  return decode_impl(q, k_cache, v_cache, block_tables, context_lens, scale, num_splits, 2,
                     true);
}

// Decode of an FP8 (float8_e4m3fn) pool with per-KV-head fp32 scales
// (K = k_cache * k_scale[h], V = v_cache * v_scale[h]); returns (out, lse).
// An addition: the reference has no FP8 pool.
std::tuple<torch::Tensor, torch::Tensor> paged_attention_v3_fp8(
    torch::Tensor q, torch::Tensor k_cache, torch::Tensor v_cache, torch::Tensor block_tables,
    torch::Tensor context_lens, double scale, torch::Tensor k_scale, torch::Tensor v_scale,
    int64_t num_splits) {
  const char* op = "paged_attention_v3_fp8";
  TORCH_CHECK(k_cache.scalar_type() == torch::kFloat8_e4m3fn,
              op, ": k_cache must be float8_e4m3fn");
  DecodeInputs in = prepare(q, k_cache, v_cache, block_tables, context_lens, op, 3);
  decode_checks(in);
  const c10::cuda::CUDAGuard guard(in.q.device());
  torch::Tensor ks = k_scale.to(in.q.device(), torch::kFloat).contiguous();
  torch::Tensor vs = v_scale.to(in.q.device(), torch::kFloat).contiguous();
  TORCH_CHECK(ks.numel() == in.HKV && vs.numel() == in.HKV, op,
              ": k_scale and v_scale need one entry per KV head");
  auto fopts = in.q.options().dtype(torch::kFloat32);
  torch::Tensor out = torch::empty({in.B, in.H, in.D}, fopts);
  torch::Tensor lse = torch::empty({in.B, in.H}, fopts);
  if (in.B == 0) return {out, lse};
  size_t ws_bytes = 0;
  check_status(pa_decode_workspace_size(in.B, in.H, in.HKV, in.D, in.dtype, in.BS, in.MB,
                                        num_splits, &ws_bytes),
               op);
  torch::Tensor ws = workspace(ws_bytes, in.q);
  check_status(pa_paged_attention_v3_fp8(
                   out.data_ptr<float>(), lse.data_ptr<float>(), in.q.data_ptr<float>(),
                   in.k.data_ptr(), in.v.data_ptr(), ks.data_ptr<float>(), vs.data_ptr<float>(),
                   in.dtype, in.bt.data_ptr<int32_t>(), in.ctx.data_ptr<int32_t>(), in.B, in.H,
                   in.HKV, in.D, in.BS, in.NB, in.MB, scale, num_splits, ws.data_ptr(),
                   ws_bytes, nullptr, stream_ptr()),
               op);
  return {out, lse};
}

int64_t choose_num_splits(int64_t num_seqs, int64_t num_heads, int64_t max_context) {
  const int64_t s = pa_choose_num_splits(num_seqs, num_heads, max_context);
  TORCH_CHECK(s > 0, "choose_num_splits: ", pa_strerror(PA_ERR_NO_DEVICE));
  return s;
}

static torch::Tensor prefill_impl(torch::Tensor q, torch::Tensor k_cache, torch::Tensor v_cache,
                                  torch::Tensor block_tables, torch::Tensor context_lens,
                                  double scale, int which) {
  static const char* names[] = {"paged_attention_prefill", "paged_attention_prefill_wmma",
                                "paged_attention_prefill_simt"};
  const char* op = names[which];
  TORCH_CHECK(q.is_cuda(), "q must be on CUDA");
  TORCH_CHECK(q.dim() == 4, "q must be [B, S, H, D]");
  if (which == 1) {
    // paged_attn_wmma.cu:220-225 (bf16 accepted as well)
    TORCH_CHECK(k_cache.scalar_type() == torch::kHalf || k_cache.scalar_type() == torch::kBFloat16,
                "the WMMA path needs an fp16 KV cache");
    TORCH_CHECK(k_cache.dim() == 4 && k_cache.size(1) == 16,
                "the WMMA path needs block_size == 16 (one page per fragment)");
  }
  DecodeInputs in = prepare(q, k_cache, v_cache, block_tables, context_lens, op, 4);
  const int64_t S = in.q.size(1);
  TORCH_CHECK(in.H % in.HKV == 0, "n_head must be divisible by n_kv_head");
  if (which == 1) {
    TORCH_CHECK(in.D % 16 == 0, "head_dim must be a multiple of 16");
    TORCH_CHECK(in.D == 32 || in.D == 64 || in.D == 128,
                "unsupported head_dim for the WMMA path: ", in.D);
  } else {
    TORCH_CHECK(in.D % 32 == 0, "head_dim must be a multiple of the warp size");
    TORCH_CHECK(in.D == 32 || in.D == 64 || in.D == 128 || in.D == 256, "unsupported head_dim ",
                in.D);
  }
  const c10::cuda::CUDAGuard guard(in.q.device());
  torch::Tensor out = torch::empty({in.B, S, in.H, in.D}, in.q.options().dtype(torch::kFloat32));
  if (in.B == 0 || S == 0) return out;
  size_t ws_bytes = 0;
  check_status(pa_prefill_workspace_size(in.B, S, in.H, in.HKV, in.D, in.dtype, in.BS, in.MB,
                                         &ws_bytes),
               op);
  torch::Tensor ws = workspace(ws_bytes, in.q);
  auto fn = which == 0 ? pa_paged_attention_prefill
                       : (which == 1 ? pa_paged_attention_prefill_wmma
                                     : pa_paged_attention_prefill_simt);
  const int st = fn(out.data_ptr<float>(), in.q.data_ptr<float>(), in.k.data_ptr(),
                    in.v.data_ptr(), in.dtype, in.bt.data_ptr<int32_t>(),
                    in.ctx.data_ptr<int32_t>(), in.B, S, in.H, in.HKV, in.D, in.BS, in.NB,
                    in.MB, scale, ws.data_ptr(), ws_bytes, nullptr, stream_ptr());
  check_status(st, op);
  return out;
}

torch::Tensor paged_attention_prefill(torch::Tensor q, torch::Tensor k_cache,
                                      torch::Tensor v_cache, torch::Tensor block_tables,
                                      torch::Tensor context_lens, double scale) {
  return prefill_impl(q, k_cache, v_cache, block_tables, context_lens, scale, 0);
}

torch::Tensor paged_attention_prefill_wmma(torch::Tensor q, torch::Tensor k_cache,
                                           torch::Tensor v_cache, torch::Tensor block_tables,
                                           torch::Tensor context_lens, double scale) {
  return prefill_impl(q, k_cache, v_cache, block_tables, context_lens, scale, 1);
}

torch::Tensor paged_attention_prefill_simt(torch::Tensor q, torch::Tensor k_cache,
                                           torch::Tensor v_cache, torch::Tensor block_tables,
                                           torch::Tensor context_lens, double scale) {
  return prefill_impl(q, k_cache, v_cache, block_tables, context_lens, scale, 2);
}

// Pool writer: k_layers / v_layers are the per-layer [NB, BS, HKV, D] K and V
// tensors (views pool[l, 0] / pool[l, 1] of a monolithic pool, or one tensor
// per layer); k, v are [n_layer, HKV, n_tok, D] device tensors (head_dim
// contiguous).  Token t goes to position start + t of the sequence whose
// pages are block_ids.
// k_scales / v_scales (FP8 pools): [n_layer, HKV] fp32, stored value = x / scale.
void write_kv_impl(std::vector<torch::Tensor> k_layers, std::vector<torch::Tensor> v_layers,
                   torch::Tensor block_ids, int64_t start, torch::Tensor k, torch::Tensor v,
                   c10::optional<torch::Tensor> k_scales, c10::optional<torch::Tensor> v_scales,
                   const char* op) {
  TORCH_CHECK(!k_layers.empty() && k_layers.size() == v_layers.size(),
              "write_kv: need one K and one V tensor per layer");
  TORCH_CHECK(k.dim() == 4 && v.sizes() == k.sizes(), "write_kv: k, v must be [L, H, T, D]");
  TORCH_CHECK(k.size(0) == (int64_t)k_layers.size(), "write_kv: layer count mismatch");
  const torch::Tensor& k0 = k_layers[0];
  TORCH_CHECK(k0.is_cuda() && k0.dim() == 4, "write_kv: pool tensors must be CUDA [NB, BS, H, D]");
  TORCH_CHECK(k.scalar_type() == v.scalar_type(), "write_kv: k and v dtypes differ");
  const c10::cuda::CUDAGuard guard(k0.device());
  std::vector<void*> kp, vp;
  const int pdt = pool_dtype(k0, op);
  for (size_t l = 0; l < k_layers.size(); ++l) {
    for (const torch::Tensor* t : {&k_layers[l], &v_layers[l]}) {
      TORCH_CHECK(t->is_contiguous() && t->sizes() == k0.sizes() &&
                      t->scalar_type() == k0.scalar_type() && t->device() == k0.device(),
                  "write_kv: pool tensors must be contiguous and alike");
    }
    kp.push_back(k_layers[l].data_ptr());
    vp.push_back(v_layers[l].data_ptr());
  }
  torch::Tensor kd = k.to(k0.device());
  torch::Tensor vd = v.to(k0.device());
  if (kd.stride(3) != 1) kd = kd.contiguous();
  if (vd.stride(3) != 1 || vd.strides() != kd.strides()) {
    kd = kd.contiguous();
    vd = vd.contiguous();
  }
  int sdt;
  switch (kd.scalar_type()) {
    case torch::kFloat: sdt = PA_DTYPE_F32; break;
    case torch::kHalf: sdt = PA_DTYPE_F16; break;
    case torch::kBFloat16: sdt = PA_DTYPE_BF16; break;
    default:
      kd = kd.to(torch::kFloat);
      vd = vd.to(torch::kFloat);
      sdt = PA_DTYPE_F32;
  }
  torch::Tensor ids = block_ids.to(k0.device(), torch::kInt32).contiguous();
  TORCH_CHECK(kd.size(1) == k0.size(2) && kd.size(3) == k0.size(3),
              "write_kv: k heads / head_dim must match the pool");
  torch::Tensor ks, vs;
  const int64_t L = (int64_t)k_layers.size();
  for (auto [src, dst] : {std::make_pair(&k_scales, &ks), std::make_pair(&v_scales, &vs)}) {
    if (!src->has_value()) continue;
    *dst = src->value().to(k0.device(), torch::kFloat).contiguous();
    TORCH_CHECK(dst->numel() == L * k0.size(2), op, ": scales must be [n_layer, HKV]");
  }
  const int st = pa_write_kv_scaled(
      kp.data(), vp.data(), pdt, kd.data_ptr(), vd.data_ptr(), sdt, kd.stride(0), kd.stride(1),
      kd.stride(2), ids.data_ptr<int32_t>(), ids.numel(), start, kd.size(2), L, k0.size(2),
      k0.size(3), k0.size(1), k0.size(0), ks.defined() ? ks.data_ptr<float>() : nullptr,
      vs.defined() ? vs.data_ptr<float>() : nullptr, nullptr, stream_ptr());
  check_status(st, op);
}

void write_kv(std::vector<torch::Tensor> k_layers, std::vector<torch::Tensor> v_layers,
              torch::Tensor block_ids, int64_t start, torch::Tensor k, torch::Tensor v) {
  write_kv_impl(std::move(k_layers), std::move(v_layers), block_ids, start, k, v,
                c10::nullopt, c10::nullopt, "write_kv");
}

void write_kv_scaled(std::vector<torch::Tensor> k_layers, std::vector<torch::Tensor> v_layers,
                     torch::Tensor block_ids, int64_t start, torch::Tensor k, torch::Tensor v,
                     torch::Tensor k_scales, torch::Tensor v_scales) {
  write_kv_impl(std::move(k_layers), std::move(v_layers), block_ids, start, k, v, k_scales,
                v_scales, "write_kv_scaled");
}

// One layer of a decode step (pa_decode_layer_step): q [B, H, D] of fp32 /
// fp16 / bf16 gives out of the same dtype; k_new / v_new ([B, HKV, D], or
// empty tensors for none) are written at position context_lens[b] - 1 of the
// pool in the same launch.  The pool tensors are written in place.
torch::Tensor decode_layer_step(torch::Tensor q, torch::Tensor k_cache, torch::Tensor v_cache,
                                torch::Tensor block_tables, torch::Tensor context_lens,
                                double scale, torch::Tensor k_new, torch::Tensor v_new) {
  const char* op = "decode_layer_step";
  TORCH_CHECK(q.is_cuda() && q.dim() == 3, op, ": q must be a CUDA [B, H, D] tensor");
  int io;
  switch (q.scalar_type()) {
    case torch::kFloat: io = PA_DTYPE_F32; break;
    case torch::kHalf: io = PA_DTYPE_F16; break;
    case torch::kBFloat16: io = PA_DTYPE_BF16; break;
    default: TORCH_CHECK(false, op, ": q must be float32, float16 or bfloat16");
  }
  TORCH_CHECK(k_cache.is_cuda() && k_cache.dim() == 4 && v_cache.sizes() == k_cache.sizes() &&
                  v_cache.scalar_type() == k_cache.scalar_type(),
              op, ": k_cache, v_cache must be alike CUDA [NB, BS, HKV, D] tensors");
  TORCH_CHECK(k_cache.is_contiguous() && v_cache.is_contiguous(),
              op, ": the pool is written in place, so it must be contiguous");
  const c10::cuda::CUDAGuard guard(q.device());
  torch::Tensor qc = q.contiguous();
  torch::Tensor bt = block_tables.to(q.device(), torch::kInt32).contiguous();
  torch::Tensor ctx = context_lens.to(q.device(), torch::kInt32).contiguous();
  const int64_t B = qc.size(0), H = qc.size(1), D = qc.size(2);
  const int64_t NB = k_cache.size(0), BS = k_cache.size(1), HKV = k_cache.size(2);
  TORCH_CHECK(k_cache.size(3) == D, op, ": k_cache head_dim must match q");
  TORCH_CHECK(bt.dim() == 2 && bt.size(0) >= B && ctx.numel() >= B,
              op, ": block_tables [B, MB] and context_lens [B] needed");
  const int kdt = pool_dtype(k_cache, op);
  torch::Tensor kn, vn;
  const bool append = k_new.defined() && k_new.numel() > 0;
  if (append) {
    TORCH_CHECK(v_new.sizes() == k_new.sizes() && k_new.dim() == 3 && k_new.size(0) == B &&
                    k_new.size(1) == HKV && k_new.size(2) == D,
                op, ": k_new, v_new must be [B, HKV, D]");
    kn = k_new.to(q.device(), q.scalar_type()).contiguous();
    vn = v_new.to(q.device(), q.scalar_type()).contiguous();
  }
  torch::Tensor out = torch::empty({B, H, D}, qc.options());
  if (B == 0) return out;
  size_t ws_bytes = 0;
  check_status(pa_decode_workspace_size(B, H, HKV, D, kdt, BS, bt.size(1), 0, &ws_bytes), op);
  torch::Tensor ws = workspace(ws_bytes, qc);
  check_status(pa_decode_layer_step(out.data_ptr(), nullptr, qc.data_ptr(), io, k_cache.data_ptr(),
                                    v_cache.data_ptr(), kdt, append ? kn.data_ptr() : nullptr,
                                    append ? vn.data_ptr() : nullptr, bt.data_ptr<int32_t>(),
                                    ctx.data_ptr<int32_t>(), B, H, HKV, D, BS, NB, bt.size(1),
                                    scale, 0, ws.data_ptr(), ws_bytes, nullptr, stream_ptr()),
               op);
  return out;
}

// Many sequences in one call (pa_write_kv_batch): entry i of block_ids,
// starts, ks, vs is one write_kv call's (block_ids, start, k, v).  All sources
// are converted to one dtype (fp32 when they differ).
void write_kv_batch(std::vector<torch::Tensor> k_layers, std::vector<torch::Tensor> v_layers,
                    std::vector<torch::Tensor> block_ids, std::vector<int64_t> starts,
                    std::vector<torch::Tensor> ks, std::vector<torch::Tensor> vs,
                    torch::Tensor k_scales, torch::Tensor v_scales) {
  const char* op = "write_kv_batch";
  TORCH_CHECK(!k_layers.empty() && k_layers.size() == v_layers.size(),
              op, ": need one K and one V tensor per layer");
  const size_t n = block_ids.size();
  TORCH_CHECK(starts.size() == n && ks.size() == n && vs.size() == n,
              op, ": block_ids, starts, ks and vs need one entry per sequence");
  const torch::Tensor& k0 = k_layers[0];
  TORCH_CHECK(k0.is_cuda() && k0.dim() == 4, op, ": pool tensors must be CUDA [NB, BS, H, D]");
  const c10::cuda::CUDAGuard guard(k0.device());
  const int64_t L = (int64_t)k_layers.size();
  std::vector<void*> kp, vp;
  const int pdt = pool_dtype(k0, op);
  for (int64_t l = 0; l < L; ++l) {
    for (const torch::Tensor* t : {&k_layers[l], &v_layers[l]}) {
      TORCH_CHECK(t->is_contiguous() && t->sizes() == k0.sizes() &&
                      t->scalar_type() == k0.scalar_type() && t->device() == k0.device(),
                  op, ": pool tensors must be contiguous and alike");
    }
    kp.push_back(k_layers[l].data_ptr());
    vp.push_back(v_layers[l].data_ptr());
  }
  // one source dtype for the call
  torch::ScalarType sty = n ? ks[0].scalar_type() : torch::kFloat;
  for (size_t i = 0; i < n; ++i)
    if (ks[i].scalar_type() != sty || vs[i].scalar_type() != sty) sty = torch::kFloat;
  if (sty != torch::kFloat && sty != torch::kHalf && sty != torch::kBFloat16) sty = torch::kFloat;
  const int sdt = sty == torch::kHalf ? PA_DTYPE_F16 : sty == torch::kBFloat16 ? PA_DTYPE_BF16
                                                                                : PA_DTYPE_F32;
  std::vector<torch::Tensor> keep;  // device copies alive until the launch is queued
  std::vector<pa_kv_seq> seqs(n);
  for (size_t i = 0; i < n; ++i) {
    TORCH_CHECK(ks[i].dim() == 4 && vs[i].sizes() == ks[i].sizes() && ks[i].size(0) == L &&
                    ks[i].size(1) == k0.size(2) && ks[i].size(3) == k0.size(3),
                op, ": k, v of each sequence must be [n_layer, HKV, T, D] matching the pool");
    torch::Tensor kd = ks[i].to(k0.device(), sty);
    torch::Tensor vd = vs[i].to(k0.device(), sty);
    if (kd.stride(3) != 1 || vd.stride(3) != 1 || vd.strides() != kd.strides()) {
      kd = kd.contiguous();
      vd = vd.contiguous();
    }
    torch::Tensor ids = block_ids[i].to(k0.device(), torch::kInt32).contiguous();
    seqs[i] = pa_kv_seq{kd.data_ptr(), vd.data_ptr(), kd.stride(0), kd.stride(1), kd.stride(2),
                        ids.data_ptr<int32_t>(), ids.numel(), starts[i], kd.size(2)};
    keep.push_back(kd);
    keep.push_back(vd);
    keep.push_back(ids);
  }
  torch::Tensor ksc, vsc;
  if (k_scales.defined() && k_scales.numel()) ksc = k_scales.to(k0.device(), torch::kFloat).contiguous();
  if (v_scales.defined() && v_scales.numel()) vsc = v_scales.to(k0.device(), torch::kFloat).contiguous();
  for (const torch::Tensor* t : {&ksc, &vsc})
    TORCH_CHECK(!t->defined() || t->numel() == L * k0.size(2), op, ": scales must be [n_layer, HKV]");
  check_status(pa_write_kv_batch(kp.data(), vp.data(), pdt, sdt, seqs.data(), (int64_t)n, L,
                                 k0.size(2), k0.size(3), k0.size(1), k0.size(0),
                                 ksc.defined() ? ksc.data_ptr<float>() : nullptr,
                                 vsc.defined() ? vsc.data_ptr<float>() : nullptr, nullptr,
                                 stream_ptr()),
               op);
}

// One decode step's append: k_new / v_new [n_layer, B, HKV, D] go to position
// positions[b] (< 0: skipped) of sequence b through its block-table row.
// k_scales / v_scales: FP8 pools only ([n_layer, HKV], may be empty tensors).
void append_kv(std::vector<torch::Tensor> k_layers, std::vector<torch::Tensor> v_layers,
               torch::Tensor block_tables, torch::Tensor positions, torch::Tensor k_new,
               torch::Tensor v_new, torch::Tensor k_scales, torch::Tensor v_scales) {
  const char* op = "append_kv";
  TORCH_CHECK(!k_layers.empty() && k_layers.size() == v_layers.size(),
              op, ": need one K and one V tensor per layer");
  const torch::Tensor& k0 = k_layers[0];
  TORCH_CHECK(k0.is_cuda() && k0.dim() == 4, op, ": pool tensors must be CUDA [NB, BS, H, D]");
  const int64_t L = (int64_t)k_layers.size();
  TORCH_CHECK(k_new.dim() == 4 && v_new.sizes() == k_new.sizes() && k_new.size(0) == L &&
                  k_new.size(2) == k0.size(2) && k_new.size(3) == k0.size(3),
              op, ": k_new, v_new must be [n_layer, B, HKV, D]");
  const c10::cuda::CUDAGuard guard(k0.device());
  std::vector<void*> kp, vp;
  const int pdt = pool_dtype(k0, op);
  for (int64_t l = 0; l < L; ++l) {
    for (const torch::Tensor* t : {&k_layers[l], &v_layers[l]}) {
      TORCH_CHECK(t->is_contiguous() && t->sizes() == k0.sizes() &&
                      t->scalar_type() == k0.scalar_type() && t->device() == k0.device(),
                  op, ": pool tensors must be contiguous and alike");
    }
    kp.push_back(k_layers[l].data_ptr());
    vp.push_back(v_layers[l].data_ptr());
  }
  torch::Tensor kd = k_new.to(k0.device());
  torch::Tensor vd = v_new.to(k0.device());
  int sdt;
  switch (kd.scalar_type()) {
    case torch::kFloat: sdt = PA_DTYPE_F32; break;
    case torch::kHalf: sdt = PA_DTYPE_F16; break;
    case torch::kBFloat16: sdt = PA_DTYPE_BF16; break;
    default:
      kd = kd.to(torch::kFloat);
      sdt = PA_DTYPE_F32;
  }
  kd = kd.contiguous();
  vd = vd.to(kd.scalar_type()).contiguous();
  torch::Tensor bt = block_tables.to(k0.device(), torch::kInt32).contiguous();
  torch::Tensor pos = positions.to(k0.device(), torch::kInt32).contiguous();
  const int64_t B = kd.size(1);
  TORCH_CHECK(bt.dim() == 2 && bt.size(0) >= B && pos.numel() >= B,
              op, ": block_tables [B, MB] and positions [B] needed");
  torch::Tensor ks, vs;
  if (k_scales.defined() && k_scales.numel()) ks = k_scales.to(k0.device(), torch::kFloat).contiguous();
  if (v_scales.defined() && v_scales.numel()) vs = v_scales.to(k0.device(), torch::kFloat).contiguous();
  for (const torch::Tensor* t : {&ks, &vs})
    TORCH_CHECK(!t->defined() || t->numel() == L * k0.size(2), op, ": scales must be [n_layer, HKV]");
  check_status(pa_append_kv(kp.data(), vp.data(), pdt, kd.data_ptr(), vd.data_ptr(), sdt,
                            bt.data_ptr<int32_t>(), bt.size(1), pos.data_ptr<int32_t>(), B, L,
                            k0.size(2), k0.size(3), k0.size(1), k0.size(0),
                            ks.defined() ? ks.data_ptr<float>() : nullptr,
                            vs.defined() ? vs.data_ptr<float>() : nullptr, nullptr,
                            stream_ptr()),
               op);
}

// Counts of (out-of-range block ids, over-long contexts); synchronises.
std::tuple<int64_t, int64_t> validate_block_tables(torch::Tensor block_tables,
                                                   torch::Tensor context_lens,
                                                   int64_t num_blocks, int64_t block_size) {
  TORCH_CHECK(block_tables.is_cuda(), "block_tables must be on CUDA");
  const c10::cuda::CUDAGuard guard(block_tables.device());
  torch::Tensor bt = block_tables.to(torch::kInt32).contiguous();
  torch::Tensor ctx = context_lens.to(bt.device(), torch::kInt32).contiguous();
  torch::Tensor counts = torch::zeros({2}, bt.options());
  check_status(pa_validate_block_tables(bt.data_ptr<int32_t>(), ctx.data_ptr<int32_t>(),
                                        bt.size(0), bt.size(1), block_size, num_blocks,
                                        counts.data_ptr<int32_t>(), stream_ptr()),
               "validate_block_tables");
  torch::Tensor h = counts.cpu();
  return {h[0].item<int64_t>(), h[1].item<int64_t>()};
}

// Log-sum-exp merge of R partial decodes: outs [R, B, H, D], lses [R, B, H].
std::tuple<torch::Tensor, torch::Tensor> merge_states(torch::Tensor outs, torch::Tensor lses) {
  TORCH_CHECK(outs.is_cuda() && outs.scalar_type() == torch::kFloat && outs.dim() == 4,
              "merge_states: outs must be CUDA float [R, B, H, D]");
  TORCH_CHECK(lses.sizes() == outs.sizes().slice(0, 3), "merge_states: lses must be [R, B, H]");
  const c10::cuda::CUDAGuard guard(outs.device());
  torch::Tensor o = outs.contiguous();
  torch::Tensor l = lses.to(torch::kFloat).contiguous();
  torch::Tensor out = torch::empty({o.size(1), o.size(2), o.size(3)}, o.options());
  torch::Tensor lse = torch::empty({o.size(1), o.size(2)}, o.options());
  check_status(pa_merge_states(out.data_ptr<float>(), lse.data_ptr<float>(), o.data_ptr<float>(),
                               l.data_ptr<float>(), o.size(0), o.size(1) * o.size(2), o.size(3),
                               stream_ptr()),
               "merge_states");
  return {out, lse};
}

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  m.doc() = "B200 paged attention: the gb10-attn operator API over libpa_b200.so";
  m.def("paged_attention", &paged_attention);
  m.def("paged_attention_v2", &paged_attention_v2);
  m.def("paged_attention_v3", &paged_attention_v3);
  m.def("paged_attention_v3_lse", &paged_attention_v3_lse);
  m.def("choose_num_splits", &choose_num_splits);
  m.def("paged_attention_prefill", &paged_attention_prefill);
  m.def("paged_attention_prefill_wmma", &paged_attention_prefill_wmma);
  m.def("paged_attention_prefill_simt", &paged_attention_prefill_simt);
  m.def("write_kv", &write_kv);
  m.def("write_kv_scaled", &write_kv_scaled);
  m.def("write_kv_batch", &write_kv_batch);
  m.def("decode_layer_step", &decode_layer_step);
  m.def("append_kv", &append_kv);
  m.def("paged_attention_v3_fp8", &paged_attention_v3_fp8);
  m.def("validate_block_tables", &validate_block_tables);
  m.def("merge_states", &merge_states);
}
