// gdn_torch_op.cpp -- torch custom ops over the C ABI (libgdn_sm120_op.so).
//
// Keeps the reference op byte-compatible: namespace gdn_sm120, schema
//   state_update(Tensor S_data, Tensor S_scales, Tensor k, Tensor v,
//                float alpha, float beta, int d) -> (Tensor, Tensor)
// with the reference's input checks and messages and freshly allocated
// outputs on the current stream (src/ops/gdn_op.cu:44-110 of
// bojak83318/blackwell-kernel-sm_120).  The batched GDN ops live in the same
// namespace; every op also has a Meta kernel so torch.compile (as vLLM runs
// it) can trace through them.
#include <ATen/ATen.h>
#include <c10/cuda/CUDAGuard.h>
#include <c10/cuda/CUDAStream.h>
#include <torch/library.h>

#include <tuple>

#include "gdn_b200.h"

namespace {

cudaStream_t cur_stream(const at::Tensor& t) {
  return c10::cuda::getCurrentCUDAStream(t.device().index()).stream();
}

void need(const at::Tensor& t, at::ScalarType dt, const char* name) {
  TORCH_CHECK(t.is_cuda(), name, " must be a CUDA tensor");
  TORCH_CHECK(t.scalar_type() == dt, name, " must be ", c10::toString(dt));
  TORCH_CHECK(t.is_contiguous(), name, " must be contiguous");
}

void check_rc(int rc, const char* fn) {
  TORCH_CHECK(rc == GDN_OK, fn, " failed with code ", rc, ": ", gdn_b200_error_string(rc));
}

// ---- state_update (reference schema) -------------------------------------------------

std::tuple<at::Tensor, at::Tensor> state_update_cuda(const at::Tensor& S_data, const at::Tensor& S_scales,
                                                     const at::Tensor& k, const at::Tensor& v, double alpha,
                                                     double beta, int64_t d) {
  // Checks and messages of src/ops/gdn_op.cu:54-74.
  TORCH_CHECK(S_data.is_cuda(), "S_data must be a CUDA tensor");
  TORCH_CHECK(S_scales.is_cuda(), "S_scales must be a CUDA tensor");
  TORCH_CHECK(k.is_cuda(), "k must be a CUDA tensor");
  TORCH_CHECK(v.is_cuda(), "v must be a CUDA tensor");
  TORCH_CHECK(S_data.scalar_type() == at::kByte, "S_data must be uint8");
  TORCH_CHECK(S_scales.scalar_type() == at::kByte, "S_scales must be uint8");
  TORCH_CHECK(k.scalar_type() == at::kBFloat16, "k must be bfloat16");
  TORCH_CHECK(v.scalar_type() == at::kBFloat16, "v must be bfloat16");
  TORCH_CHECK(S_data.is_contiguous(), "S_data must be contiguous");
  TORCH_CHECK(S_scales.is_contiguous(), "S_scales must be contiguous");
  TORCH_CHECK(k.is_contiguous(), "k must be contiguous");
  TORCH_CHECK(v.is_contiguous(), "v must be contiguous");
  const int64_t n = d * d;
  TORCH_CHECK(S_data.numel() == n / 2, "S_data size mismatch: expected ", n / 2, " got ", S_data.numel());
  TORCH_CHECK(S_scales.numel() == n / 16, "S_scales size mismatch");
  TORCH_CHECK(k.numel() == d, "k size mismatch");
  TORCH_CHECK(v.numel() == d, "v size mismatch");
  TORCH_CHECK(n % 16 == 0, "d*d must be divisible by 16 for NVFP4 block scaling");
  c10::cuda::CUDAGuard guard(S_data.device());
  auto opts = at::TensorOptions().dtype(at::kByte).device(S_data.device());
  at::Tensor out_data = at::empty({n / 2}, opts);
  at::Tensor out_scales = at::empty({n / 16}, opts);
  const int rc = launch_gdn_state_update(
      S_data.data_ptr<uint8_t>(), S_scales.data_ptr<uint8_t>(),
      reinterpret_cast<const gdn_bf16_t*>(k.data_ptr()), reinterpret_cast<const gdn_bf16_t*>(v.data_ptr()),
      out_data.data_ptr<uint8_t>(), out_scales.data_ptr<uint8_t>(), static_cast<float>(alpha),
      static_cast<float>(beta), static_cast<int>(d), cur_stream(S_data));
  TORCH_CHECK(rc == 0, "launch_gdn_state_update failed with code ", rc);
  return {out_data, out_scales};
}

std::tuple<at::Tensor, at::Tensor> state_update_meta(const at::Tensor& S_data, const at::Tensor&, const at::Tensor&,
                                                     const at::Tensor&, double, double, int64_t d) {
  auto opts = at::TensorOptions().dtype(at::kByte).device(S_data.device());
  return {at::empty({d * d / 2}, opts), at::empty({d * d / 16}, opts)};
}

// ---- codec ---------------------------------------------------------------------------------

std::tuple<at::Tensor, at::Tensor> quantize_cuda(const at::Tensor& x, int64_t scale_mode) {
  need(x, at::kFloat, "x");
  c10::cuda::CUDAGuard guard(x.device());
  const int64_t n = x.numel();
  auto opts = at::TensorOptions().dtype(at::kByte).device(x.device());
  at::Tensor codes = at::empty({n / 2}, opts), scales = at::empty({n / 16}, opts);
  check_rc(gdn_nvfp4_quantize(x.data_ptr<float>(), codes.data_ptr<uint8_t>(), scales.data_ptr<uint8_t>(), n,
                              (int32_t)scale_mode, cur_stream(x)),
           "gdn_nvfp4_quantize");
  return {codes, scales};
}

std::tuple<at::Tensor, at::Tensor> quantize_meta(const at::Tensor& x, int64_t) {
  auto opts = at::TensorOptions().dtype(at::kByte).device(x.device());
  return {at::empty({x.numel() / 2}, opts), at::empty({x.numel() / 16}, opts)};
}

at::Tensor dequantize_cuda(const at::Tensor& codes, const at::Tensor& scales, int64_t scale_mode) {
  need(codes, at::kByte, "codes");
  need(scales, at::kByte, "scales");
  TORCH_CHECK(scales.numel() * 8 == codes.numel(), "scales must hold one byte per 16 elements");
  c10::cuda::CUDAGuard guard(codes.device());
  const int64_t n = codes.numel() * 2;
  at::Tensor out = at::empty({n}, at::TensorOptions().dtype(at::kFloat).device(codes.device()));
  check_rc(gdn_nvfp4_dequantize(codes.data_ptr<uint8_t>(), scales.data_ptr<uint8_t>(), out.data_ptr<float>(), n,
                                (int32_t)scale_mode, cur_stream(codes)),
           "gdn_nvfp4_dequantize");
  return out;
}

at::Tensor dequantize_meta(const at::Tensor& codes, const at::Tensor&, int64_t) {
  return at::empty({codes.numel() * 2}, at::TensorOptions().dtype(at::kFloat).device(codes.device()));
}

// ---- fused decode over the slot-indexed pool ------------------------------------------------

at::Tensor decode_cuda(const at::Tensor& q, const at::Tensor& k, const at::Tensor& v, const at::Tensor& g,
                       const at::Tensor& beta, const at::Tensor& slot_idx, at::Tensor& pool_codes,
                       at::Tensor& pool_scales, at::Tensor& pool_gscale, double q_scale, int64_t scale_mode,
                       double gscale_den) {
  TORCH_CHECK(q.dim() == 3 && k.dim() == 3 && v.dim() == 3, "q, k, v must be [B, heads, D]");
  const int64_t B = q.size(0), HK = q.size(1), D = q.size(2), HV = v.size(1);
  for (const at::Tensor* t : {&q, &k, &v}) {
    TORCH_CHECK(t->is_cuda() && t->scalar_type() == at::kBFloat16, "q, k, v must be CUDA bfloat16");
    TORCH_CHECK(t->stride(2) == 1 && t->stride(1) == D, "q, k, v heads must be contiguous");
  }
  TORCH_CHECK(k.sizes() == q.sizes() && v.size(0) == B && v.size(2) == D, "q, k, v shape mismatch");
  need(g, at::kFloat, "g");
  need(beta, at::kFloat, "beta");
  need(slot_idx, at::kInt, "slot_idx");
  need(pool_codes, at::kByte, "pool_codes");
  need(pool_scales, at::kByte, "pool_scales");
  need(pool_gscale, at::kFloat, "pool_gscale");
  TORCH_CHECK(g.numel() == B * HV && beta.numel() == B * HV && slot_idx.numel() == B, "g/beta/slot_idx size");
  TORCH_CHECK(pool_codes.dim() == 4 && pool_codes.size(1) == HV && pool_codes.size(2) == D &&
                  pool_codes.size(3) == D / 2,
              "pool_codes must be [slots, HV, D, D/2]");
  c10::cuda::CUDAGuard guard(q.device());
  at::Tensor out = at::empty({B, HV, D}, q.options());
  gdn_decode_params p{};
  p.batch = (int32_t)B;
  p.num_k_heads = (int32_t)HK;
  p.num_v_heads = (int32_t)HV;
  p.head_dim = (int32_t)D;
  p.num_slots = pool_codes.size(0);
  p.q = reinterpret_cast<const gdn_bf16_t*>(q.data_ptr());
  p.k = reinterpret_cast<const gdn_bf16_t*>(k.data_ptr());
  p.v = reinterpret_cast<const gdn_bf16_t*>(v.data_ptr());
  p.q_stride = q.stride(0);
  p.k_stride = k.stride(0);
  p.v_stride = v.stride(0);
  p.g = g.data_ptr<float>();
  p.beta = beta.data_ptr<float>();
  p.slot_idx = slot_idx.data_ptr<int32_t>();
  p.pool_codes = pool_codes.data_ptr<uint8_t>();
  p.pool_scales = pool_scales.data_ptr<uint8_t>();
  p.pool_gscale = pool_gscale.data_ptr<float>();
  p.out = reinterpret_cast<gdn_bf16_t*>(out.data_ptr());
  p.q_scale = (float)q_scale;
  p.scale_mode = (int32_t)scale_mode;
  p.gscale_den = (float)gscale_den;
  check_rc(gdn_decode(&p, cur_stream(q)), "gdn_decode");
  return out;
}

at::Tensor decode_meta(const at::Tensor& q, const at::Tensor&, const at::Tensor& v, const at::Tensor&,
                       const at::Tensor&, const at::Tensor&, at::Tensor&, at::Tensor&, at::Tensor&, double, int64_t,
                       double) {
  return at::empty({q.size(0), v.size(1), q.size(2)}, q.options());
}

// ---- chunked prefill over packed variable-length sequences --------------------------------

at::Tensor prefill_cuda(const at::Tensor& q, const at::Tensor& k, const at::Tensor& v, const at::Tensor& g,
                        const at::Tensor& beta, const at::Tensor& cu_seqlens,
                        const c10::optional<at::Tensor>& slot_idx, const c10::optional<at::Tensor>& has_initial_state,
                        at::Tensor& pool_codes, at::Tensor& pool_scales, at::Tensor& pool_gscale, double q_scale,
                        int64_t scale_mode, double gscale_den) {
  TORCH_CHECK(q.dim() == 3 && k.dim() == 3 && v.dim() == 3, "q, k, v must be [T, heads, D]");
  const int64_t T = q.size(0), HK = q.size(1), D = q.size(2), HV = v.size(1);
  for (const at::Tensor* t : {&q, &k, &v}) {
    TORCH_CHECK(t->is_cuda() && t->scalar_type() == at::kBFloat16, "q, k, v must be CUDA bfloat16");
    TORCH_CHECK(t->stride(2) == 1 && t->stride(1) == D, "q, k, v heads must be contiguous");
  }
  TORCH_CHECK(k.sizes() == q.sizes() && v.size(0) == T && v.size(2) == D, "q, k, v shape mismatch");
  need(g, at::kFloat, "g");
  need(beta, at::kFloat, "beta");
  need(cu_seqlens, at::kInt, "cu_seqlens");
  TORCH_CHECK(g.numel() == T * HV && beta.numel() == T * HV, "g/beta must be [T, HV]");
  const int64_t N = cu_seqlens.numel() - 1;
  TORCH_CHECK(N >= 0, "cu_seqlens needs N + 1 entries");
  c10::cuda::CUDAGuard guard(q.device());
  at::Tensor out = at::empty({T, HV, D}, q.options());
  gdn_prefill_params p{};
  p.num_seqs = (int32_t)N;
  p.num_k_heads = (int32_t)HK;
  p.num_v_heads = (int32_t)HV;
  p.head_dim = (int32_t)D;
  p.total_tokens = T;
  p.q = reinterpret_cast<const gdn_bf16_t*>(q.data_ptr());
  p.k = reinterpret_cast<const gdn_bf16_t*>(k.data_ptr());
  p.v = reinterpret_cast<const gdn_bf16_t*>(v.data_ptr());
  p.q_stride = q.stride(0);
  p.k_stride = k.stride(0);
  p.v_stride = v.stride(0);
  p.g = g.data_ptr<float>();
  p.beta = beta.data_ptr<float>();
  p.cu_seqlens = cu_seqlens.data_ptr<int32_t>();
  if (has_initial_state.has_value()) {
    need(*has_initial_state, at::kBool, "has_initial_state");
    TORCH_CHECK(has_initial_state->numel() == N, "has_initial_state must be [N]");
    p.has_initial_state = reinterpret_cast<const uint8_t*>(has_initial_state->data_ptr());
  }
  if (slot_idx.has_value()) {
    need(*slot_idx, at::kInt, "slot_idx");
    TORCH_CHECK(slot_idx->numel() == N, "slot_idx must be [N]");
    need(pool_codes, at::kByte, "pool_codes");
    need(pool_scales, at::kByte, "pool_scales");
    need(pool_gscale, at::kFloat, "pool_gscale");
    TORCH_CHECK(pool_codes.dim() == 4 && pool_codes.size(1) == HV && pool_codes.size(2) == D &&
                    pool_codes.size(3) == D / 2,
                "pool_codes must be [slots, HV, D, D/2]");
    p.num_slots = pool_codes.size(0);
    p.slot_idx = slot_idx->data_ptr<int32_t>();
    p.pool_codes = pool_codes.data_ptr<uint8_t>();
    p.pool_scales = pool_scales.data_ptr<uint8_t>();
    p.pool_gscale = pool_gscale.data_ptr<float>();
  }
  p.out = reinterpret_cast<gdn_bf16_t*>(out.data_ptr());
  p.q_scale = (float)q_scale;
  p.scale_mode = (int32_t)scale_mode;
  p.gscale_den = (float)gscale_den;
  check_rc(gdn_prefill(&p, cur_stream(q)), "gdn_prefill");
  return out;
}

at::Tensor prefill_meta(const at::Tensor& q, const at::Tensor&, const at::Tensor& v, const at::Tensor&,
                        const at::Tensor&, const at::Tensor&, const c10::optional<at::Tensor>&,
                        const c10::optional<at::Tensor>&, at::Tensor&, at::Tensor&, at::Tensor&, double, int64_t,
                        double) {
  return at::empty({q.size(0), v.size(1), q.size(2)}, q.options());
}

}  // namespace

TORCH_LIBRARY(gdn_sm120, m) {
  m.def("state_update(Tensor S_data, Tensor S_scales, Tensor k, Tensor v, "
        "float alpha, float beta, int d) -> (Tensor, Tensor)");
  m.def("nvfp4_quantize(Tensor x, int scale_mode=0) -> (Tensor, Tensor)");
  m.def("nvfp4_dequantize(Tensor codes, Tensor scales, int scale_mode=0) -> Tensor");
  m.def("decode(Tensor q, Tensor k, Tensor v, Tensor g, Tensor beta, Tensor slot_idx, "
        "Tensor(a!) pool_codes, Tensor(b!) pool_scales, Tensor(c!) pool_gscale, "
        "float q_scale=0., int scale_mode=0, float gscale_den=0.) -> Tensor");
  m.def("prefill(Tensor q, Tensor k, Tensor v, Tensor g, Tensor beta, Tensor cu_seqlens, Tensor? slot_idx, "
        "Tensor? has_initial_state, Tensor(a!) pool_codes, Tensor(b!) pool_scales, Tensor(c!) pool_gscale, "
        "float q_scale=0., int scale_mode=0, float gscale_den=0.) -> Tensor");
}

TORCH_LIBRARY_IMPL(gdn_sm120, CUDA, m) {
  m.impl("state_update", &state_update_cuda);
  m.impl("nvfp4_quantize", &quantize_cuda);
  m.impl("nvfp4_dequantize", &dequantize_cuda);
  m.impl("decode", &decode_cuda);
  m.impl("prefill", &prefill_cuda);
}

TORCH_LIBRARY_IMPL(gdn_sm120, Meta, m) {
  m.impl("state_update", &state_update_meta);
  m.impl("nvfp4_quantize", &quantize_meta);
  m.impl("nvfp4_dequantize", &dequantize_meta);
  m.impl("decode", &decode_meta);
  m.impl("prefill", &prefill_meta);
}
