// libgwb200_torch.so: the TORCH_LIBRARY face of libgwb200.so.
//
// Counterpart of the reference's `_cozy_kernels` extension
// (csrc/cozy_kernels/ops.cpp:29-36, loaded by
// src/gen_worker/models/native_kernels.py:96-143 with torch.ops.load_library
// from GEN_WORKER_NATIVE_KERNELS_LIB): the same namespace `cozy_kernels`, the
// same `build_info() -> str` and `probe_add_one(Tensor) -> Tensor` the
// reference's loader probes, and the quantized-linear ops of this library on
// top. Every op checks device, dtype, shape and contiguity with TORCH_CHECK,
// allocates its outputs on the input's device, launches on the current CUDA
// stream through the C ABI (include/gwb200.h) and raises on a non-zero status.
// There is no CPU kernel: a CPU tensor is refused.
#include <ATen/ATen.h>
#include <c10/cuda/CUDAStream.h>
#include <torch/library.h>
#include <torch/version.h>

#include <string>
#include <tuple>

#include "../../include/gwb200.h"

namespace gwb200_torch {

using at::Tensor;

void* stream_of(const Tensor& t) {
  return static_cast<void*>(c10::cuda::getCurrentCUDAStream(t.device().index()).stream());
}

void check_status(int rc, const char* what) {
  TORCH_CHECK(rc == 0, what, ": ", gwb_status_string(rc), " (status ", rc, ")");
}

void need(const Tensor& t, const char* name, at::ScalarType dtype, int64_t ndim) {
  TORCH_CHECK(t.is_cuda(), name, " must be a CUDA tensor (no CPU path)");
  TORCH_CHECK(t.scalar_type() == dtype, name, " must be ", dtype, ", got ", t.scalar_type());
  TORCH_CHECK(t.dim() == ndim, name, " must be ", ndim, "-D, got ", t.dim(), "-D");
  TORCH_CHECK(t.is_contiguous(), name, " must be contiguous");
}

const void* opt_ptr(const c10::optional<Tensor>& t) {
  return t.has_value() ? t->data_ptr() : nullptr;
}

int64_t rank_pad_of(const c10::optional<Tensor>& proj_down_t) {
  return proj_down_t.has_value() ? proj_down_t->size(0) : 0;
}

std::string build_info() {
  char buf[160];
  gwb_build_info(buf, sizeof(buf));
  return std::string("torch=") + TORCH_VERSION + " " + buf;
}

Tensor probe_add_one(const Tensor& x) {
  need(x, "x", at::kFloat, x.dim());
  Tensor y = at::empty_like(x);
  check_status(gwb_probe_add_one(x.data_ptr<float>(), y.data_ptr<float>(), x.numel(),
                                 stream_of(x)),
               "probe_add_one");
  return y;
}

// x2 bf16 [M, K] -> (a_q8 u8 [M, K], a_scale_k8 f16 [K/64, M, 8], la bf16 [M, rank_pad])
std::tuple<Tensor, Tensor, Tensor> svdq_w4a4_quant(const Tensor& x2,
                                                   const c10::optional<Tensor>& smooth,
                                                   const c10::optional<Tensor>& proj_down_t) {
  need(x2, "x2", at::kBFloat16, 2);
  if (smooth.has_value()) need(*smooth, "smooth", at::kBFloat16, 1);
  if (proj_down_t.has_value()) need(*proj_down_t, "proj_down_t", at::kBFloat16, 2);
  const int64_t m = x2.size(0), k = x2.size(1), rp = rank_pad_of(proj_down_t);
  auto u8 = x2.options().dtype(at::kByte);
  Tensor a_q8 = at::empty({m, k}, u8);
  Tensor a_sk8 = at::empty({k / 64, m, 8}, x2.options().dtype(at::kHalf));
  Tensor la = at::empty({m, rp}, x2.options());
  check_status(gwb_svdq_w4a4_quant_mma(x2.data_ptr(), opt_ptr(smooth), opt_ptr(proj_down_t), m,
                                       k, (int)rp, a_q8.data_ptr(), a_sk8.data_ptr(),
                                       rp ? la.data_ptr() : nullptr, stream_of(x2)),
               "svdq_w4a4_quant");
  return {a_q8, a_sk8, la};
}

// The GEMM on the weights as stored: weight u8 [N, K/2], weight_scale f16 [N, K/64].
Tensor svdq_w4a4_gemm(const Tensor& a_q8, const Tensor& a_scale_k8, const Tensor& weight,
                      const Tensor& weight_scale, const c10::optional<Tensor>& la,
                      const c10::optional<Tensor>& proj_up, const c10::optional<Tensor>& bias,
                      bool gelu) {
  need(a_q8, "a_q8", at::kByte, 2);
  need(a_scale_k8, "a_scale_k8", at::kHalf, 3);
  need(weight, "weight", at::kByte, 2);
  need(weight_scale, "weight_scale", at::kHalf, 2);
  const int64_t m = a_q8.size(0), k = a_q8.size(1), n = weight.size(0);
  TORCH_CHECK(weight.size(1) * 2 == k && weight_scale.size(0) == n &&
                  weight_scale.size(1) == k / 64,
              "stored weight / weight_scale do not match activation K ", k);
  int64_t rp = 0;
  if (la.has_value() && proj_up.has_value() && la->size(1) > 0) {
    need(*la, "la", at::kBFloat16, 2);
    need(*proj_up, "proj_up", at::kBFloat16, 2);
    rp = la->size(1);
    TORCH_CHECK(proj_up->size(0) == n && proj_up->size(1) == rp, "proj_up must be [N, rank_pad]");
  }
  if (bias.has_value()) need(*bias, "bias", at::kBFloat16, 1);
  Tensor out = at::empty({m, n}, a_q8.options().dtype(at::kBFloat16));
  check_status(gwb_svdq_w4a4_gemm_stored(a_q8.data_ptr(), a_scale_k8.data_ptr(),
                                         weight.data_ptr(), weight_scale.data_ptr(),
                                         rp ? la->data_ptr() : nullptr,
                                         rp ? proj_up->data_ptr() : nullptr, opt_ptr(bias), m,
                                         n, k, (int)rp, gelu ? 1 : 0, out.data_ptr(),
                                         stream_of(a_q8)),
               "svdq_w4a4_gemm");
  return out;
}

// Whole SvdqLinear forward on the weights as stored (two launches).
Tensor svdq_w4a4_linear(const Tensor& x2, const c10::optional<Tensor>& smooth,
                        const c10::optional<Tensor>& proj_down_t, const Tensor& weight,
                        const Tensor& weight_scale, const c10::optional<Tensor>& proj_up,
                        const c10::optional<Tensor>& bias, bool gelu) {
  auto q = svdq_w4a4_quant(x2, smooth, proj_down_t);
  const bool lr = proj_down_t.has_value();
  return svdq_w4a4_gemm(std::get<0>(q), std::get<1>(q), weight, weight_scale,
                        lr ? c10::optional<Tensor>(std::get<2>(q)) : c10::nullopt,
                        lr ? proj_up : c10::nullopt, bias, gelu);
}

// FP8 e4m3 rowwise (Fp8ScaledLinear.forward): weight e4m3 bytes or
// float8_e4m3fn [N, K], weight_scale f32 [N].
Tensor fp8_linear(const Tensor& x2, const Tensor& weight, const Tensor& weight_scale,
                  const c10::optional<Tensor>& bias, bool gelu) {
  need(x2, "x2", at::kBFloat16, 2);
  TORCH_CHECK(weight.is_cuda() && weight.is_contiguous() && weight.dim() == 2 &&
                  weight.element_size() == 1,
              "weight must be contiguous CUDA e4m3 bytes [N, K]");
  need(weight_scale, "weight_scale", at::kFloat, 1);
  if (bias.has_value()) need(*bias, "bias", at::kBFloat16, 1);
  const int64_t m = x2.size(0), k = x2.size(1), n = weight.size(0);
  TORCH_CHECK(weight.size(1) == k && weight_scale.size(0) == n, "weight must be [N, K]");
  Tensor q = at::empty({m, k}, x2.options().dtype(at::kByte));
  Tensor s = at::empty({m}, x2.options().dtype(at::kFloat));
  Tensor out = at::empty({m, n}, x2.options());
  check_status(gwb_fp8_linear(x2.data_ptr(), weight.data_ptr(), weight_scale.data_ptr<float>(),
                              opt_ptr(bias), m, n, k, gelu ? 1 : 0, q.data_ptr(), s.data_ptr(),
                              out.data_ptr(), stream_of(x2)),
               "fp8_linear");
  return out;
}

}  // namespace gwb200_torch

TORCH_LIBRARY(cozy_kernels, m) {
  m.def("build_info", &gwb200_torch::build_info);
  m.def("probe_add_one(Tensor x) -> Tensor");
  m.def("svdq_w4a4_quant(Tensor x2, Tensor? smooth, Tensor? proj_down_t) -> (Tensor, Tensor, Tensor)");
  m.def("svdq_w4a4_gemm(Tensor a_q8, Tensor a_scale_k8, Tensor weight, Tensor weight_scale, "
        "Tensor? la, Tensor? proj_up, Tensor? bias, bool gelu) -> Tensor");
  m.def("svdq_w4a4_linear(Tensor x2, Tensor? smooth, Tensor? proj_down_t, Tensor weight, "
        "Tensor weight_scale, Tensor? proj_up, Tensor? bias, bool gelu) -> Tensor");
  m.def("fp8_linear(Tensor x2, Tensor weight, Tensor weight_scale, Tensor? bias, bool gelu) "
        "-> Tensor");
}

TORCH_LIBRARY_IMPL(cozy_kernels, CUDA, m) {
  m.impl("probe_add_one", &gwb200_torch::probe_add_one);
  m.impl("svdq_w4a4_quant", &gwb200_torch::svdq_w4a4_quant);
  m.impl("svdq_w4a4_gemm", &gwb200_torch::svdq_w4a4_gemm);
  m.impl("svdq_w4a4_linear", &gwb200_torch::svdq_w4a4_linear);
  m.impl("fp8_linear", &gwb200_torch::fp8_linear);
}
