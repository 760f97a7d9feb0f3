// torch operator library `aot_kernel`: the same schemas as the reference's
// registration (aot_kernel/csrc/registration.cc:10-25) plus the fused ops
// (silu_mul_forward, add_rmsnorm_forward, gemm_silu_mul) and scaled_gemm, the
// 8-bit GEMM the reference provides as a Triton kernel.
// Each kernel checks its tensors, pins the device, and calls the C ABI of
// libaotk (include/aotk.h) on the current torch stream.  Unlike the
// reference, launches go to at::cuda::getCurrentCUDAStream() under a device
// guard rather than to the legacy default stream, and every launch status is
// checked.
#include <Python.h>
#include <ATen/ATen.h>
#include <c10/cuda/CUDAGuard.h>
#include <c10/cuda/CUDAStream.h>
#include <torch/library.h>

#include "aotk.h"

namespace {

int aotk_dtype(const at::Tensor& t, const char* op) {
  switch (t.scalar_type()) {
    case at::ScalarType::Float: return AOTK_FLOAT32;
    case at::ScalarType::Half: return AOTK_FLOAT16;
    case at::ScalarType::BFloat16: return AOTK_BFLOAT16;
    default: TORCH_CHECK(false, "[", op, "] unsupported dtype: ", t.scalar_type());
  }
  return -1;
}

void* current_stream(const at::Tensor& t) {
  return at::cuda::getCurrentCUDAStream(t.device().index()).stream();
}

void check_status(int status, const char* op) {
  TORCH_CHECK(status == AOTK_OK, "[", op, "] ", aotk_last_error());
}

void check_cuda(const at::Tensor& t, const char* op, const char* name) {
  TORCH_CHECK(t.is_cuda(), "[", op, "] ", name, " must be a CUDA tensor, got ", t.device());
}

void check_same(const at::Tensor& a, const at::Tensor& b, const char* op, const char* an,
                const char* bn) {
  TORCH_CHECK(a.device() == b.device(), "[", op, "] ", an, " and ", bn,
              " are not on the same device: ", a.device(), " vs ", b.device());
  TORCH_CHECK(a.scalar_type() == b.scalar_type(), "[", op, "] ", an, " and ", bn,
              " have different dtypes: ", a.scalar_type(), " vs ", b.scalar_type());
}

void check_out_like(const at::Tensor& out, const at::Tensor& x, const char* op) {
  check_cuda(out, op, "out");
  check_same(out, x, op, "out", "x");
  TORCH_CHECK(out.is_contiguous(), "[", op, "] out is not contiguous");
  TORCH_CHECK(out.sizes() == x.sizes(), "[", op, "] out shape ", out.sizes(),
              " does not match input shape ", x.sizes());
}

void relu_forward(at::Tensor out, at::Tensor x) {
  const char* op = "relu_forward";
  check_cuda(x, op, "x");
  TORCH_CHECK(x.is_contiguous(), "[", op, "] x must be contiguous");
  check_out_like(out, x, op);
  c10::cuda::CUDAGuard guard(x.device());
  check_status(aotk_relu_forward(out.data_ptr(), x.data_ptr(), x.numel(), aotk_dtype(x, op),
                                 current_stream(x)),
               op);
}

void silu_forward(at::Tensor out, at::Tensor x) {
  const char* op = "silu_forward";
  check_cuda(x, op, "x");
  TORCH_CHECK(x.is_contiguous(), "[", op, "] x must be contiguous");
  check_out_like(out, x, op);
  c10::cuda::CUDAGuard guard(x.device());
  check_status(aotk_silu_forward(out.data_ptr(), x.data_ptr(), x.numel(), aotk_dtype(x, op),
                                 current_stream(x)),
               op);
}

// gate / up / out: same shape; each either contiguous or a 2-D view whose
// rows are contiguous (e.g. the two column halves of a [rows, 2*cols] tensor).
int64_t row_stride(const at::Tensor& t, const char* op, const char* name) {
  if (t.is_contiguous()) return t.dim() == 0 ? 1 : t.size(-1);
  TORCH_CHECK(t.dim() == 2 && t.stride(1) == 1 && t.stride(0) >= t.size(1), "[", op, "] ", name,
              " must be contiguous or a 2-D view with contiguous rows");
  return t.stride(0);
}

void silu_mul_forward(at::Tensor out, at::Tensor gate, at::Tensor up) {
  const char* op = "silu_mul_forward";
  check_cuda(gate, op, "gate");
  check_cuda(up, op, "up");
  check_cuda(out, op, "out");
  check_same(gate, up, op, "gate", "up");
  check_same(out, gate, op, "out", "gate");
  TORCH_CHECK(gate.sizes() == up.sizes() && out.sizes() == gate.sizes(), "[", op,
              "] shape mismatch: gate ", gate.sizes(), " up ", up.sizes(), " out ", out.sizes());
  const int64_t cols = gate.dim() == 0 ? 1 : gate.size(-1);
  const int64_t rows = cols == 0 ? 0 : gate.numel() / cols;
  const int64_t gs = row_stride(gate, op, "gate");
  const int64_t us = row_stride(up, op, "up");
  const int64_t os = row_stride(out, op, "out");
  c10::cuda::CUDAGuard guard(gate.device());
  check_status(aotk_silu_mul_forward(out.data_ptr(), os, gate.data_ptr(), gs, up.data_ptr(), us,
                                     rows, cols, aotk_dtype(gate, op), current_stream(gate)),
               op);
}

void rmsnorm_forward(at::Tensor out, at::Tensor x, at::Tensor weight, double eps) {
  const char* op = "rmsnorm";
  check_cuda(x, op, "x");
  check_cuda(weight, op, "weight");
  check_same(x, weight, op, "x", "weight");
  TORCH_CHECK(x.is_contiguous(), "[", op, "] x is not contiguous");
  TORCH_CHECK(weight.is_contiguous(), "[", op, "] weight is not contiguous");
  TORCH_CHECK(weight.dim() == 1, "[", op, "] dim of weight is not 1, got ", weight.dim());
  TORCH_CHECK(x.dim() >= 1 && weight.size(0) == x.size(-1), "[", op,
              "] weight length must equal x.size(-1), got weight_length=", weight.size(0),
              " x.size(-1)=", x.dim() >= 1 ? x.size(-1) : 0);
  check_out_like(out, x, op);
  if (x.numel() == 0) return;
  const int64_t cols = x.size(-1);
  const int64_t rows = x.numel() / cols;
  c10::cuda::CUDAGuard guard(x.device());
  check_status(aotk_rmsnorm_forward(out.data_ptr(), x.data_ptr(), weight.data_ptr(), rows, cols,
                                    eps, aotk_dtype(x, op), current_stream(x)),
               op);
}

// rstd[r] = rsqrt(mean(x[r]^2) + eps), fp32, one value per row of x.
void rmsnorm_rstd(at::Tensor rstd, at::Tensor x, double eps) {
  const char* op = "rmsnorm_rstd";
  check_cuda(x, op, "x");
  check_cuda(rstd, op, "rstd");
  TORCH_CHECK(x.is_contiguous() && x.dim() >= 1, "[", op, "] x must be contiguous and at least 1-D");
  TORCH_CHECK(rstd.scalar_type() == at::kFloat && rstd.is_contiguous() && rstd.device() == x.device(),
              "[", op, "] rstd must be a contiguous float32 tensor on x's device");
  const int64_t cols = x.dim() >= 1 ? x.size(-1) : 0;
  const int64_t rows = cols > 0 ? x.numel() / cols : 0;
  TORCH_CHECK(rstd.numel() == rows, "[", op, "] rstd needs ", rows, " elements, got ", rstd.numel());
  if (rows == 0) return;
  c10::cuda::CUDAGuard guard(x.device());
  check_status(aotk_rmsnorm_rstd(static_cast<float*>(rstd.data_ptr()), x.data_ptr(), rows, cols,
                                 eps, aotk_dtype(x, op), current_stream(x)),
               op);
}

void add_rmsnorm_forward(at::Tensor out, at::Tensor residual_out, at::Tensor x,
                         at::Tensor residual, at::Tensor weight, double eps) {
  const char* op = "add_rmsnorm";
  check_cuda(x, op, "x");
  check_cuda(residual, op, "residual");
  check_cuda(weight, op, "weight");
  check_same(x, residual, op, "x", "residual");
  check_same(x, weight, op, "x", "weight");
  TORCH_CHECK(x.is_contiguous() && residual.is_contiguous() && weight.is_contiguous(), "[", op,
              "] inputs must be contiguous");
  TORCH_CHECK(x.sizes() == residual.sizes(), "[", op, "] x and residual shapes differ: ", x.sizes(),
              " vs ", residual.sizes());
  TORCH_CHECK(weight.dim() == 1 && x.dim() >= 1 && weight.size(0) == x.size(-1), "[", op,
              "] weight must be [x.size(-1)]");
  check_out_like(out, x, op);
  check_out_like(residual_out, x, op);
  if (x.numel() == 0) return;
  const int64_t cols = x.size(-1);
  const int64_t rows = x.numel() / cols;
  c10::cuda::CUDAGuard guard(x.device());
  check_status(aotk_add_rmsnorm_forward(out.data_ptr(), residual_out.data_ptr(), x.data_ptr(),
                                        residual.data_ptr(), weight.data_ptr(), rows, cols, eps,
                                        aotk_dtype(x, op), current_stream(x)),
               op);
}

struct GemmArgs {
  int64_t M, N, K;
  int dtype;
};

GemmArgs check_gemm(const at::Tensor& out, const at::Tensor& a, const at::Tensor& b,
                    const char* op) {
  check_cuda(a, op, "a");
  check_cuda(b, op, "b");
  check_cuda(out, op, "out");
  check_same(a, b, op, "a", "b");
  check_same(out, a, op, "out", "a");
  TORCH_CHECK(a.dim() == 2 && b.dim() == 2, "[", op, "] expects 2D tensors, got a.dim=", a.dim(),
              " b.dim=", b.dim());
  TORCH_CHECK(a.size(1) == b.size(0), "[", op, "] inner dims mismatch: ", a.size(1), " vs ",
              b.size(0));
  TORCH_CHECK(a.is_contiguous() && b.is_contiguous() && out.is_contiguous(), "[", op,
              "] tensors must be contiguous");
  TORCH_CHECK(out.dim() == 2 && out.size(0) == a.size(0) && out.size(1) == b.size(1), "[", op,
              "] out must be [", a.size(0), ", ", b.size(1), "], got ", out.sizes());
  return GemmArgs{a.size(0), b.size(1), a.size(1), aotk_dtype(a, op)};
}

void gemm(at::Tensor out, at::Tensor a, at::Tensor b) {
  const char* op = "gemm";
  const GemmArgs g = check_gemm(out, a, b, op);
  c10::cuda::CUDAGuard guard(a.device());
  check_status(aotk_gemm(out.data_ptr(), a.data_ptr(), b.data_ptr(), g.M, g.N, g.K, g.dtype,
                         current_stream(a)),
               op);
}

void gemm_opt(at::Tensor out, at::Tensor a, at::Tensor b) {
  const char* op = "gemm_opt";
  const GemmArgs g = check_gemm(out, a, b, op);
  c10::cuda::CUDAGuard guard(a.device());
  size_t ws_bytes = 0;
  check_status(aotk_gemm_opt_workspace_size(g.M, g.N, g.K, g.dtype, &ws_bytes), op);
  // Scratch for the K-split last wave comes from torch's caching allocator
  // (stream-ordered, so reuse by the next call on this stream is safe).
  at::Tensor ws;
  if (ws_bytes > 0)
    ws = at::empty({static_cast<int64_t>(ws_bytes)}, a.options().dtype(at::kByte));
  check_status(aotk_gemm_opt_ws(out.data_ptr(), a.data_ptr(), b.data_ptr(), g.M, g.N, g.K, g.dtype,
                                ws_bytes > 0 ? ws.data_ptr() : nullptr, ws_bytes,
                                current_stream(a)),
               op);
}

void gemm_silu_mul_impl(at::Tensor out, at::Tensor a, at::Tensor b_gate_up,
                        const at::Tensor* row_scale, const char* op) {
  check_cuda(a, op, "a");
  check_cuda(b_gate_up, op, "b_gate_up");
  check_cuda(out, op, "out");
  check_same(a, b_gate_up, op, "a", "b_gate_up");
  check_same(out, a, op, "out", "a");
  TORCH_CHECK(a.dim() == 2 && b_gate_up.dim() == 2 && out.dim() == 2, "[", op, "] expects 2D tensors");
  TORCH_CHECK(a.size(1) == b_gate_up.size(0), "[", op, "] inner dims mismatch: ", a.size(1), " vs ",
              b_gate_up.size(0));
  TORCH_CHECK(b_gate_up.size(1) % 2 == 0 && out.size(0) == a.size(0) &&
                  out.size(1) == b_gate_up.size(1) / 2,
              "[", op, "] out must be [M, N / 2] for b_gate_up [K, N]");
  TORCH_CHECK(a.is_contiguous() && b_gate_up.is_contiguous() && out.is_contiguous(), "[", op,
              "] tensors must be contiguous");
  const int64_t M = a.size(0), K = a.size(1), I = out.size(1);
  const int dtype = aotk_dtype(a, op);
  if (row_scale) {
    TORCH_CHECK(row_scale->scalar_type() == at::kFloat && row_scale->is_contiguous() &&
                    row_scale->device() == a.device() && row_scale->numel() == M,
                "[", op, "] row_scale must be a contiguous float32 [M] tensor on a's device");
  }
  c10::cuda::CUDAGuard guard(a.device());
  size_t ws_bytes = 0;
  check_status(aotk_gemm_silu_mul_workspace_size(M, I, K, dtype, &ws_bytes), op);
  at::Tensor ws;
  if (ws_bytes > 0)
    ws = at::empty({static_cast<int64_t>(ws_bytes)}, a.options().dtype(at::kByte));
  void* wsp = ws_bytes > 0 ? ws.data_ptr() : nullptr;
  if (row_scale) {
    check_status(aotk_gemm_silu_mul_rowscale(out.data_ptr(), a.data_ptr(), b_gate_up.data_ptr(),
                                             static_cast<const float*>(row_scale->data_ptr()), M,
                                             I, K, dtype, wsp, ws_bytes, current_stream(a)),
                 op);
  } else {
    check_status(aotk_gemm_silu_mul(out.data_ptr(), a.data_ptr(), b_gate_up.data_ptr(), M, I, K,
                                    dtype, wsp, ws_bytes, current_stream(a)),
                 op);
  }
}

void gemm_silu_mul(at::Tensor out, at::Tensor a, at::Tensor b_gate_up) {
  gemm_silu_mul_impl(out, a, b_gate_up, nullptr, "gemm_silu_mul");
}

void gemm_silu_mul_rowscale(at::Tensor out, at::Tensor a, at::Tensor b_gate_up,
                            at::Tensor row_scale) {
  gemm_silu_mul_impl(out, a, b_gate_up, &row_scale, "gemm_silu_mul_rowscale");
}

// out = (a @ b) * scale_a * scale_b for 8-bit a / b (e4m3, e5m2 or int8);
// scale_a / scale_b fp32 with 1 value each or M / N values.  `optimized`
// selects the tensor-core dispatch (tcgen05 where the shape allows) or the
// SIMT kernel, as the reference's flag selects its optimized or naive kernel.
void scaled_gemm(at::Tensor out, at::Tensor a, at::Tensor b, at::Tensor scale_a,
                 at::Tensor scale_b, bool optimized) {
  const char* op = "scaled_gemm";
  check_cuda(a, op, "a");
  check_cuda(b, op, "b");
  check_cuda(out, op, "out");
  check_cuda(scale_a, op, "scale_a");
  check_cuda(scale_b, op, "scale_b");
  check_same(a, b, op, "a", "b");
  TORCH_CHECK(out.device() == a.device() && scale_a.device() == a.device() &&
                  scale_b.device() == a.device(),
              "[", op, "] tensors are not on one device");
  int in_dtype = -1;
  switch (a.scalar_type()) {
    case at::ScalarType::Float8_e4m3fn: in_dtype = AOTK_FLOAT8_E4M3; break;
    case at::ScalarType::Float8_e5m2: in_dtype = AOTK_FLOAT8_E5M2; break;
    case at::ScalarType::Char: in_dtype = AOTK_INT8; break;
    default: TORCH_CHECK(false, "[", op, "] unsupported input dtype: ", a.scalar_type());
  }
  const int out_dtype = aotk_dtype(out, op);
  TORCH_CHECK(a.dim() == 2 && b.dim() == 2 && out.dim() == 2, "[", op, "] expects 2D tensors");
  TORCH_CHECK(a.size(1) == b.size(0), "[", op, "] inner dims mismatch: ", a.size(1), " vs ",
              b.size(0));
  const int64_t M = a.size(0), K = a.size(1), N = b.size(1);
  TORCH_CHECK(out.size(0) == M && out.size(1) == N, "[", op, "] out must be [", M, ", ", N,
              "], got ", out.sizes());
  TORCH_CHECK(a.is_contiguous() && b.is_contiguous() && out.is_contiguous(), "[", op,
              "] tensors must be contiguous");
  TORCH_CHECK(scale_a.scalar_type() == at::kFloat && scale_b.scalar_type() == at::kFloat, "[", op,
              "] scales must be float32");
  TORCH_CHECK(scale_a.is_contiguous() && scale_b.is_contiguous(), "[", op,
              "] scales must be contiguous");
  int mode = -1;
  if (scale_a.numel() == 1 && scale_b.numel() == 1)
    mode = AOTK_SCALE_TENSOR;
  else if (scale_a.numel() == M && scale_b.numel() == N)
    mode = AOTK_SCALE_ROW;
  TORCH_CHECK(mode >= 0, "[", op, "] expect tensorwise (scalar scale_a and scale_b) or rowwise ",
              "(scale_a.numel()==M, scale_b.numel()==N), got ", scale_a.numel(), " and ",
              scale_b.numel());
  c10::cuda::CUDAGuard guard(a.device());
  const auto* sa = static_cast<const float*>(scale_a.data_ptr());
  const auto* sb = static_cast<const float*>(scale_b.data_ptr());
  if (!optimized) {
    check_status(aotk_scaled_gemm_simt(out.data_ptr(), a.data_ptr(), b.data_ptr(), sa, sb, M, N,
                                       K, in_dtype, out_dtype, mode, current_stream(a)),
                 op);
    return;
  }
  size_t ws_bytes = 0;
  check_status(aotk_scaled_gemm_workspace_size(M, N, K, in_dtype, &ws_bytes), op);
  at::Tensor ws;
  if (ws_bytes > 0)
    ws = at::empty({static_cast<int64_t>(ws_bytes)}, a.options().dtype(at::kByte));
  check_status(aotk_scaled_gemm(out.data_ptr(), a.data_ptr(), b.data_ptr(), sa, sb, M, N, K,
                                in_dtype, out_dtype, mode, ws_bytes > 0 ? ws.data_ptr() : nullptr,
                                ws_bytes, current_stream(a)),
               op);
}

}  // namespace

TORCH_LIBRARY(aot_kernel, m) {
  m.def("relu_forward(Tensor! out, Tensor x) -> ()");
  m.impl("relu_forward", c10::kCUDA, &relu_forward);

  m.def("silu_forward(Tensor! out, Tensor x) -> ()");
  m.impl("silu_forward", c10::kCUDA, &silu_forward);

  m.def("silu_mul_forward(Tensor! out, Tensor gate, Tensor up) -> ()");
  m.impl("silu_mul_forward", c10::kCUDA, &silu_mul_forward);

  m.def("rmsnorm_forward(Tensor! out, Tensor x, Tensor weight, float eps) -> ()");
  m.impl("rmsnorm_forward", c10::kCUDA, &rmsnorm_forward);

  m.def(
      "add_rmsnorm_forward(Tensor! out, Tensor! residual_out, Tensor x, Tensor residual, Tensor "
      "weight, float eps) -> ()");
  m.impl("add_rmsnorm_forward", c10::kCUDA, &add_rmsnorm_forward);

  m.def("gemm(Tensor! out, Tensor a, Tensor b) -> ()");
  m.impl("gemm", c10::kCUDA, &gemm);

  m.def("gemm_opt(Tensor! out, Tensor a, Tensor b) -> ()");
  m.impl("gemm_opt", c10::kCUDA, &gemm_opt);

  m.def("gemm_silu_mul(Tensor! out, Tensor a, Tensor b_gate_up) -> ()");
  m.impl("gemm_silu_mul", c10::kCUDA, &gemm_silu_mul);

  m.def("rmsnorm_rstd(Tensor! rstd, Tensor x, float eps) -> ()");
  m.impl("rmsnorm_rstd", c10::kCUDA, &rmsnorm_rstd);

  m.def("gemm_silu_mul_rowscale(Tensor! out, Tensor a, Tensor b_gate_up, Tensor row_scale) -> ()");
  m.impl("gemm_silu_mul_rowscale", c10::kCUDA, &gemm_silu_mul_rowscale);

  m.def(
      "scaled_gemm(Tensor! out, Tensor a, Tensor b, Tensor scale_a, Tensor scale_b, bool "
      "optimized) -> ()");
  m.impl("scaled_gemm", c10::kCUDA, &scaled_gemm);
}

// `import aot_kernel._C` runs the static registration above; the module itself is empty.
PyMODINIT_FUNC PyInit__C(void) {
  static struct PyModuleDef module = {PyModuleDef_HEAD_INIT, "_C", nullptr, 0, nullptr};
  return PyModule_Create(&module);
}
