// qf_torch_ops.cpp -- the thin PyTorch operator over the C ABI of libqf_b200 (include/qf_b200.h).
//
// torch.ops.qf_b200.int8_linear(x, w_q, w_s, bias) is the body of the reference plugin's qf_int8_linear custom op
// (plugin/qwen_fastpath/patches.py:84-101) for bf16 activations on a K-major int8 weight: leading dimensions
// flattened to rows, M <= 16 rows on the small-M W8A16 kernel (bias fused with the reference's two roundings), more
// rows on the tcgen05 W8A8 prefill kernel (the reference's vLLM fallback arithmetic), output in x's shape with N
// columns.  It exists so that an eager call costs one dispatcher hop and the argument checks of the C ABI, instead
// of Python-level checks and a ctypes call.  Workspaces come from the PyTorch caching allocator, one per
// (device, stream) and kind, zero-filled when allocated (the kernels leave their counters at zero).  The caller
// decides eligibility (bf16 activations, a weight the tensor maps can take); anything else raises.
#include <ATen/ATen.h>
#include <c10/cuda/CUDAGuard.h>
#include <c10/cuda/CUDAStream.h>
#include <torch/library.h>

#include <cstdint>
#include <map>
#include <mutex>
#include <tuple>

#include "../../include/qf_b200.h"

namespace {

std::mutex g_ws_mu;
std::map<std::tuple<int, uintptr_t, int>, at::Tensor> g_ws;  // (device, stream, kind) -> workspace

at::Tensor workspace(const at::Device& dev, cudaStream_t stream, int kind, size_t nbytes) {
  std::lock_guard<std::mutex> lk(g_ws_mu);
  auto key = std::make_tuple(static_cast<int>(dev.index()), reinterpret_cast<uintptr_t>(stream), kind);
  auto it = g_ws.find(key);
  if (it == g_ws.end() || static_cast<size_t>(it->second.numel()) < nbytes) {
    const int64_t n = static_cast<int64_t>(nbytes < (8u << 20) ? (8u << 20) : nbytes);
    at::Tensor t = at::zeros({n}, at::TensorOptions().dtype(at::kByte).device(dev));
    g_ws[key] = t;
    return t;
  }
  return it->second;
}

void check(int rc, const char* fn) {
  TORCH_CHECK(rc == QF_OK, fn, ": ", qf_strerror(rc), " (", rc, "): ", qf_last_error_detail());
}

at::Tensor int8_linear(const at::Tensor& x, const at::Tensor& w_q, const at::Tensor& w_s,
                       const c10::optional<at::Tensor>& bias) {
  TORCH_CHECK(x.is_cuda() && w_q.is_cuda() && w_s.is_cuda(), "qf_b200.int8_linear needs CUDA tensors");
  TORCH_CHECK(x.scalar_type() == at::kBFloat16, "activations must be bf16");
  TORCH_CHECK(w_q.scalar_type() == at::kChar && w_q.dim() == 2 && w_q.stride(0) == 1,
              "w_q must be int8 [K, N] with stride (1, ldw)");
  TORCH_CHECK(w_s.scalar_type() == at::kFloat, "w_s must be fp32");
  const int64_t K = x.size(-1);
  const int64_t N = w_q.size(1);
  TORCH_CHECK(w_q.size(0) == K, "w_q rows must match the activations' last dimension");
  TORCH_CHECK(w_s.numel() == N, "w_s must hold N per-channel scales");
  c10::cuda::CUDAGuard guard(x.device());
  at::Tensor x2 = x.reshape({-1, K});
  const int64_t M = x2.size(0);
  std::vector<int64_t> out_shape(x.sizes().begin(), x.sizes().end());
  out_shape.back() = N;
  at::Tensor y = at::empty({M, N}, x.options());
  if (M == 0 || N == 0) return y.view(out_shape);
  if (x2.stride(-1) != 1) x2 = x2.contiguous();
  const at::Tensor scale = w_s.reshape({-1}).contiguous();
  at::Tensor b;
  if (bias.has_value() && bias->defined()) {
    TORCH_CHECK(bias->scalar_type() == at::kBFloat16 && bias->numel() == N, "bias must be bf16 [N]");
    b = bias->reshape({-1}).contiguous();
  }
  const int64_t ldw = N > 1 ? w_q.stride(1) : (K + 15) / 16 * 16;
  cudaStream_t stream = c10::cuda::getCurrentCUDAStream(x.device().index()).stream();
  int rc;
  if (M <= QF_MAX_M) {
    if (reinterpret_cast<uintptr_t>(x2.data_ptr()) % 16 || (M > 1 && x2.stride(0) % 8))
      x2 = x2.clone(at::MemoryFormat::Contiguous);
    at::Tensor ws = workspace(x.device(), stream, 0,
                              qf_w8a16_workspace_bytes(static_cast<int>(M), static_cast<int>(N), static_cast<int>(K)));
    rc = qf_w8a16_gemm(x2.data_ptr(), x2.stride(0), static_cast<const int8_t*>(w_q.data_ptr()), ldw,
                       scale.data_ptr<float>(), b.defined() ? b.data_ptr() : nullptr, y.data_ptr(), N, QF_DTYPE_BF16,
                       static_cast<int>(M), static_cast<int>(N), static_cast<int>(K), ws.data_ptr(),
                       static_cast<size_t>(ws.numel()), QF_FLAG_PDL, stream);
    check(rc, "qf_w8a16_gemm");
  } else {
    at::Tensor ws = workspace(x.device(), stream, 1, qf_w8a8_workspace_bytes(static_cast<int>(M), static_cast<int>(K)));
    rc = qf_w8a8_gemm(x2.data_ptr(), x2.stride(0), static_cast<const int8_t*>(w_q.data_ptr()), ldw,
                      scale.data_ptr<float>(), b.defined() ? b.data_ptr() : nullptr, y.data_ptr(), N,
                      static_cast<int>(M), static_cast<int>(N), static_cast<int>(K), ws.data_ptr(),
                      static_cast<size_t>(ws.numel()), QF_FLAG_PDL, stream);
    check(rc, "qf_w8a8_gemm");
  }
  return y.view(out_shape);
}

at::Tensor int8_linear_meta(const at::Tensor& x, const at::Tensor& w_q, const at::Tensor& w_s,
                            const c10::optional<at::Tensor>& bias) {
  std::vector<int64_t> out_shape(x.sizes().begin(), x.sizes().end());
  out_shape.back() = w_q.size(1);
  return at::empty(out_shape, x.options());
}

}  // namespace

TORCH_LIBRARY(qf_b200, m) {
  m.def("int8_linear(Tensor x, Tensor w_q, Tensor w_s, Tensor? bias) -> Tensor");
}
TORCH_LIBRARY_IMPL(qf_b200, CUDA, m) { m.impl("int8_linear", int8_linear); }
TORCH_LIBRARY_IMPL(qf_b200, Meta, m) { m.impl("int8_linear", int8_linear_meta); }
