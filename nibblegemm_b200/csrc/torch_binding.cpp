// Compiled torch binding over the C ABI: the reference extension's three ops
// (gemv_w4a16, gemm_w4a16, dequant_w4; arvindcr4/nibblegemm csrc/bindings.cpp)
// taking tensors, with the argument checks, the output allocation, the device
// guard, the current-stream lookup and the per-stream workspace cache done in
// C++ -- a few microseconds per call instead of the tens a Python + ctypes path
// costs.  The kernels are the ones of libnibblegemm_b200.so; this file only
// marshals.  Argument-check failures raise RuntimeError (TORCH_CHECK), as the
// reference's do; the library's own status is returned beside the output and
// the Python wrapper raises on a non-zero one.
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#include <mutex>
#include <optional>
#include <tuple>
#include <unordered_map>

#include "nibblegemm_b200.h"

namespace {

int dtype_code(const torch::Tensor& t) {
  if (t.scalar_type() == torch::kHalf) return NG_DTYPE_F16;
  if (t.scalar_type() == torch::kBFloat16) return NG_DTYPE_BF16;
  TORCH_CHECK(false, "activations must be fp16 or bf16");
}

void check_weight(const torch::Tensor& Wq, const torch::Tensor& S, const torch::Device& dev) {
  TORCH_CHECK(Wq.is_cuda() && S.is_cuda(), "all tensors must live on CUDA");
  TORCH_CHECK(Wq.device() == dev && S.device() == dev, "all tensors must be on the same device");
  TORCH_CHECK(Wq.scalar_type() == torch::kInt, "packed weights must be int32");
  TORCH_CHECK(S.scalar_type() == torch::kHalf, "scales must be fp16");
  TORCH_CHECK(Wq.is_contiguous() && S.is_contiguous(), "inputs must be contiguous");
  TORCH_CHECK(Wq.dim() == 2 && S.dim() == 2, "expected 2-D inputs");
}

std::tuple<int64_t, int64_t, int64_t> check_act(const torch::Tensor& X, const torch::Tensor& Wq,
                                                const torch::Tensor& S, int64_t group_size) {
  TORCH_CHECK(X.is_cuda(), "all tensors must live on CUDA");
  check_weight(Wq, S, X.device());
  dtype_code(X);
  TORCH_CHECK(X.is_contiguous(), "inputs must be contiguous");
  TORCH_CHECK(X.dim() == 2, "expected 2-D inputs");
  const int64_t M = X.size(0), K = X.size(1), N = Wq.size(1);
  TORCH_CHECK(Wq.size(0) * 8 == K, "packed weight rows disagree with K");
  TORCH_CHECK(group_size > 0 && S.size(0) * group_size == K, "scale rows disagree with K/group_size");
  TORCH_CHECK(S.size(1) == N, "scale columns disagree with N");
  return {M, K, N};
}

torch::Tensor output(const std::optional<torch::Tensor>& out, int64_t M, int64_t N,
                     const torch::Tensor& X) {
  if (!out.has_value()) return torch::empty({M, N}, X.options());
  const auto& o = *out;
  TORCH_CHECK(o.dim() == 2 && o.size(0) == M && o.size(1) == N && o.scalar_type() == X.scalar_type() &&
                  o.device() == X.device() && o.is_contiguous(),
              "out must be a contiguous [M, N] tensor like X");
  return o;
}

// Zero-filled workspace per (device, stream, kind), grown on demand.  Every
// call leaves its counters at zero, so the buffer is reused as is; one per
// stream because calls sharing a workspace must not overlap on the GPU.
torch::Tensor workspace(const torch::Device& dev, cudaStream_t stream, int kind, size_t need) {
  // Heap-held and never destroyed: a static map of tensors would be torn down at
  // process exit after torch's CUDA allocator, and crash there.
  static std::mutex mu;
  static auto* cache = new std::unordered_map<uint64_t, torch::Tensor>();
  const uint64_t key = (reinterpret_cast<uint64_t>(stream) << 8) ^ (static_cast<uint64_t>(dev.index()) << 2) ^
                       static_cast<uint64_t>(kind);
  std::lock_guard<std::mutex> lock(mu);
  auto it = cache->find(key);
  if (it != cache->end() && static_cast<size_t>(it->second.numel()) >= need) return it->second;
  const int64_t bytes = static_cast<int64_t>(std::max<size_t>(need, kind == 0 ? (4u << 20) : (1u << 20)));
  auto ws = torch::zeros({bytes}, torch::TensorOptions().dtype(torch::kUInt8).device(dev));
  (*cache)[key] = ws;
  return ws;
}

std::tuple<torch::Tensor, int64_t> gemv_w4a16(torch::Tensor X, torch::Tensor Wq, torch::Tensor S, int64_t group_size,
                         int64_t version, int64_t splits_override, int64_t threads_override,
                         int64_t algo, std::optional<torch::Tensor> out) {
  auto [M, K, N] = check_act(X, Wq, S, group_size);
  TORCH_CHECK(N % 4 == 0, "N must be a multiple of 4 for 128-bit weight loads");
  TORCH_CHECK(group_size == 64 || group_size == 128 || group_size == 256,
              "group_size must be 64, 128 or 256");
  TORCH_CHECK(M >= 1 && M <= 16, "gemv path supports 1 <= M <= 16; use gemm_w4a16 for larger M");
  TORCH_CHECK(version >= 0 && version <= 4, "version must be one of 0..4");
  // Version 3 of the reference ladder is version 4 pinned to one K split.
  const int splits = version == 3 ? 1 : static_cast<int>(splits_override);
  const c10::cuda::CUDAGuard guard(X.device());
  auto Y = output(out, M, N, X);
  cudaStream_t stream = at::cuda::getCurrentCUDAStream(X.device().index()).stream();
  auto ws = workspace(X.device(), stream, 0, ng_gemv_workspace_bytes(1, static_cast<int>(N)));
  const int st = ng_gemv_w4a16(X.data_ptr(), dtype_code(X), Wq.data_ptr<int32_t>(),
                             reinterpret_cast<const uint16_t*>(S.data_ptr()), Y.data_ptr(),
                             static_cast<int>(M), static_cast<int>(K), static_cast<int>(N),
                             static_cast<int>(group_size), splits, static_cast<int>(threads_override),
                             static_cast<int>(algo), ws.data_ptr(), static_cast<size_t>(ws.numel()), stream);
  return {Y, st};
}

std::tuple<torch::Tensor, int64_t> gemm_w4a16(torch::Tensor X, torch::Tensor Wq, torch::Tensor S, int64_t group_size,
                         int64_t version, int64_t tile_tokens, std::optional<torch::Tensor> out) {
  auto [M, K, N] = check_act(X, Wq, S, group_size);
  TORCH_CHECK(version == 6 || version == 7, "version must be 6 or 7");
  const c10::cuda::CUDAGuard guard(X.device());
  auto Y = output(out, M, N, X);
  cudaStream_t stream = at::cuda::getCurrentCUDAStream(X.device().index()).stream();
  auto ws = workspace(X.device(), stream, 1, ng_gemm_workspace_bytes(static_cast<int>(M), static_cast<int>(N)));
  const int st = ng_gemm_w4a16(X.data_ptr(), dtype_code(X), Wq.data_ptr<int32_t>(),
                             reinterpret_cast<const uint16_t*>(S.data_ptr()), Y.data_ptr(),
                             static_cast<int>(M), static_cast<int>(K), static_cast<int>(N),
                             static_cast<int>(group_size), static_cast<int>(tile_tokens), ws.data_ptr(),
                             static_cast<size_t>(ws.numel()), stream);
  return {Y, st};
}

std::tuple<torch::Tensor, int64_t> dequant_w4(torch::Tensor Wq, torch::Tensor S, int64_t group_size, bool fast,
                         std::optional<torch::ScalarType> out_dtype) {
  check_weight(Wq, S, Wq.device());
  const int64_t K = Wq.size(0) * 8, N = Wq.size(1);
  TORCH_CHECK(S.size(1) == N, "scale columns disagree with N");
  TORCH_CHECK(group_size > 0 && S.size(0) * group_size == K, "scale rows disagree with K/group_size");
  const auto dt = out_dtype.value_or(torch::kHalf);
  TORCH_CHECK(dt == torch::kHalf || dt == torch::kBFloat16, "out_dtype must be fp16 or bf16");
  const c10::cuda::CUDAGuard guard(Wq.device());
  auto out = torch::empty({K, N}, Wq.options().dtype(dt));
  cudaStream_t stream = at::cuda::getCurrentCUDAStream(Wq.device().index()).stream();
  const int st = ng_dequant_w4(Wq.data_ptr<int32_t>(), reinterpret_cast<const uint16_t*>(S.data_ptr()),
                             out.data_ptr(), dt == torch::kHalf ? NG_DTYPE_F16 : NG_DTYPE_BF16,
                             static_cast<int>(K), static_cast<int>(N), static_cast<int>(group_size),
                             fast ? 1 : 0, stream);
  return {out, st};
}

// The cached workspace a call on (device, stream) uses (for inspection).
torch::Tensor workspace_for(int64_t device_index, int64_t stream, int64_t kind, int64_t need) {
  return workspace(torch::Device(torch::kCUDA, static_cast<c10::DeviceIndex>(device_index)),
                   reinterpret_cast<cudaStream_t>(stream), static_cast<int>(kind), static_cast<size_t>(need));
}

}  // namespace

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  m.def("gemv_w4a16", &gemv_w4a16, "Decode-regime W4A16 GEMV (M <= 16).", py::arg("X"), py::arg("Wq"),
        py::arg("S"), py::arg("group_size"), py::arg("version") = 4, py::arg("splits_override") = 0,
        py::arg("threads_override") = 0, py::arg("algo") = 0, py::arg("out") = py::none());
  m.def("gemm_w4a16", &gemm_w4a16, "Prefill-regime W4A16 GEMM (tcgen05).", py::arg("X"), py::arg("Wq"),
        py::arg("S"), py::arg("group_size"), py::arg("version") = 6, py::arg("tile_tokens") = 0,
        py::arg("out") = py::none());
  m.def("workspace", &workspace_for, "The zero-initialised workspace of (device, stream); kind 0 = GEMV, 1 = GEMM.",
        py::arg("device_index"), py::arg("stream"), py::arg("kind"), py::arg("need"));
  m.def("dequant_w4", &dequant_w4, "Packed INT4 to dense fp16 / bf16.", py::arg("Wq"), py::arg("S"),
        py::arg("group_size"), py::arg("fast") = true, py::arg("out_dtype") = py::none());
}
