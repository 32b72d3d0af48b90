// torch_binding.cpp — the `my_plugins` Python module: the reference plugin's three functions
// with the same names, argument order, tensor types/shapes and error behaviour (TORCH_CHECK ->
// RuntimeError), implemented on top of the C ABI of libnvfp4_b200.so.
//
//   quantize_nvfp4(input, input_scale)            csrc/quantize/quantize_nvfp4_bindling.cpp:4-20
//   de_quantize_nvfp4(input, input_scale, sf)     csrc/quantize/quantize_nvfp4_bindling.cpp:23-37
//   gemm_nvfp4(A, B, A_sf, B_sf, scale)           csrc/gemm/gemm_nvfp4_bindling.cpp:4-25
//
// Differences, all on the side of the reference's undefined behaviour:
//   * a CUDA scale tensor is passed to the kernels by device pointer: no .item() device->host
//     synchronisation per call (a CPU scale tensor is read on the host, also without a sync);
//   * shapes the reference silently mis-handles or aborts on are rejected with RuntimeError:
//     last dim % 16 (quantize), sf shape mismatches, K mismatch between A and B, K % 256 and
//     N % 8 (the reference assert()s, gemm_nvfp4.cu:246);
//   * sizes are 64-bit.
#include <vector>

#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <pybind11/stl.h>
#include <torch/extension.h>

#include "../../include/nvfp4_b200.h"

namespace {

void check_status(int st, const char* what) {
  TORCH_CHECK(st == NVFP4_OK, what, " failed: ", nvfp4_status_string(st));
}

struct ScaleArg {
  const float* dev = nullptr;
  float host = 0.0f;
};

ScaleArg scale_arg(const torch::Tensor& s, const torch::Device& data_device, const char* name) {
  TORCH_CHECK(s.dtype() == torch::kFloat32 && 0 == s.dim(), name, " must be float32 and scalar");
  ScaleArg a;
  if (s.is_cuda()) {
    TORCH_CHECK(s.device() == data_device, name, " must be on the same device as the data (",
                data_device, "), got ", s.device());
    a.dev = s.data_ptr<float>();
  } else {
    TORCH_CHECK(s.device().is_cpu(), name, " must be a CPU or CUDA tensor");
    a.host = *s.data_ptr<float>();
  }
  return a;
}

std::tuple<torch::Tensor, torch::Tensor> py_quantize_nvfp4(const torch::Tensor& input,
                                                           const torch::Tensor& input_scale) {
  TORCH_CHECK(input.dtype() == torch::kBFloat16 && input.is_contiguous(),
              "input must be bf16 and contiguous");
  TORCH_CHECK(input_scale.dtype() == torch::kFloat32 && 0 == input_scale.dim(),
              "input_scale must be float32 and scalar");
  TORCH_CHECK(input.device().is_cuda(), "input must be on cuda device");
  TORCH_CHECK(input.dim() >= 1 && input.size(-1) % 16 == 0,
              "input's last dimension must be a multiple of 16, got ", input.sizes());
  const c10::cuda::CUDAGuard guard(input.device());
  const ScaleArg sc = scale_arg(input_scale, input.device(), "input_scale");

  auto out_sizes = input.sizes().vec();
  auto sf_sizes = input.sizes().vec();
  out_sizes.back() /= 2;
  sf_sizes.back() /= 16;
  auto output = torch::empty(out_sizes, torch::dtype(torch::kUInt8).device(input.device()));
  auto output_sf = torch::empty(sf_sizes, torch::dtype(torch::kFloat8_e4m3fn).device(input.device()));
  cudaStream_t stream = at::cuda::getCurrentCUDAStream(input.device().index());
  const int st = sc.dev ? nvfp4_quantize(input.data_ptr(), sc.dev, input.numel(), output.data_ptr(),
                                         output_sf.data_ptr(), stream)
                        : nvfp4_quantize_host_scale(input.data_ptr(), sc.host, input.numel(),
                                                    output.data_ptr(), output_sf.data_ptr(), stream);
  check_status(st, "quantize_nvfp4");
  return std::make_tuple(output, output_sf);
}

// Extension (no reference counterpart): quantize with the per-tensor scale computed on the
// device from the input itself, s = 6*448/amax evaluated as torch evaluates the reference recipe.
// Returns (packed, sf, s) with s a 0-dim fp32 tensor on the input's device.
std::tuple<torch::Tensor, torch::Tensor, torch::Tensor> py_quantize_nvfp4_auto_scale(
    const torch::Tensor& input) {
  TORCH_CHECK(input.dtype() == torch::kBFloat16 && input.is_contiguous(),
              "input must be bf16 and contiguous");
  TORCH_CHECK(input.device().is_cuda(), "input must be on cuda device");
  TORCH_CHECK(input.dim() >= 1 && input.size(-1) % 16 == 0,
              "input's last dimension must be a multiple of 16, got ", input.sizes());
  const c10::cuda::CUDAGuard guard(input.device());
  auto out_sizes = input.sizes().vec();
  auto sf_sizes = input.sizes().vec();
  out_sizes.back() /= 2;
  sf_sizes.back() /= 16;
  auto opts = torch::TensorOptions().device(input.device());
  auto output = torch::empty(out_sizes, opts.dtype(torch::kUInt8));
  auto output_sf = torch::empty(sf_sizes, opts.dtype(torch::kFloat8_e4m3fn));
  auto scale = torch::empty({}, opts.dtype(torch::kFloat32));
  const int64_t ws_bytes = nvfp4_quantize_auto_scale_workspace_bytes(input.numel());
  auto ws = torch::empty({ws_bytes}, opts.dtype(torch::kUInt8));
  cudaStream_t stream = at::cuda::getCurrentCUDAStream(input.device().index());
  check_status(nvfp4_quantize_auto_scale(input.data_ptr(), input.numel(), output.data_ptr(),
                                         output_sf.data_ptr(), scale.data_ptr<float>(),
                                         ws.data_ptr(), ws_bytes, stream),
               "quantize_nvfp4_auto_scale");
  return std::make_tuple(output, output_sf, scale);
}

torch::Tensor py_de_quantize_nvfp4(const torch::Tensor& input, const torch::Tensor& input_scale,
                                   const torch::Tensor& input_sf) {
  TORCH_CHECK(input.dtype() == torch::kUInt8 && input.is_contiguous(),
              "input must be uint8 and contiguous");
  TORCH_CHECK(input_scale.dtype() == torch::kFloat32 && 0 == input_scale.dim(),
              "input_scale must be float32 and scalar");
  TORCH_CHECK(input_sf.dtype() == torch::kFloat8_e4m3fn && input_sf.is_contiguous(),
              "input_sf must be float8_e4m3 and contiguous");
  TORCH_CHECK(input.device().is_cuda() && input_sf.device().is_cuda(),
              "input&input_sf must be on cuda device");
  TORCH_CHECK(input_sf.device() == input.device(), "input_sf must be on the input's device");
  TORCH_CHECK(input.dim() >= 1 && input.size(-1) % 8 == 0,
              "input's last dimension must be a multiple of 8 (16 elements per scale), got ",
              input.sizes());
  TORCH_CHECK(input_sf.numel() * 8 == input.numel(), "input_sf has ", input_sf.numel(),
              " scale factors, expected ", input.numel() / 8);
  const c10::cuda::CUDAGuard guard(input.device());
  const ScaleArg sc = scale_arg(input_scale, input.device(), "input_scale");

  auto out_sizes = input.sizes().vec();
  out_sizes.back() *= 2;
  auto output = torch::empty(out_sizes, torch::dtype(torch::kBFloat16).device(input.device()));
  cudaStream_t stream = at::cuda::getCurrentCUDAStream(input.device().index());
  const int st =
      sc.dev ? nvfp4_dequantize(input.data_ptr(), sc.dev, input_sf.data_ptr(), input.numel(),
                                output.data_ptr(), stream)
             : nvfp4_dequantize_host_scale(input.data_ptr(), sc.host, input_sf.data_ptr(),
                                           input.numel(), output.data_ptr(), stream);
  check_status(st, "de_quantize_nvfp4");
  return output;
}

torch::Tensor py_gemm_nvfp4(const torch::Tensor& A, const torch::Tensor& B,
                            const torch::Tensor& A_sf, const torch::Tensor& B_sf,
                            const torch::Tensor& scale) {
  TORCH_CHECK(A.dtype() == torch::kUInt8 && A.is_contiguous(), "A must be uint8 and contiguous");
  TORCH_CHECK(B.dtype() == torch::kUInt8 && B.is_contiguous(), "B must be uint8 and contiguous");
  TORCH_CHECK(2 == A.dim() && 2 == B.dim(), "A and B must be 2D");
  TORCH_CHECK(A_sf.dtype() == torch::kFloat8_e4m3fn && A_sf.is_contiguous(),
              "A_sf must be float8_e4m3 and contiguous");
  TORCH_CHECK(B_sf.dtype() == torch::kFloat8_e4m3fn && B_sf.is_contiguous(),
              "B_sf must be float8_e4m3 and contiguous");
  TORCH_CHECK(scale.dtype() == torch::kFloat32 && 0 == scale.dim(),
              "scale must be float32 and scalar");
  TORCH_CHECK(A.device().is_cuda() && B.device().is_cuda() && A_sf.device().is_cuda() &&
                  B_sf.device().is_cuda(),
              "A&B&A_sf&B_sf must be on cuda device");
  TORCH_CHECK(B.device() == A.device() && A_sf.device() == A.device() &&
                  B_sf.device() == A.device(),
              "A, B, A_sf and B_sf must be on the same device");
  const int64_t M = A.size(0), N = B.size(0), K = A.size(1) * 2;
  TORCH_CHECK(B.size(1) * 2 == K, "A and B must have the same K: A is ", A.sizes(), ", B is ",
              B.sizes());
  TORCH_CHECK(K % 256 == 0, "K must be a multiple of 256, got ", K);
  TORCH_CHECK(N % 8 == 0, "N must be a multiple of 8, got ", N);
  TORCH_CHECK(A_sf.numel() == M * (K / 16) && (A_sf.dim() < 2 || A_sf.size(0) == M),
              "A_sf must hold [M, K/16] = [", M, ", ", K / 16, "] scale factors, got ",
              A_sf.sizes());
  TORCH_CHECK(B_sf.numel() == N * (K / 16) && (B_sf.dim() < 2 || B_sf.size(0) == N),
              "B_sf must hold [N, K/16] = [", N, ", ", K / 16, "] scale factors, got ",
              B_sf.sizes());
  const c10::cuda::CUDAGuard guard(A.device());
  const ScaleArg sc = scale_arg(scale, A.device(), "scale");

  auto D = torch::empty({M, N}, torch::dtype(torch::kBFloat16).device(A.device()));
  cudaStream_t stream = at::cuda::getCurrentCUDAStream(A.device().index());
  const int st = sc.dev ? nvfp4_gemm(A.data_ptr(), B.data_ptr(), A_sf.data_ptr(), B_sf.data_ptr(),
                                     sc.dev, D.data_ptr(), M, N, K, stream)
                        : nvfp4_gemm_host_scale(A.data_ptr(), B.data_ptr(), A_sf.data_ptr(),
                                                B_sf.data_ptr(), sc.host, D.data_ptr(), M, N, K,
                                                stream);
  check_status(st, "gemm_nvfp4");
  return D;
}

// Extension (no reference counterpart): GEMM with the output quantized to NVFP4 in its
// epilogue; the same bytes as quantize_nvfp4(gemm_nvfp4(A, B, A_sf, B_sf, scale), out_scale).
// Both scales must be float32 scalars on the GPU. Returns (uint8 [M, N/2], float8_e4m3fn
// [M, N/16]).
std::tuple<torch::Tensor, torch::Tensor> py_gemm_nvfp4_quantized(
    const torch::Tensor& A, const torch::Tensor& B, const torch::Tensor& A_sf,
    const torch::Tensor& B_sf, const torch::Tensor& scale, const torch::Tensor& out_scale) {
  TORCH_CHECK(A.dtype() == torch::kUInt8 && A.is_contiguous() && A.dim() == 2 &&
                  B.dtype() == torch::kUInt8 && B.is_contiguous() && B.dim() == 2,
              "A and B must be 2D uint8 and contiguous");
  TORCH_CHECK(A_sf.dtype() == torch::kFloat8_e4m3fn && A_sf.is_contiguous() &&
                  B_sf.dtype() == torch::kFloat8_e4m3fn && B_sf.is_contiguous(),
              "A_sf and B_sf must be float8_e4m3 and contiguous");
  for (const torch::Tensor* t : {&scale, &out_scale})
    TORCH_CHECK(t->dtype() == torch::kFloat32 && 0 == t->dim() && t->is_cuda(),
                "scale and out_scale must be float32 scalars on the GPU");
  TORCH_CHECK(A.is_cuda() && B.device() == A.device() && A_sf.device() == A.device() &&
                  B_sf.device() == A.device() && scale.device() == A.device() &&
                  out_scale.device() == A.device(),
              "all tensors must be on the same cuda device");
  const int64_t M = A.size(0), N = B.size(0), K = A.size(1) * 2;
  TORCH_CHECK(B.size(1) * 2 == K, "A and B must have the same K");
  TORCH_CHECK(K % 256 == 0 && K > 0, "K must be a positive multiple of 256, got ", K);
  TORCH_CHECK(N % 32 == 0, "N must be a multiple of 32 for the quantized output, got ", N);
  TORCH_CHECK(A_sf.numel() == M * (K / 16) && B_sf.numel() == N * (K / 16),
              "scale-factor tensors must hold [rows, K/16] factors");
  const c10::cuda::CUDAGuard guard(A.device());
  auto opts = torch::TensorOptions().device(A.device());
  auto q = torch::empty({M, N / 2}, opts.dtype(torch::kUInt8));
  auto sf = torch::empty({M, N / 16}, opts.dtype(torch::kFloat8_e4m3fn));
  cudaStream_t stream = at::cuda::getCurrentCUDAStream(A.device().index());
  check_status(nvfp4_gemm_quantized(A.data_ptr(), B.data_ptr(), A_sf.data_ptr(), B_sf.data_ptr(),
                                    scale.data_ptr<float>(), out_scale.data_ptr<float>(),
                                    q.data_ptr(), sf.data_ptr(), M, N, K, stream),
               "gemm_nvfp4_quantized");
  return std::make_tuple(q, sf);
}

// Extension (no reference counterpart): gate+up GEMM with SwiGLU in the epilogue. B_gate_up is
// [2I, K/2] with rows interleaved in groups of 128 (gate, up, gate, up, ...; see
// my_nvfp4_gemm_b200.swiglu). Returns bf16 [M, I] = bf16(silu(Dg) * Du) in fp32.
torch::Tensor py_gemm_nvfp4_swiglu(const torch::Tensor& A, const torch::Tensor& B_gate_up,
                                   const torch::Tensor& A_sf, const torch::Tensor& B_gate_up_sf,
                                   const torch::Tensor& scale) {
  TORCH_CHECK(A.dtype() == torch::kUInt8 && A.is_contiguous() && A.dim() == 2 &&
                  B_gate_up.dtype() == torch::kUInt8 && B_gate_up.is_contiguous() &&
                  B_gate_up.dim() == 2,
              "A and B_gate_up must be 2D uint8 and contiguous");
  TORCH_CHECK(A_sf.dtype() == torch::kFloat8_e4m3fn && A_sf.is_contiguous() &&
                  B_gate_up_sf.dtype() == torch::kFloat8_e4m3fn && B_gate_up_sf.is_contiguous(),
              "A_sf and B_gate_up_sf must be float8_e4m3 and contiguous");
  TORCH_CHECK(scale.dtype() == torch::kFloat32 && 0 == scale.dim() && scale.is_cuda(),
              "scale must be a float32 scalar on the GPU");
  TORCH_CHECK(A.is_cuda() && B_gate_up.device() == A.device() && A_sf.device() == A.device() &&
                  B_gate_up_sf.device() == A.device() && scale.device() == A.device(),
              "all tensors must be on the same cuda device");
  const int64_t M = A.size(0), N = B_gate_up.size(0), K = A.size(1) * 2;
  TORCH_CHECK(B_gate_up.size(1) * 2 == K, "A and B_gate_up must have the same K");
  TORCH_CHECK(K % 256 == 0 && K > 0, "K must be a positive multiple of 256, got ", K);
  TORCH_CHECK(N % 256 == 0, "B_gate_up must have a multiple of 256 rows (2*I, I % 128 == 0), got ", N);
  TORCH_CHECK(A_sf.numel() == M * (K / 16) && B_gate_up_sf.numel() == N * (K / 16),
              "scale-factor tensors must hold [rows, K/16] factors");
  const c10::cuda::CUDAGuard guard(A.device());
  auto out = torch::empty({M, N / 2}, torch::dtype(torch::kBFloat16).device(A.device()));
  cudaStream_t stream = at::cuda::getCurrentCUDAStream(A.device().index());
  check_status(nvfp4_gemm_swiglu(A.data_ptr(), B_gate_up.data_ptr(), A_sf.data_ptr(),
                                 B_gate_up_sf.data_ptr(), scale.data_ptr<float>(), out.data_ptr(),
                                 M, N, K, stream),
               "gemm_nvfp4_swiglu");
  return out;
}

// Extension (no reference counterpart): the column-parallel GEMM with the all-gather fused into
// its epilogue. `output` is this rank's full D [M, world * N_local] (bf16, contiguous) and
// `output_ptrs[r]` the address, in this process, of rank r's D (output_ptrs[rank] ==
// output.data_ptr(); the others mapped through nvfp4_ipc_open). The caller orders the ranks:
// every rank's call completes before any rank reads D, and no rank reuses the buffers before
// every rank has read the previous result (my_nvfp4_gemm_b200.sharded does both).
void py_gemm_nvfp4_allgather(const torch::Tensor& A, const torch::Tensor& B_shard,
                             const torch::Tensor& A_sf, const torch::Tensor& B_sf_shard,
                             const torch::Tensor& scale, const torch::Tensor& output,
                             const std::vector<int64_t>& output_ptrs, int64_t rank) {
  TORCH_CHECK(A.dtype() == torch::kUInt8 && A.is_contiguous() && A.dim() == 2,
              "A must be 2D uint8 and contiguous");
  TORCH_CHECK(B_shard.dtype() == torch::kUInt8 && B_shard.is_contiguous() && B_shard.dim() == 2,
              "B_shard must be 2D uint8 and contiguous");
  TORCH_CHECK(A_sf.dtype() == torch::kFloat8_e4m3fn && A_sf.is_contiguous() &&
                  B_sf_shard.dtype() == torch::kFloat8_e4m3fn && B_sf_shard.is_contiguous(),
              "A_sf and B_sf_shard must be float8_e4m3 and contiguous");
  TORCH_CHECK(scale.dtype() == torch::kFloat32 && 0 == scale.dim() && scale.is_cuda(),
              "scale must be a float32 scalar on the GPU");
  TORCH_CHECK(A.is_cuda() && B_shard.device() == A.device() && A_sf.device() == A.device() &&
                  B_sf_shard.device() == A.device() && scale.device() == A.device() &&
                  output.device() == A.device(),
              "all tensors must be on the same cuda device");
  const int64_t world = int64_t(output_ptrs.size());
  const int64_t M = A.size(0), N_local = B_shard.size(0), K = A.size(1) * 2;
  TORCH_CHECK(world >= 1 && world <= 8, "1..8 ranks supported, got ", world);
  TORCH_CHECK(rank >= 0 && rank < world, "rank out of range");
  TORCH_CHECK(B_shard.size(1) * 2 == K, "A and B_shard must have the same K");
  TORCH_CHECK(K % 256 == 0 && N_local % 8 == 0, "K % 256 == 0 and N_local % 8 == 0 required");
  TORCH_CHECK(A_sf.numel() == M * (K / 16) && B_sf_shard.numel() == N_local * (K / 16),
              "scale-factor tensors must hold [rows, K/16] factors");
  TORCH_CHECK(output.dtype() == torch::kBFloat16 && output.is_contiguous() && output.dim() == 2 &&
                  output.size(0) == M && output.size(1) == world * N_local,
              "output must be bf16 [M, world * N_local] and contiguous");
  TORCH_CHECK(output_ptrs[rank] == reinterpret_cast<int64_t>(output.data_ptr()),
              "output_ptrs[rank] must be output's own address");
  const c10::cuda::CUDAGuard guard(A.device());
  std::vector<void*> ptrs(world);
  for (int64_t r = 0; r < world; ++r) ptrs[r] = reinterpret_cast<void*>(output_ptrs[r]);
  cudaStream_t stream = at::cuda::getCurrentCUDAStream(A.device().index());
  check_status(nvfp4_gemm_allgather(A.data_ptr(), B_shard.data_ptr(), A_sf.data_ptr(),
                                    B_sf_shard.data_ptr(), scale.data_ptr<float>(), ptrs.data(),
                                    int(world), int(rank), M, N_local, K, stream),
               "gemm_nvfp4_allgather");
}

// Device status word of the library on the current CUDA device (synchronises the stream).
int64_t py_device_status() {
  int v = 0;
  cudaStream_t stream = at::cuda::getCurrentCUDAStream();
  check_status(nvfp4_device_status(&v, stream), "device_status");
  return v;
}

// Extension (no reference counterpart): scale factors in the 128x4 blocked layout that library
// block-scaled GEMMs consume. `sf` [..., cols] (float8_e4m3fn or uint8, contiguous, CUDA); all
// leading dimensions are rows. Returns a 1-D float8_e4m3fn tensor of
// round_up(rows, 128) * round_up(cols, 4) bytes.
torch::Tensor py_swizzle_scale_factors(const torch::Tensor& sf) {
  TORCH_CHECK((sf.dtype() == torch::kFloat8_e4m3fn || sf.dtype() == torch::kUInt8) &&
                  sf.is_contiguous(),
              "sf must be float8_e4m3fn (or uint8) and contiguous");
  TORCH_CHECK(sf.device().is_cuda(), "sf must be on cuda device");
  TORCH_CHECK(sf.dim() >= 1, "sf must have at least one dimension");
  const c10::cuda::CUDAGuard guard(sf.device());
  const int64_t cols = sf.size(-1);
  const int64_t rows = cols == 0 ? 0 : sf.numel() / cols;
  const int64_t bytes = nvfp4_blocked_scale_bytes(rows, cols);
  auto out = torch::empty({bytes}, torch::dtype(torch::kFloat8_e4m3fn).device(sf.device()));
  cudaStream_t stream = at::cuda::getCurrentCUDAStream(sf.device().index());
  check_status(nvfp4_scale_to_blocked(sf.data_ptr(), rows, cols, out.data_ptr(), stream),
               "swizzle_scale_factors");
  return out;
}

// Inverse of swizzle_scale_factors: blocked (1-D, CUDA) -> float8_e4m3fn [rows, cols].
torch::Tensor py_unswizzle_scale_factors(const torch::Tensor& blocked, int64_t rows, int64_t cols) {
  TORCH_CHECK((blocked.dtype() == torch::kFloat8_e4m3fn || blocked.dtype() == torch::kUInt8) &&
                  blocked.is_contiguous(),
              "blocked must be float8_e4m3fn (or uint8) and contiguous");
  TORCH_CHECK(blocked.device().is_cuda(), "blocked must be on cuda device");
  TORCH_CHECK(rows >= 0 && cols >= 0, "rows and cols must be non-negative");
  TORCH_CHECK(blocked.numel() == nvfp4_blocked_scale_bytes(rows, cols),
              "blocked holds ", blocked.numel(), " bytes, expected ",
              nvfp4_blocked_scale_bytes(rows, cols), " for ", rows, " x ", cols);
  const c10::cuda::CUDAGuard guard(blocked.device());
  auto out = torch::empty({rows, cols}, torch::dtype(torch::kFloat8_e4m3fn).device(blocked.device()));
  cudaStream_t stream = at::cuda::getCurrentCUDAStream(blocked.device().index());
  check_status(nvfp4_scale_from_blocked(blocked.data_ptr(), rows, cols, out.data_ptr(), stream),
               "unswizzle_scale_factors");
  return out;
}

void py_clear_device_status() {
  cudaStream_t stream = at::cuda::getCurrentCUDAStream();
  check_status(nvfp4_clear_device_status(stream), "clear_device_status");
}

}  // namespace

PYBIND11_MODULE(my_plugins, m) {
  m.doc() = "my_plugins: NVFP4 quantize / dequantize / GEMM for B200 (sm_100a)";
  m.def("quantize_nvfp4", &py_quantize_nvfp4, "quantize_nvfp4", py::arg("input"),
        py::arg("input_scale"));
  m.def("de_quantize_nvfp4", &py_de_quantize_nvfp4, "de_quantize_nvfp4", py::arg("input"),
        py::arg("input_scale"), py::arg("input_sf"));
  m.def("gemm_nvfp4", &py_gemm_nvfp4, "gemm_nvfp4", py::arg("A"), py::arg("B"), py::arg("A_sf"),
        py::arg("B_sf"), py::arg("scale"));
  m.def("quantize_nvfp4_auto_scale", &py_quantize_nvfp4_auto_scale,
        "quantize with s = 6*448/amax computed on the device; returns (packed, sf, s)",
        py::arg("input"));
  m.def("gemm_nvfp4_quantized", &py_gemm_nvfp4_quantized,
        "GEMM with the output quantized to NVFP4 in the epilogue; returns (packed, sf)",
        py::arg("A"), py::arg("B"), py::arg("A_sf"), py::arg("B_sf"), py::arg("scale"),
        py::arg("out_scale"));
  m.def("gemm_nvfp4_swiglu", &py_gemm_nvfp4_swiglu,
        "gate+up GEMM with SwiGLU in the epilogue; B_gate_up rows interleaved in groups of 128",
        py::arg("A"), py::arg("B_gate_up"), py::arg("A_sf"), py::arg("B_gate_up_sf"),
        py::arg("scale"));
  m.def("gemm_nvfp4_allgather", &py_gemm_nvfp4_allgather,
        "column-parallel GEMM storing this rank's columns into every rank's output",
        py::arg("A"), py::arg("B_shard"), py::arg("A_sf"), py::arg("B_sf_shard"), py::arg("scale"),
        py::arg("output"), py::arg("output_ptrs"), py::arg("rank"));
  m.def("swizzle_scale_factors", &py_swizzle_scale_factors,
        "scale factors [..., cols] -> the 128x4 blocked layout of library block-scaled GEMMs",
        py::arg("sf"));
  m.def("unswizzle_scale_factors", &py_unswizzle_scale_factors,
        "blocked scale factors -> float8_e4m3fn [rows, cols]", py::arg("blocked"), py::arg("rows"),
        py::arg("cols"));
  m.def("device_status", &py_device_status,
        "status word of the library's kernels on the current device (0 = OK)");
  m.def("clear_device_status", &py_clear_device_status, "reset the device status word to 0");
}
