// ref_shim.cu — TEST INFRASTRUCTURE ONLY (the checker).
//
// Exposes the reference plugin's own quantize/dequantize launchers, compiled from the
// reference sources for sm_100a (see oracle/Makefile, target `ref`), through a C ABI so the
// tests can run the reference kernels on a B200 and pin the CPU oracle bit-for-bit.
// The declarations restate the reference launcher prototypes of
// csrc/quantize/quantize_nvfp4.h:6-7 (an interface that must match to link).
#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <cuda_fp8.h>
#include <cstdint>

namespace my_plugins {
void quantize_nvfp4(const __nv_bfloat162 *input, const float input_scale, const int input_numel,
                    uint8_t *output, __nv_fp8_e4m3 *output_sf, cudaStream_t stream);
void de_quantize_nvfp4(const uint8_t *input, const float input_scale,
                       const __nv_fp8_e4m3 *input_sf, const int input_numel,
                       __nv_bfloat162 *output, cudaStream_t stream);
}  // namespace my_plugins

extern "C" {
// n_bf16: number of bf16 elements (the reference takes the bf162 pair count).
int ref_quantize_nvfp4(const void *input, float input_scale, int64_t n_bf16, void *output,
                       void *output_sf, cudaStream_t stream) {
  my_plugins::quantize_nvfp4((const __nv_bfloat162 *)input, input_scale, (int)(n_bf16 / 2),
                             (uint8_t *)output, (__nv_fp8_e4m3 *)output_sf, stream);
  return (int)cudaGetLastError();
}
// n_bytes: packed byte count, as the reference takes it.
int ref_de_quantize_nvfp4(const void *input, float input_scale, const void *input_sf,
                          int64_t n_bytes, void *output, cudaStream_t stream) {
  my_plugins::de_quantize_nvfp4((const uint8_t *)input, input_scale,
                                (const __nv_fp8_e4m3 *)input_sf, (int)n_bytes,
                                (__nv_bfloat162 *)output, stream);
  return (int)cudaGetLastError();
}
}
