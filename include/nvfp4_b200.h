/*
 * nvfp4_b200.h — C ABI of the B200 (sm_100a) NVFP4 quantize / dequantize / GEMM library.
 *
 * Packed format (unchanged from the reference plugin):
 *   - two E2M1 codes per byte, the element with the even index in the low nibble;
 *   - one UE4M3 scale factor per 16 consecutive elements along the last (K) dimension,
 *     stored row-major as [rows, K/16];
 *   - one fp32 per-tensor scale `s = 6*448/amax` (the reciprocal of the usual
 *     "global scale"), exactly as the reference's test recipe builds it.
 *
 * Every entry point:
 *   - takes plain device pointers, 64-bit sizes and a cudaStream_t; the caller owns all buffers;
 *   - is asynchronous on `stream` and allocates nothing;
 *   - returns NVFP4_OK or an nvfp4_status_t error code and never exits the process;
 *   - must be called with the device that owns the buffers current (like cuBLAS).
 *
 * Scales come in two forms, mirroring the reference's by-value float while removing its
 * per-call device->host synchronisation:
 *   - `const float* scale`  : a device pointer to one fp32 value (read by the kernel);
 *   - `*_host_scale` variant : the fp32 value itself, as the reference launchers take it.
 */
#ifndef NVFP4_B200_H_
#define NVFP4_B200_H_

#include <stdint.h>
#include <cuda_runtime.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef enum nvfp4_status_t {
  NVFP4_OK = 0,
  NVFP4_ERR_INVALID_VALUE = 1,     /* null pointer, negative size, bad argument */
  NVFP4_ERR_UNSUPPORTED_SHAPE = 2, /* e.g. K % 256 != 0, N % 8 != 0, numel % 16 != 0 */
  NVFP4_ERR_MISALIGNED = 3,        /* a pointer lacks the alignment its kernel needs */
  NVFP4_ERR_CUDA = 4,              /* a CUDA runtime call or kernel launch failed */
  NVFP4_ERR_NO_DEVICE = 5,         /* no sm_100 device current, or driver entry point missing */
  NVFP4_ERR_DEVICE_TIMEOUT = 6,    /* a bounded device-side wait gave up (see nvfp4_device_status) */
  NVFP4_ERR_TOO_LARGE = 7          /* a size exceeds what the kernel addresses */
} nvfp4_status_t;

/* Human-readable name of a status code (static storage, never NULL). */
const char* nvfp4_status_string(int status);

/* Library version, e.g. 0x000100 for 0.1.0. */
int nvfp4_version(void);

/*
 * Quantize bf16 -> NVFP4 (packed E2M1 + UE4M3 per 16 elements).
 * Replaces my_plugins::quantize_nvfp4 (csrc/quantize/quantize_nvfp4.h:6, launcher
 * csrc/quantize/quantize_nvfp4.cu:37-41). The reference passes the bf162 pair count as
 * `int`; here `numel` is the number of bf16 elements (= 2 x the reference's count), int64.
 *   input      : bf16[numel], 16-byte aligned, treated as a flat array of 16-element blocks
 *   input_scale: device pointer to fp32 s (= 6*448/amax)
 *   output     : uint8[numel/2], 4-byte aligned
 *   output_sf  : e4m3[numel/16]
 * Requires numel % 16 == 0. numel == 0 is a no-op.
 */
int nvfp4_quantize(const void* input, const float* input_scale, int64_t numel,
                   void* output, void* output_sf, cudaStream_t stream);
/* Same, with the scale passed by value (the reference launcher's form). */
int nvfp4_quantize_host_scale(const void* input, float input_scale, int64_t numel,
                              void* output, void* output_sf, cudaStream_t stream);

/*
 * Quantize with the per-tensor scale computed on the device, in one call and with no host
 * synchronisation: amax = NaN-propagating max |x|, s = fp32(1/amax) * 2688 — exactly how torch
 * evaluates the reference recipe `6*448 / A.abs().max().float()` (test.py:10-11) — then the
 * quantization of nvfp4_quantize with that s. *scale_out (device fp32) receives s.
 * `workspace` is a device buffer of at least nvfp4_quantize_auto_scale_workspace_bytes(numel)
 * bytes (4-byte aligned) that the call uses for partial maxima; its contents on entry do not
 * matter. Same input/output rules as nvfp4_quantize. No reference counterpart (the reference
 * computes the scale in torch and synchronises the host with .item()).
 */
int64_t nvfp4_quantize_auto_scale_workspace_bytes(int64_t numel);
int nvfp4_quantize_auto_scale(const void* input, int64_t numel, void* output, void* output_sf,
                              float* scale_out, void* workspace, int64_t workspace_bytes,
                              cudaStream_t stream);

/*
 * Allocation-free form of nvfp4_quantize_auto_scale, for callers that cannot allocate device
 * memory (a plugin inside another runtime's enqueue where allocation is forbidden, a process
 * whose device memory belongs to a pool it does not control, code with a fixed memory budget).
 * No counterpart in the reference. It allocates nothing: its scratch (partial maxima) is a fixed
 * 32 KiB device array inside this library, present on every GPU that loads it until the process
 * exits. Inputs are limited to numel <= 2^30 elements; larger calls return NVFP4_ERR_TOO_LARGE
 * before doing anything. Every call looks up the array's device address on the current device
 * (so a cudaDeviceReset in between is harmless); the first lookup on a device may load the
 * library's device code there, so make that first call outside any stream capture. All calls on a device share
 * the array: calls that overlap on the GPU (e.g. on two streams at once) race and must be
 * ordered by the caller. Results are identical to nvfp4_quantize_auto_scale.
 */
int nvfp4_quantize_auto_scale_noalloc(const void* input, int64_t numel, void* output,
                                      void* output_sf, float* scale_out, cudaStream_t stream);

/*
 * Dequantize NVFP4 -> bf16.
 * Replaces my_plugins::de_quantize_nvfp4 (csrc/quantize/quantize_nvfp4.h:7, launcher
 * csrc/quantize/quantize_nvfp4.cu:64-68). `n_bytes` is the packed byte count, as in the
 * reference (input.numel() of the uint8 tensor), widened to int64.
 *   input      : uint8[n_bytes], 4-byte aligned
 *   input_scale: device pointer to fp32 s
 *   input_sf   : e4m3[n_bytes/8]
 *   output     : bf16[2*n_bytes], 16-byte aligned
 * Requires n_bytes % 8 == 0.
 */
int nvfp4_dequantize(const void* input, const float* input_scale, const void* input_sf,
                     int64_t n_bytes, void* output, cudaStream_t stream);
int nvfp4_dequantize_host_scale(const void* input, float input_scale, const void* input_sf,
                                int64_t n_bytes, void* output, cudaStream_t stream);

/*
 * Block-scaled NVFP4 GEMM, "TN": D[m,n] = bf16( sum_k a[m,k]*sfa[m,k/16]*b[n,k]*sfb[n,k/16] / scale ).
 * Replaces my_plugins::gemm_nvfp4 (csrc/gemm/gemm_nvfp4.h:44-47, launcher
 * csrc/gemm/gemm_nvfp4.cu:242-252). Sizes are int64 instead of int; failures return a status
 * instead of assert()/exit().
 *   A    : uint8[M, K/2]  packed E2M1, K-major
 *   B    : uint8[N, K/2]  packed E2M1, K-major
 *   A_sf : e4m3[M, K/16]  row-major
 *   B_sf : e4m3[N, K/16]  row-major
 *   scale: device pointer to fp32 (the product s_A*s_B of the two tensors' scales)
 *   D    : bf16[M, N] row-major
 * Requires K % 256 == 0 and N % 8 == 0 (the reference's preconditions); any M >= 0.
 * All pointers must be 16-byte aligned (TMA).
 */
int nvfp4_gemm(const void* A, const void* B, const void* A_sf, const void* B_sf,
               const float* scale, void* D, int64_t M, int64_t N, int64_t K,
               cudaStream_t stream);
int nvfp4_gemm_host_scale(const void* A, const void* B, const void* A_sf, const void* B_sf,
                          float scale, void* D, int64_t M, int64_t N, int64_t K,
                          cudaStream_t stream);

/*
 * The kernel form nvfp4_gemm runs for an M x N x K problem on a device with `sms` SMs (0: the
 * current device): output tile rows (256 for the CTA-pair form, else 128), tile columns (256,
 * 128, 64 or 32) and the number of CTAs K is split over (1, 2 or 4; decode shapes whose
 * 256-column tiles fill less than half the SMs). No reference counterpart: for tests of the
 * dispatch rules and for callers sizing column shards. Touches no device when sms > 0. Returns
 * the same shape errors as nvfp4_gemm; K must be > 0.
 */
int nvfp4_gemm_plan(int64_t M, int64_t N, int64_t K, int sms, int* tile_m, int* tile_n,
                    int* k_split);

/*
 * GEMM whose output is quantized to NVFP4 in the epilogue, for a layer whose consumer takes
 * NVFP4 input. No reference counterpart: it replaces nvfp4_gemm followed by nvfp4_quantize of
 * its bf16 output and produces exactly those bytes, q_out = packed E2M1 [M, N/2] and
 * sf_out = UE4M3 [M, N/16] of quantize(bf16(A.B^T / *scale), *out_scale), without writing or
 * re-reading bf16 D. `scale` and `out_scale` are device pointers to fp32 values. Requires
 * K % 256 == 0, K > 0, N % 32 == 0 (rows of q_out a multiple of 16 bytes); q_out 16-byte
 * aligned.
 */
int nvfp4_gemm_quantized(const void* A, const void* B, const void* A_sf, const void* B_sf,
                         const float* scale, const float* out_scale, void* q_out, void* sf_out,
                         int64_t M, int64_t N, int64_t K, cudaStream_t stream);

/*
 * Gate+up GEMM with SwiGLU in the epilogue (an MLP's first layer). No reference counterpart:
 * it replaces gemm_nvfp4 of A against the concatenated [gate; up] weight followed by
 * silu(gate) * up. B_gate_up holds the 2*I weight rows interleaved in groups of 128 — gate rows
 * 128t..128t+127, then up rows 128t..128t+127, for t = 0..I/128-1 — with B_gate_up_sf in the
 * same row order (my_nvfp4_gemm_b200.swiglu.interleave_gate_up builds both). N = 2*I.
 * out [M, I] bf16 = bf16(silu(Dg) * Du) evaluated in fp32, where Dg, Du are the bf16 values
 * bf16(A.B^T / scale) of the gate and up columns and silu(x) = x / (1 + exp(-x)).
 * Requires K % 256 == 0, K > 0, N % 256 == 0; out 16-byte aligned.
 */
int nvfp4_gemm_swiglu(const void* A, const void* B_gate_up, const void* A_sf,
                      const void* B_gate_up_sf, const float* scale, void* out, int64_t M,
                      int64_t N, int64_t K, cudaStream_t stream);

/*
 * Column-parallel GEMM with the all-gather of D fused into the epilogue (one process per GPU).
 * The reference has no multi-GPU path; this replaces "gemm_nvfp4 on a column shard of B, then an
 * all-gather of the shards' outputs". Every rank passes the same A, its own shard B_shard
 * [N_local, K/2] (+ B_sf_shard [N_local, K/16]) and `outputs`: a HOST array of `world` device
 * addresses, outputs[r] = rank r's full output D_r, bf16 [M, world * N_local] row-major, as
 * mapped in this process (its own buffer, and peers' buffers opened with nvfp4_ipc_open). The
 * kernel stores this rank's columns [rank*N_local, (rank+1)*N_local) of every tile into every
 * D_r over NVLink while later tiles compute. It does not wait for the other ranks: before any
 * rank reads D_r, every rank's call must have completed (e.g. a small all-reduce on the stream
 * after the call), and no rank may start the next call into the same buffers before every rank
 * has finished reading the previous result. Requires N_local % 8 == 0, world <= 8.
 */
int nvfp4_gemm_allgather(const void* A, const void* B_shard, const void* A_sf,
                         const void* B_sf_shard, const float* scale, void* const* outputs,
                         int world, int rank, int64_t M, int64_t N_local, int64_t K,
                         cudaStream_t stream);

/*
 * Sharing a device buffer with the other processes of the node (CUDA IPC). No reference
 * counterpart. nvfp4_ipc_export writes the IPC handle (NVFP4_IPC_HANDLE_BYTES bytes) of the
 * allocation containing `ptr` and ptr's offset in it; another process maps it with
 * nvfp4_ipc_open (on its current device, peer access enabled lazily) and unmaps it with
 * nvfp4_ipc_close(ptr, offset). A process cannot open its own handles.
 */
#define NVFP4_IPC_HANDLE_BYTES 64
int nvfp4_ipc_export(const void* ptr, void* handle_out, int64_t* offset_out);
int nvfp4_ipc_open(const void* handle, int64_t offset, void** ptr_out);
int nvfp4_ipc_close(void* ptr, int64_t offset);

/*
 * Scale factors in the 128x4 blocked layout that library block-scaled GEMMs consume (cuBLASLt's
 * block-scaling-factor layout; torch._scaled_mm with float4_e2m1fn_x2 operands). No reference
 * counterpart: the reference's factors only feed its own kernel. Row-major sf[rows][cols]
 * (cols = K/16 UE4M3 bytes per row, as every entry point above produces) <-> blocked: rows
 * padded to a multiple of 128 and cols to a multiple of 4 with zero bytes, cut into 128x4
 * blocks stored row-block-major; inside a block, row 32*i + j and column c sit at byte
 * 16*j + 4*i + c.
 *   nvfp4_blocked_scale_bytes: size of the blocked buffer (-1 for negative sizes)
 *   nvfp4_scale_to_blocked   : sf (any alignment) -> blocked (16-byte aligned, full size)
 *   nvfp4_scale_from_blocked : blocked (16-byte aligned) -> sf; padding is dropped
 * Sizes beyond 4,194,240 columns return NVFP4_ERR_TOO_LARGE.
 */
int64_t nvfp4_blocked_scale_bytes(int64_t rows, int64_t cols);
int nvfp4_scale_to_blocked(const void* sf, int64_t rows, int64_t cols, void* blocked,
                           cudaStream_t stream);
int nvfp4_scale_from_blocked(const void* blocked, int64_t rows, int64_t cols, void* sf,
                             cudaStream_t stream);

/*
 * Device-side status word, shared by all kernels of this library on the current device.
 * Kernels that wait on barriers give up after a bounded time, record
 * NVFP4_ERR_DEVICE_TIMEOUT here and return instead of hanging. Reading synchronises `stream`.
 * The reference has no counterpart (its waits spin forever, csrc/common/common.h:158-170).
 */
int nvfp4_device_status(int* status_out, cudaStream_t stream);
int nvfp4_clear_device_status(cudaStream_t stream);

/*
 * Self-test of the bounded-wait path: launches one warp that waits on a barrier nothing
 * ever completes, with the given limit in nanoseconds. The wait gives up, records
 * NVFP4_ERR_DEVICE_TIMEOUT in the device status word and the kernel returns normally.
 * No reference counterpart.
 */
int nvfp4_selftest_wait_timeout(uint64_t timeout_ns, cudaStream_t stream);

#ifdef __cplusplus
}
#endif

#endif /* NVFP4_B200_H_ */
