// scale_layout.cu — conversion of NVFP4 scale factors between the API's row-major layout and the
// 128x4 blocked layout that block-scaled GEMM libraries consume (cuBLASLt's block-scaling
// factor layout, and torch._scaled_mm for float4_e2m1fn_x2 operands).
//
// Row-major: sf[r][c], rows = the operand's rows, cols = K/16 (one UE4M3 byte per 16 elements).
// Blocked: rows padded to a multiple of 128 and cols to a multiple of 4 (padding bytes are 0);
// the padded matrix is cut into 128x4 blocks stored one after another, row-blocks outermost; one
// block is 512 contiguous bytes in which row r = 32*i + j (i < 4, j < 32) and column c (< 4) of
// the block sit at byte 16*j + 4*i + c.
//
// The reference has no such export (its scale factors only feed its own kernel); this is the
// format for handing quantized tensors to a library GEMM. Both directions are byte shuffles,
// HBM-bound: a CTA moves a 128-row x 64-column tile through shared memory so that global reads
// and writes are contiguous on both sides.
#include <cstdint>

#include "capi_util.h"

namespace nvfp4 {
namespace {

constexpr int kTileRows = 128;
constexpr int kTileCols = 64;                       // 16 blocks of 4 columns
constexpr int kTileWords = kTileCols / 4;           // 32-bit words per tile row
constexpr int kPitch = kTileWords + 1;              // padded: conflict-free column reads
constexpr int kThreads = 256;

__host__ __device__ inline int64_t round_up(int64_t x, int64_t m) { return (x + m - 1) / m * m; }

// One 32-bit word = 4 consecutive scale bytes of one row; out-of-range bytes read as 0.
template <bool kWordLoads>
__device__ __forceinline__ uint32_t load_word(const uint8_t* __restrict__ sf, int64_t rows,
                                              int64_t cols, int64_t r, int64_t c4) {
  if (r >= rows || c4 >= cols) return 0u;
  const uint8_t* p = sf + r * cols + c4;
  if (kWordLoads && c4 + 4 <= cols) return __ldg(reinterpret_cast<const uint32_t*>(p));
  uint32_t w = 0;
  for (int b = 0; b < 4 && c4 + b < cols; ++b) w |= uint32_t(__ldg(p + b)) << (8 * b);
  return w;
}

template <bool kWordLoads>
__global__ void __launch_bounds__(kThreads)
to_blocked_kernel(const uint8_t* __restrict__ sf, int64_t rows, int64_t cols,
                  uint4* __restrict__ out, int64_t col_blocks) {
  __shared__ uint32_t tile[kTileRows * kPitch];
  const int64_t r0 = int64_t(blockIdx.x) * kTileRows;
  const int64_t c0 = int64_t(blockIdx.y) * kTileCols;
  // Read the tile row by row: consecutive threads take consecutive words of a row.
  for (int i = threadIdx.x; i < kTileRows * kTileWords; i += kThreads) {
    const int tr = i / kTileWords, tw = i % kTileWords;
    tile[tr * kPitch + tw] = load_word<kWordLoads>(sf, rows, cols, r0 + tr, c0 + 4 * tw);
  }
  __syncthreads();
  // Write whole 512-byte blocks: 32 16-byte chunks each, chunk j = rows j, j+32, j+64, j+96.
  const int64_t cb0 = c0 / 4;
  for (int i = threadIdx.x; i < kTileWords * 32; i += kThreads) {
    const int tw = i / 32, j = i % 32;
    if (cb0 + tw >= col_blocks) continue;
    const uint4 v = make_uint4(tile[j * kPitch + tw], tile[(j + 32) * kPitch + tw],
                               tile[(j + 64) * kPitch + tw], tile[(j + 96) * kPitch + tw]);
    out[(int64_t(blockIdx.x) * col_blocks + cb0 + tw) * 32 + j] = v;
  }
}

template <bool kWordStores>
__global__ void __launch_bounds__(kThreads)
from_blocked_kernel(const uint4* __restrict__ blocked, int64_t rows, int64_t cols,
                    uint8_t* __restrict__ sf, int64_t col_blocks) {
  __shared__ uint32_t tile[kTileRows * kPitch];
  const int64_t r0 = int64_t(blockIdx.x) * kTileRows;
  const int64_t c0 = int64_t(blockIdx.y) * kTileCols;
  const int64_t cb0 = c0 / 4;
  for (int i = threadIdx.x; i < kTileWords * 32; i += kThreads) {
    const int tw = i / 32, j = i % 32;
    uint4 v = make_uint4(0u, 0u, 0u, 0u);
    if (cb0 + tw < col_blocks) v = __ldg(&blocked[(int64_t(blockIdx.x) * col_blocks + cb0 + tw) * 32 + j]);
    tile[j * kPitch + tw] = v.x;
    tile[(j + 32) * kPitch + tw] = v.y;
    tile[(j + 64) * kPitch + tw] = v.z;
    tile[(j + 96) * kPitch + tw] = v.w;
  }
  __syncthreads();
  for (int i = threadIdx.x; i < kTileRows * kTileWords; i += kThreads) {
    const int tr = i / kTileWords, tw = i % kTileWords;
    const int64_t r = r0 + tr, c4 = c0 + 4 * tw;
    if (r >= rows || c4 >= cols) continue;
    const uint32_t w = tile[tr * kPitch + tw];
    uint8_t* p = sf + r * cols + c4;
    if (kWordStores && c4 + 4 <= cols) {
      *reinterpret_cast<uint32_t*>(p) = w;
    } else {
      for (int b = 0; b < 4 && c4 + b < cols; ++b) p[b] = uint8_t(w >> (8 * b));
    }
  }
}

int check_shape(int64_t rows, int64_t cols) {
  if (rows < 0 || cols < 0) return NVFP4_ERR_INVALID_VALUE;
  // grid.y = ceil(cols / 64) must stay within 65535.
  if (round_up(cols, kTileCols) / kTileCols > 65535 || round_up(rows, kTileRows) / kTileRows > 0x7FFFFFFF)
    return NVFP4_ERR_TOO_LARGE;
  return NVFP4_OK;
}

}  // namespace
}  // namespace nvfp4

extern "C" {

int64_t nvfp4_blocked_scale_bytes(int64_t rows, int64_t cols) {
  if (rows < 0 || cols < 0) return -1;
  return nvfp4::round_up(rows, 128) * nvfp4::round_up(cols, 4);
}

int nvfp4_scale_to_blocked(const void* sf, int64_t rows, int64_t cols, void* blocked,
                           cudaStream_t stream) {
  using namespace nvfp4;
  const int st = check_shape(rows, cols);
  if (st != NVFP4_OK) return st;
  if (rows == 0 || cols == 0) return NVFP4_OK;
  if (!sf || !blocked) return NVFP4_ERR_INVALID_VALUE;
  if (!aligned_to(blocked, 16)) return NVFP4_ERR_MISALIGNED;
  const int64_t col_blocks = round_up(cols, 4) / 4;
  const dim3 grid(unsigned(round_up(rows, kTileRows) / kTileRows),
                  unsigned(round_up(cols, kTileCols) / kTileCols));
  const bool words = cols % 4 == 0 && aligned_to(sf, 4);
  if (words)
    to_blocked_kernel<true><<<grid, kThreads, 0, stream>>>(static_cast<const uint8_t*>(sf), rows, cols,
                                                           static_cast<uint4*>(blocked), col_blocks);
  else
    to_blocked_kernel<false><<<grid, kThreads, 0, stream>>>(static_cast<const uint8_t*>(sf), rows, cols,
                                                            static_cast<uint4*>(blocked), col_blocks);
  return status_from_cuda(cudaGetLastError());
}

int nvfp4_scale_from_blocked(const void* blocked, int64_t rows, int64_t cols, void* sf,
                             cudaStream_t stream) {
  using namespace nvfp4;
  const int st = check_shape(rows, cols);
  if (st != NVFP4_OK) return st;
  if (rows == 0 || cols == 0) return NVFP4_OK;
  if (!sf || !blocked) return NVFP4_ERR_INVALID_VALUE;
  if (!aligned_to(blocked, 16)) return NVFP4_ERR_MISALIGNED;
  const int64_t col_blocks = round_up(cols, 4) / 4;
  const dim3 grid(unsigned(round_up(rows, kTileRows) / kTileRows),
                  unsigned(round_up(cols, kTileCols) / kTileCols));
  const bool words = cols % 4 == 0 && aligned_to(sf, 4);
  if (words)
    from_blocked_kernel<true><<<grid, kThreads, 0, stream>>>(static_cast<const uint4*>(blocked), rows, cols,
                                                             static_cast<uint8_t*>(sf), col_blocks);
  else
    from_blocked_kernel<false><<<grid, kThreads, 0, stream>>>(static_cast<const uint4*>(blocked), rows, cols,
                                                              static_cast<uint8_t*>(sf), col_blocks);
  return status_from_cuda(cudaGetLastError());
}

}  // extern "C"
