// gemm_sm100.cu — block-scaled NVFP4 GEMM for B200 (sm_100a) on the 5th-generation tensor cores.
//
//   D[m, n] = bf16( sum_k e2m1(A[m,k]) sfA[m,k/16] e2m1(B[n,k]) sfB[n,k/16] / scale )
//
// Same operands, layouts and result as the reference kernel (csrc/gemm/gemm_nvfp4.cu:5-240):
// A [M, K/2] and B [N, K/2] packed E2M1, both K-major ("TN"); row-major UE4M3 scale factors
// [rows, K/16]; fp32 accumulation; bf16 row-major output. The reference's SM120 warp-level
// mma.sync design does not exist on sm_100a and is not followed. This kernel is:
//
//   * persistent over output tiles, in two forms:
//       single CTA (cta_group::1): 128 x 256 tiles, one CTA per SM (used when M <= 128);
//       CTA pair  (cta_group::2, cluster of 2): 256 x 256 tiles; each CTA loads its own 128
//               rows of A and its own 128-row half of B, the leader issues M=256 MMAs that read
//               both CTAs' shared memory and accumulate into both CTAs' tensor memory; per-SM
//               operand traffic per FLOP drops by a third and the ring is one stage deeper;
//   * warp-specialised (352 threads per CTA):
//       warp 8  TMA producer of the A/B tiles (128B-swizzled) into a STAGES-deep shared-memory
//               ring, guarded by full and empty mbarriers;
//       warp 10 TMA producer of the scale-factor tiles into their own ring (up to 64 bytes of
//               every row per load, so whole sectors are fetched);
//       warps 0-3 scale-factor writers: read the API's row-major UE4M3 factors from shared
//               memory and write them with tcgen05.st into the stage's tensor-memory slot, in
//               the lane/column layout the block-scaled MMA reads (one warp per lane quarter);
//       warp 9  MMA issuer (the pair's leader only): owns the tensor-memory allocation and
//               issues tcgen05.mma .kind::mxf4nvf4.block_scale.scale_vec::4X (K=64) into a
//               TMEM fp32 accumulator;
//       warps 4-7 epilogue: tcgen05.ld of the accumulator, x (1/scale), bf16 convert in
//               registers, release of TMEM, then 64B-swizzled shared-memory staging and TMA
//               tensor stores (bounds-clipped, so ragged M and N need no masking);
//   * fault-safe: every mbarrier wait is bounded; a wait that times out raises a CTA-wide abort
//     flag, every role returns, copies and MMAs in flight are drained (bounded), TMEM is freed,
//     and NVFP4_ERR_DEVICE_TIMEOUT is recorded in the device status word.
// No TMA load uses cluster multicast: every CTA loads only into its own shared memory.
#include <cstdint>
#include <mutex>

#include "block_quant.cuh"
#include "capi_util.h"
#include "ptx.cuh"

// Device status word (NVFP4_OK or the first error a kernel recorded).
__device__ int g_nvfp4_device_status = 0;

namespace nvfp4 {
namespace gemm {

constexpr int kRowsPerCta = 128;    // accumulator rows per CTA (TMEM lanes)
constexpr int kBK = 256;            // K elements per pipeline stage = 128 packed bytes
constexpr int kBKBytes = kBK / 2;
constexpr int kUmmaK = 64;          // K per tcgen05.mma kind::mxf4nvf4
constexpr int kKSteps = kBK / kUmmaK;
constexpr int kSfBytesPerRow = kBK / 16;  // 16 scale bytes per row per stage
constexpr int kNumSfWarps = 4;            // warps 0-3: scale-factor writers (TMEM quarters 0-3)
constexpr int kFirstEpiWarp = 4;          // warps 4-7: epilogue (TMEM quarters 0-3)
constexpr int kNumEpiWarps = 4;
constexpr int kProducerWarp = 8;          // TMA producer of the A/B tiles
constexpr int kMmaWarp = 9;               // MMA issuer, owns the TMEM allocation
constexpr int kSfProducerWarp = 10;       // TMA producer of the scale-factor tiles
constexpr int kThreads = 32 * 11;

// Scale factors have their own shared-memory ring of SF_SLOTS slots, filled by their own
// producer warp. One slot holds SF_KB consecutive k-blocks (16 * SF_KB bytes of every row): the
// API's row-major factors are 16 bytes per row per k-block with rows K/16 bytes apart, so a
// 16-byte box row would fetch half of a 32-byte sector per request; 64-byte rows (SF_KB = 4)
// use whole sectors and a quarter of the requests. Rows of 32 or 64 bytes are swizzled by the
// TMA unit so that the writers' 16-byte reads stay free of bank conflicts.
//
// EPI_COLS: output columns per epilogue store box (32 rows x EPI_COLS bf16 staged in shared
// memory per warp): 64 gives 128-byte rows (128B-swizzled), which is what TMA stores into
// another GPU's memory over NVLink need to run near link rate (~666 GB/s measured, against
// ~440 GB/s with 64-byte rows); 32 halves the staging memory.
// EPI_BUFS: staging buffers per epilogue warp (a warp fills one while the TMA unit reads the
// other).
// KSPLIT (single-CTA form, bf16 output): the K range of a tile is split over KSPLIT CTAs of one
// cluster, each CTA one tile and K / KSPLIT of it. Decode shapes sharded along N leave too few
// 256-column tiles for the SMs, and each CTA's MMA chain (K / 64 block-scaled MMAs at a fixed
// cost of ~130 cycles each when interleaved with barrier waits, whatever N) then bounds the
// call; splitting K divides the chain. The epilogue sums the fp32 partials across the cluster
// in a fixed order (see the split epilogue).
template <int BN_, int STAGES_, int ACC_STAGES_, bool PAIR_, int SF_KB_, int SF_SLOTS_,
          int EPI_COLS_ = 32, int EPI_BUFS_ = 1, int KSPLIT_ = 1>
struct Cfg {
  static constexpr int BN = BN_;
  static constexpr int EPI_COLS = EPI_COLS_;
  static constexpr int EPI_BUFS = EPI_BUFS_;
  static constexpr int EPI_ROW_BYTES = EPI_COLS * 2;
  static constexpr int EPI_BUF_BYTES = 32 * EPI_ROW_BYTES;
  static_assert(EPI_COLS == 32 || EPI_COLS == 64, "EPI_COLS must be 32 or 64");
  static constexpr int STAGES = STAGES_;
  static constexpr int ACC_STAGES = ACC_STAGES_;
  static constexpr bool PAIR = PAIR_;
  static constexpr int SF_KB = SF_KB_;                     // k-blocks per scale-factor slot
  static constexpr int SF_SLOTS = SF_SLOTS_;
  static constexpr int SF_ROW_BYTES = kSfBytesPerRow * SF_KB;
  static_assert(SF_KB == 1 || SF_KB == 2 || SF_KB == 4, "SF_KB must be 1, 2 or 4");
  static constexpr int CTAS = PAIR ? 2 : 1;
  static constexpr int TILE_M = kRowsPerCta * CTAS;        // output rows per tile
  static constexpr int B_ROWS = BN / CTAS;                 // B rows each CTA loads
  static_assert(BN == 256 || (!PAIR && (BN == 32 || BN == 64 || BN == 128)),
                "BN must be 256, or 32/64/128 for the single-CTA form");
  static constexpr int KSPLIT = KSPLIT_;
  static_assert(KSPLIT == 1 || ((KSPLIT == 2 || KSPLIT == 4 || KSPLIT == 8) && !PAIR && SF_KB == 1 &&
                                BN % (8 * KSPLIT) == 0),
                "KSPLIT: 1, or 2/4/8 in the single-CTA form with one-k-block scale-factor slots");

  static constexpr int A_STAGE = kRowsPerCta * kBKBytes;   // 16 KiB
  static constexpr int B_STAGE = B_ROWS * kBKBytes;
  static constexpr int SFA_SLOT = kRowsPerCta * SF_ROW_BYTES;
  static constexpr int SFB_SLOT = BN * SF_ROW_BYTES;       // every CTA holds all BN rows

  static constexpr int OFF_A = 0;
  static constexpr int OFF_B = OFF_A + STAGES * A_STAGE;
  static constexpr int OFF_SFA = OFF_B + STAGES * B_STAGE;
  static constexpr int OFF_SFB = OFF_SFA + SF_SLOTS * SFA_SLOT;
  static constexpr int OFF_EPI = OFF_SFB + SF_SLOTS * SFB_SLOT;
  static constexpr int OFF_BAR = OFF_EPI + kNumEpiWarps * EPI_BUFS * EPI_BUF_BYTES;
  static constexpr int NUM_BARS = 2 * STAGES + 2 * SF_SLOTS + 2 * ACC_STAGES + 1;
  static constexpr int OFF_MISC = OFF_BAR + NUM_BARS * 8;
  static constexpr int OFF_QTAB = OFF_MISC + 16;           // 256 fp32: quantized-output table
  static constexpr int SMEM_BYTES = OFF_QTAB + 256 * 4;
  static constexpr int SMEM_ALLOC = SMEM_BYTES + 1024;     // slack to align the base to 1 KiB
  static_assert(SMEM_ALLOC <= 232448, "shared memory budget exceeded");
  // Split epilogue: the fp32 partial tile, kRowsPerCta rows of BN + 4 floats (16-byte aligned
  // rows whose 16-byte chunks fall in distinct bank groups for the 8 lanes of a store phase),
  // goes in the A/B ring, idle once the tile's MMAs are done.
  static constexpr int PART_STRIDE = BN + 4;
  static_assert(KSPLIT == 1 || kRowsPerCta * PART_STRIDE * 4 <= STAGES * (A_STAGE + B_STAGE),
                "split epilogue: the partial tile must fit in the A/B ring");

  // Tensor memory columns: accumulators, then one scale-factor slot per pipeline stage, so the
  // factors of later fills are written while the MMAs of earlier ones still read theirs. Within
  // a slot: B's factors for K-steps 0..3 (BN/32 columns each, padded to 8 so that every step's
  // address stays 8-column aligned), then A's (4 columns each).
  static constexpr uint32_t SFB_COLS_PER_STEP = 8;
  static constexpr uint32_t SFB_PART = kKSteps * SFB_COLS_PER_STEP;
  static constexpr uint32_t SF_SLOT_COLS = kKSteps * (4 + SFB_COLS_PER_STEP);
  static constexpr uint32_t COL_SF = BN * ACC_STAGES;
  static constexpr uint32_t COLS_USED = COL_SF + STAGES * SF_SLOT_COLS;
  static constexpr uint32_t TMEM_COLS = COLS_USED <= 32 ? 32 : COLS_USED <= 64 ? 64
                                      : COLS_USED <= 128 ? 128 : COLS_USED <= 256 ? 256 : 512;
  static_assert(COLS_USED <= 512, "tensor memory budget exceeded");
};

struct Params {
  const float* scale_ptr;  // device scalar, or nullptr -> scale_val
  float scale_val;
  int m;                   // rows of D
  int n;                   // columns of D
  int m_blocks;            // tiles along M (TILE_M rows each)
  int n_blocks;            // tiles along N (BN columns each)
  int k_stages;
  // transaction bytes of one A/B fill (the pair's total) and of one scale-factor slot (this
  // CTA's): the A and A-scale boxes cover a_rows rows (kRowsPerCta, or M for a single-CTA
  // launch with M < kRowsPerCta)
  uint32_t ab_tx;
  uint32_t sf_tx;
  uint64_t timeout_ns;
  // quantized output (kEpiQuant): D is quantized to NVFP4 with the per-tensor scale *out_scale_ptr;
  // the codes go through the destination map, the scale bytes to sf_out [m][sf_pitch].
  const float* out_scale_ptr;
  uint8_t* sf_out;
  int64_t sf_pitch;
  // bf16 D of a single destination: base and row pitch in elements (direct-store epilogue)
  uint16_t* d;
  int64_t ldd;
  // every destination's base (this rank's column slice of each rank's D, local first; row pitch
  // ldd): the split-K epilogue stores its sums to each
  uint16_t* dsts[8];
  int ndst;
};

// Tile order: the M x N tile grid is walked in bands of kGroupM tile rows, column by column
// within a band, so the tiles the persistent CTAs work on at any moment share a narrow band of
// A rows and a few B column blocks in L2.
constexpr int kGroupM = 16;

__device__ __forceinline__ void tile_coords(int tile, const Params& p, int& mb, int& nb) {
  const int per_band = kGroupM * p.n_blocks;
  const int band = tile / per_band;
  const int first = band * kGroupM;
  const int rows = min(p.m_blocks - first, kGroupM);
  const int r = tile - band * per_band;
  mb = first + r % rows;
  nb = r / rows;
}

// Scale-factor writer (one warp per TMEM lane quarter q). The block-scaled MMA of sub-partition
// q reads the scale factors of A row 32q+r from TMEM lane 32q+r, column sfa+q, and those of B
// row n from lane 32q+(n%32), column sfb+n/32 (B's factors are needed by every quarter). The
// warp reads its rows' factors for k-block c of the shared-memory slot (16 bytes per row =
// K-steps 0..3) and writes its quarter of the stage's TMEM slot with tcgen05.st:
//   slot + j*(BN/32) + i   <- step-j word of B row 32i + lane     (BN/8 columns)
//   slot + BN/8 + 4j + q   <- step-j word of A row 32q + lane     (4 of the 16 A columns)
//
// Shared-memory address of k-block c's 16 bytes of row `row` in a scale-factor slot. The TMA
// unit's 32B/64B swizzle XORs the 16-byte chunk index with address bits 7 and up of the row.
template <class C>
__device__ __forceinline__ uint32_t sf_chunk_addr(uint32_t base, int row, int c) {
  const int sw = (row * C::SF_KB / 8) % C::SF_KB;
  return base + uint32_t(row * C::SF_ROW_BYTES + ((c ^ sw) << 4));
}

template <class C>
__device__ __forceinline__ void write_sf_slot(uint32_t slot, uint32_t sfa_s, uint32_t sfb_s, int c,
                                              int q, int lane) {
  constexpr int kChunksB = C::BN / 32;
  constexpr int kStep = int(C::SFB_COLS_PER_STEP);
  if constexpr (kChunksB == kStep) {
    uint32_t vb[C::SFB_PART];
#pragma unroll
    for (int i = 0; i < kChunksB; ++i) {
      const uint4 w = ptx::ld_shared_v4(sf_chunk_addr<C>(sfb_s, 32 * i + lane, c));
      vb[0 * kStep + i] = w.x;
      vb[1 * kStep + i] = w.y;
      vb[2 * kStep + i] = w.z;
      vb[3 * kStep + i] = w.w;
    }
    ptx::tmem_st_32x32b_x32(slot, vb);
  } else {
    // BN < 256: only the BN/32 columns of each K-step that the MMA reads are written (the rest of
    // the step's 8 columns is alignment padding).
    uint32_t w[kChunksB][4];
#pragma unroll
    for (int i = 0; i < kChunksB; ++i) {
      const uint4 v = ptx::ld_shared_v4(sf_chunk_addr<C>(sfb_s, 32 * i + lane, c));
      w[i][0] = v.x;
      w[i][1] = v.y;
      w[i][2] = v.z;
      w[i][3] = v.w;
    }
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const uint32_t col = slot + uint32_t(j * kStep);
      if constexpr (kChunksB == 1) ptx::tmem_st_32x32b_x1(col, w[0][j]);
      else if constexpr (kChunksB == 2) ptx::tmem_st_32x32b_x2(col, w[0][j], w[1][j]);
      else ptx::tmem_st_32x32b_x4(col, w[0][j], w[1][j], w[2][j], w[3][j]);
    }
  }
  const uint4 a = ptx::ld_shared_v4(sf_chunk_addr<C>(sfa_s, 32 * q + lane, c));
  // A: quarter q's MMA reads K-step j's factors from column SFB_PART + 4j + q only; the other
  // three columns of each group belong to the other quarters' lanes and are left alone.
  const uint32_t sfa = slot + C::SFB_PART + uint32_t(q);
  ptx::tmem_st_32x32b_x1(sfa + 0, a.x);
  ptx::tmem_st_32x32b_x1(sfa + 4, a.y);
  ptx::tmem_st_32x32b_x1(sfa + 8, a.z);
  ptx::tmem_st_32x32b_x1(sfa + 12, a.w);
}

// Where the epilogue stores D: NDST = 1 for the plain GEMM; the column-parallel form with a
// fused all-gather passes one map per rank, each covering this rank's column slice of that
// rank's full output (so the TMA unit clips at the slice edge), local output first.
constexpr int kMaxRanks = 8;

template <int NDST>
struct DstMaps {
  CUtensorMap map[NDST];
  int count;  // maps in use, 1..NDST
};

// What the epilogue stores (MODE):
//   kEpiBf16   : bf16 D;
//   kEpiQuant  : each finished bf16 row quantized to NVFP4 (block_quant.cuh, the arithmetic of
//                quantize_kernel): packed codes through the destination map, scale bytes to
//                p.sf_out;
//   kEpiSwiglu : the tile's first BN/2 columns are gate and the last BN/2 the matching up
//                columns (B's rows interleaved that way); stores bf16(silu(g) * u) computed in
//                fp32 from the bf16 values of g and u, BN/2 output columns per tile.
constexpr int kEpiBf16 = 0;
constexpr int kEpiQuant = 1;
constexpr int kEpiSwiglu = 2;

// silu(x) = x / (1 + exp(-x)) in fp32 (IEEE division, no contraction), as torch evaluates it.
__device__ __forceinline__ float silu_f32(float x) {
  return __fdiv_rn(x, __fadd_rn(1.0f, expf(-x)));
}

// bf16 pair of gate values and the matching pair of up values -> bf16 pair of silu(g) * u.
__device__ __forceinline__ uint32_t swiglu_bf16x2(uint32_t g, uint32_t u) {
  return ptx::f32x2_to_bf16x2(__fmul_rn(silu_f32(bq::bf16lo_to_f32(g)), bq::bf16lo_to_f32(u)),
                              __fmul_rn(silu_f32(bq::bf16hi_to_f32(g)), bq::bf16hi_to_f32(u)));
}

template <class C, int NDST, int MODE = kEpiBf16>
__global__ void __launch_bounds__(kThreads, 1)
gemm_kernel(const __grid_constant__ CUtensorMap tm_a, const __grid_constant__ CUtensorMap tm_b,
            const __grid_constant__ CUtensorMap tm_sfa, const __grid_constant__ CUtensorMap tm_sfb,
            const __grid_constant__ DstMaps<NDST> dst, const Params p) {
  constexpr bool kPair = C::PAIR;
  constexpr int kSplit = C::KSPLIT;
  static_assert(MODE == kEpiBf16 || C::BN == 256, "epilogue variants use 256-column tiles");
  static_assert(kSplit == 1 || MODE == kEpiBf16, "split K: bf16 output");
  constexpr int kGroup = C::CTAS;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  uint8_t* sA = smem + C::OFF_A;
  uint8_t* sB = smem + C::OFF_B;
  uint8_t* sSFA = smem + C::OFF_SFA;
  uint8_t* sSFB = smem + C::OFF_SFB;
  uint8_t* sEPI = smem + C::OFF_EPI;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + C::OFF_BAR);
  // full[s] (the leader's) completes when the stage's A/B tiles of both CTAs have landed (the
  // producer's expect-tx arrival plus the bytes) and every writer warp of both CTAs has put
  // the stage's scale factors into tensor memory: one barrier for the MMA warp to poll.
  uint64_t* full_bar = bars;
  uint64_t* empty_bar = bars + C::STAGES;           // MMAs done with the stage -> producers
  uint64_t* sfull_bar = bars + 2 * C::STAGES;       // this CTA's scale-factor slot landed
  uint64_t* sempty_bar = sfull_bar + C::SF_SLOTS;   // writers done reading the slot
  uint64_t* tfull_bar = sempty_bar + C::SF_SLOTS;   // accumulator ready -> epilogue
  uint64_t* tempty_bar = tfull_bar + C::ACC_STAGES; // accumulator drained -> MMA (leader's)
  uint64_t* drain_bar = tempty_bar + C::ACC_STAGES; // MMA drain before TMEM free
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + C::OFF_MISC);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + C::OFF_MISC + 4);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t rank = kPair ? ptx::cluster_ctarank() : 0u;
  const int num_tiles = p.m_blocks * p.n_blocks;
  // Split K: cluster c works on tile c (one tile per cluster), its CTA s on k-blocks
  // [s * k_stages / KSPLIT, (s + 1) * k_stages / KSPLIT).
  const int split = kSplit > 1 ? int(ptx::cluster_ctarank()) : 0;
  const int first_tile = kPair ? int(blockIdx.x >> 1) : int(blockIdx.x) / kSplit;
  const int tile_step = kPair ? int(gridDim.x >> 1) : int(gridDim.x) / kSplit;
  const int kb_count = p.k_stages / kSplit;
  const int kb_lo = split * kb_count;
  const int kb_hi = kb_lo + kb_count;

  if (threadIdx.x == 0) {
    for (int i = 0; i < C::STAGES; ++i) {
      ptx::mbar_init(&full_bar[i], 1 + kNumSfWarps * C::CTAS);
      ptx::mbar_init(&empty_bar[i], 1);
    }
    for (int i = 0; i < C::SF_SLOTS; ++i) {
      ptx::mbar_init(&sfull_bar[i], 1);
      ptx::mbar_init(&sempty_bar[i], kNumSfWarps);
    }
    for (int i = 0; i < C::ACC_STAGES; ++i) {
      ptx::mbar_init(&tfull_bar[i], 1);
      ptx::mbar_init(&tempty_bar[i], kNumEpiWarps * C::CTAS);
    }
    ptx::mbar_init(drain_bar, 1);
    *abort_flag = 0;
    ptx::fence_mbar_init();
  }
  if (warp == kProducerWarp && lane == 0) {
    ptx::tma_prefetch_desc(&tm_a);
    ptx::tma_prefetch_desc(&tm_b);
    ptx::tma_prefetch_desc(&tm_sfa);
    ptx::tma_prefetch_desc(&tm_sfb);
    for (int i = 0; i < dst.count; ++i) ptx::tma_prefetch_desc(&dst.map[i]);
  }
  if (warp == kMmaWarp) {
    ptx::tmem_alloc_g<kGroup>(tmem_slot, C::TMEM_COLS);
    ptx::tmem_relinquish_g<kGroup>();
  }
  ptx::tc_fence_before_sync();
  if constexpr (kPair || kSplit > 1) ptx::cluster_sync(); else __syncthreads();
  ptx::tc_fence_after_sync();
  const uint32_t tmem_base = *tmem_slot;

  // Programmatic dependent launch (single-destination launches): the grid is launched as soon as
  // every CTA of the previous kernel on the stream has exited, and the setup above (barriers,
  // TMEM, descriptor prefetch) overlaps that kernel's completion. It touches no global memory;
  // every thread waits for the previous kernel's completion before its first global access.
  // There is no early trigger for the next kernel: CTAs that launch into the SMs this grid leaves
  // idle, and wait there, slowed the decode-shape main loop by ~12 % in measurements.
  if constexpr (NDST == 1) {
    // While the previous kernel completes, warm L2 with this CTA's first weight fills: a
    // prefetch changes no memory, so it is safe even for operands that kernel writes, and the
    // loads issued after the wait then start from L2 instead of paying the DRAM latency.
    if (warp == kProducerWarp && lane == 0 && first_tile < num_tiles) {
      int mb, nb;
      tile_coords(first_tile, p, mb, nb);
      const int n_cta = nb * C::BN + int(rank) * C::B_ROWS;
      for (int kb = kb_lo; kb < kb_lo + C::STAGES && kb < kb_hi; ++kb)
        ptx::tma_prefetch_2d(&tm_b, kb * kBKBytes, n_cta);
      ptx::tma_prefetch_2d(&tm_sfb, kb_lo * kSfBytesPerRow, nb * C::BN);
    }
    ptx::griddep_wait();
  }

  if (warp == kProducerWarp) {
    // ------------------------------------------------------------------ TMA producer
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      for (int tile = first_tile; tile < num_tiles; tile += tile_step) {
        int mb, nb;
        tile_coords(tile, p, mb, nb);
        const int m_cta = mb * C::TILE_M + int(rank) * kRowsPerCta;
        const int n_cta = nb * C::BN + int(rank) * C::B_ROWS;
        for (int kb = kb_lo; kb < kb_hi; ++kb) {
          if (!ptx::mbar_wait<kPair>(&empty_bar[stage], phase ^ 1, abort_flag, p.timeout_ns))
            goto producer_done;
          if (rank == 0) ptx::mbar_arrive_expect_tx(&full_bar[stage], p.ab_tx);
          if constexpr (kPair) {
            ptx::tma_load_2d_pair(sA + stage * C::A_STAGE, &tm_a, &full_bar[stage], kb * kBKBytes, m_cta);
            ptx::tma_load_2d_pair(sB + stage * C::B_STAGE, &tm_b, &full_bar[stage], kb * kBKBytes, n_cta);
          } else {
            ptx::tma_load_2d(sA + stage * C::A_STAGE, &tm_a, &full_bar[stage], kb * kBKBytes, m_cta);
            ptx::tma_load_2d(sB + stage * C::B_STAGE, &tm_b, &full_bar[stage], kb * kBKBytes, n_cta);
          }
          if (++stage == C::STAGES) { stage = 0; phase ^= 1; }
        }
      }
    producer_done:
      // Never leave a TMA write in flight into shared memory of an exiting CTA. Without an
      // abort, the MMA warp has consumed every fill, so every copy has landed. After an abort
      // the full barriers may never complete (they also count the writer warps, which stop), so
      // wait a fixed bounded time, far above a copy's latency, instead.
      if (*abort_flag) {
        const uint64_t t0 = ptx::globaltimer_ns();
        while (ptx::globaltimer_ns() - t0 < 1000000ull) {
        }
      }
    }
  } else if (warp == kSfProducerWarp) {
    // ------------------------------------------------------------------ scale-factor producer
    // Slot loads of SF_KB k-blocks of this CTA's A rows and all BN B rows, as far ahead of the
    // writers as the SF_SLOTS-deep ring allows (each CTA of a pair loads its own).
    if (lane == 0) {
      int slot = 0;
      uint32_t phase = 0;
      int64_t loads = 0;
      for (int tile = first_tile; tile < num_tiles; tile += tile_step) {
        int mb, nb;
        tile_coords(tile, p, mb, nb);
        const int row_a = mb * C::TILE_M + int(rank) * kRowsPerCta;
        const int row_b = nb * C::BN;
        for (int kb = kb_lo; kb < kb_hi; kb += C::SF_KB) {
          if (!ptx::mbar_wait<kPair>(&sempty_bar[slot], phase ^ 1, abort_flag, p.timeout_ns))
            goto sf_producer_done;
          ptx::mbar_arrive_expect_tx(&sfull_bar[slot], p.sf_tx);
          ptx::tma_load_2d(sSFA + slot * C::SFA_SLOT, &tm_sfa, &sfull_bar[slot],
                           kb * kSfBytesPerRow, row_a);
          ptx::tma_load_2d(sSFB + slot * C::SFB_SLOT, &tm_sfb, &sfull_bar[slot],
                           kb * kSfBytesPerRow, row_b);
          ++loads;
          if (++slot == C::SF_SLOTS) { slot = 0; phase ^= 1; }
        }
      }
    sf_producer_done:
      {
        int no_abort = 0;
        const int64_t last = loads < C::SF_SLOTS ? loads : C::SF_SLOTS;
        for (int64_t i = 0; i < last; ++i) {
          const int64_t g = loads - 1 - i;
          ptx::mbar_wait<kPair>(&sfull_bar[g % C::SF_SLOTS], uint32_t((g / C::SF_SLOTS) & 1),
                                &no_abort, p.timeout_ns);
        }
      }
    }
  } else if (warp == kMmaWarp) {
    // ------------------------------------------------------------------ MMA issuer
    if (lane == 0 && rank == 0) {
      // The tensor pipe does not let this thread run ahead of it: every instruction between two
      // MMAs delays the next one. So the loop polls one barrier per k-block and advances
      // precomputed descriptors and TMEM addresses by constants.
      constexpr uint32_t idesc = ptx::make_idesc_mxf4nvf4(C::TILE_M, C::BN);
      constexpr uint32_t kADescStep = C::A_STAGE >> 4;   // descriptor start-address units
      constexpr uint32_t kBDescStep = C::B_STAGE >> 4;
      const uint64_t a_desc0 = ptx::make_smem_desc(ptx::smem_u32(sA), 0, 1024, ptx::kLayoutSW128);
      const uint64_t b_desc0 = ptx::make_smem_desc(ptx::smem_u32(sB), 0, 1024, ptx::kLayoutSW128);
      const uint32_t t_sf0 = tmem_base + C::COL_SF;
      int stage = 0;
      uint32_t phase = 0;
      int acc = 0;
      uint32_t acc_phase = 0;
      for (int tile = first_tile; tile < num_tiles; tile += tile_step) {
        if (!ptx::mbar_wait<kPair>(&tempty_bar[acc], acc_phase ^ 1, abort_flag, p.timeout_ns))
          goto mma_done;
        ptx::tc_fence_after_sync();
        const uint32_t d_tmem = tmem_base + uint32_t(acc * C::BN);
        for (int kb = kb_lo; kb < kb_hi; ++kb) {
          if (!ptx::mbar_wait<kPair>(&full_bar[stage], phase, abort_flag, p.timeout_ns)) goto mma_done;
          ptx::tc_fence_after_sync();
          const uint64_t a_desc = a_desc0 + uint32_t(stage) * kADescStep;
          const uint64_t b_desc = b_desc0 + uint32_t(stage) * kBDescStep;
          const uint32_t t_sfb = t_sf0 + uint32_t(stage) * C::SF_SLOT_COLS;
          const uint32_t t_sfa = t_sfb + C::SFB_PART;
          // K-step j starts 32 bytes (2 descriptor units) further along the swizzled rows.
          if constexpr (kPair) {
            ptx::tc_mma_mxf4nvf4_pair(d_tmem, a_desc, b_desc, idesc, t_sfa, t_sfb, kb != kb_lo ? 1u : 0u);
#pragma unroll
            for (int j = 1; j < kKSteps; ++j)
              ptx::tc_mma_mxf4nvf4_pair(d_tmem, a_desc + 2 * j, b_desc + 2 * j, idesc, t_sfa + 4 * j,
                                        t_sfb + j * C::SFB_COLS_PER_STEP, 1u);
            ptx::tc_commit_pair(&empty_bar[stage], 0x3);  // stage free in both CTAs
          } else {
            ptx::tc_mma_mxf4nvf4(d_tmem, a_desc, b_desc, idesc, t_sfa, t_sfb, kb != kb_lo ? 1u : 0u);
#pragma unroll
            for (int j = 1; j < kKSteps; ++j)
              ptx::tc_mma_mxf4nvf4(d_tmem, a_desc + 2 * j, b_desc + 2 * j, idesc, t_sfa + 4 * j,
                                   t_sfb + j * C::SFB_COLS_PER_STEP, 1u);
            ptx::tc_commit(&empty_bar[stage]);
          }
          if (++stage == C::STAGES) { stage = 0; phase ^= 1; }
        }
        if constexpr (kPair) ptx::tc_commit_pair(&tfull_bar[acc], 0x3);
        else ptx::tc_commit(&tfull_bar[acc]);
        if (++acc == C::ACC_STAGES) { acc = 0; acc_phase ^= 1; }
      }
    mma_done:
      // Drain every tcgen05 operation this thread issued before TMEM is released.
      {
        int no_abort = 0;
        if constexpr (kPair) ptx::tc_commit_pair(drain_bar, 0x1);
        else ptx::tc_commit(drain_bar);
        ptx::mbar_wait<kPair>(drain_bar, 0, &no_abort, p.timeout_ns);
      }
    }
  } else if (warp < kNumSfWarps) {
    // ------------------------------------------------------------------ scale-factor writers
    // Fill f = (tile, kb) uses k-block c = kb % SF_KB of the current scale-factor slot. Its
    // factors go to the TMEM slot of stage f % STAGES once (1) the shared-memory slot has landed
    // (waited for at its first k-block) and (2) the MMAs of fill f - STAGES, which read the TMEM
    // slot's previous contents, are done (the empty phase the A/B producer also waits for).
    // After the slot's last k-block of the tile, the slot goes back to the scale-factor
    // producer.
    const int q = warp;
    const uint32_t lane_base = uint32_t(q * 32) << 16;
    int stage = 0;
    uint32_t phase = 0;
    int slot = 0;
    uint32_t slot_phase = 0;
    for (int tile = first_tile; tile < num_tiles; tile += tile_step) {
      for (int kb = kb_lo; kb < kb_hi; ++kb) {
        const int c = kb % C::SF_KB;
        bool ok = true;
        if (c == 0) ok = ptx::mbar_wait<kPair>(&sfull_bar[slot], slot_phase, abort_flag, p.timeout_ns);
        if (ok) ok = ptx::mbar_wait<kPair>(&empty_bar[stage], phase ^ 1, abort_flag, p.timeout_ns);
        if (!__all_sync(0xFFFFFFFFu, ok)) goto sf_done;
        ptx::tc_fence_after_sync();
        write_sf_slot<C>(tmem_base + lane_base + C::COL_SF + uint32_t(stage) * C::SF_SLOT_COLS,
                         ptx::smem_u32(sSFA + slot * C::SFA_SLOT),
                         ptx::smem_u32(sSFB + slot * C::SFB_SLOT), c, q, lane);
        ptx::tmem_wait_st();
        ptx::tc_fence_before_sync();
        __syncwarp();
        if (lane == 0) {
          if constexpr (kPair) ptx::mbar_arrive_cta(&full_bar[stage], 0);
          else ptx::mbar_arrive(&full_bar[stage]);
        }
        if (c == C::SF_KB - 1 || kb == kb_hi - 1) {
          if (lane == 0) ptx::mbar_arrive(&sempty_bar[slot]);
          if (++slot == C::SF_SLOTS) { slot = 0; slot_phase ^= 1; }
        }
        if (++stage == C::STAGES) { stage = 0; phase ^= 1; }
      }
    }
  sf_done:;
  } else if (warp >= kFirstEpiWarp && warp < kFirstEpiWarp + kNumEpiWarps) {
    // ------------------------------------------------------------------ epilogue
    const int ew = warp - kFirstEpiWarp;  // == warp % 4: TMEM lanes 32*ew .. 32*ew+31
    // Single-CTA bf16 form (decode shapes, usually one tile per CTA): see the store loop.
    constexpr bool kRingStage = !kPair && kSplit == 1 && NDST == 1 && MODE == kEpiBf16;
    static_assert(!kRingStage || kNumEpiWarps * 64 * C::BN <= C::STAGES * (C::A_STAGE + C::B_STAGE),
                  "the A/B ring must hold every epilogue warp's boxes of one tile");
    const float scale = p.scale_ptr ? __ldg(p.scale_ptr) : p.scale_val;
    const float alpha = __frcp_rn(scale);
    const uint64_t alpha2 = ptx::f32x2_splat(alpha);
    uint8_t* buf = sEPI + ew * C::EPI_BUFS * C::EPI_BUF_BYTES;
    const uint32_t buf_s = ptx::smem_u32(buf);
    // TMA swizzle of staging row `lane`: the 16-byte chunk index XOR address bits 7.. of the row
    const uint32_t swz = C::EPI_COLS == 64 ? uint32_t(lane & 7) : uint32_t((lane >> 1) & 3);
    if constexpr (MODE == kEpiQuant) {
      // Encode multiplier per scale byte, computed once (the per-block reciprocal would cost a
      // slow-path call with the whole drained row live in registers).
      const float rcp_s_out = __frcp_rn(__ldg(p.out_scale_ptr));
      float* tab = reinterpret_cast<float*>(smem + C::OFF_QTAB);
      for (int i = ew * 32 + lane; i < 256; i += kNumEpiWarps * 32)
        tab[i] = bq::os_of_scale_byte(uint32_t(i), rcp_s_out);
      asm volatile("bar.sync 1, %0;" ::"n"(kNumEpiWarps * 32) : "memory");  // epilogue warps only
    }
    if constexpr (kSplit > 1) {
      // Split K (one tile per cluster). Step 1: this CTA's fp32 partial rows that lie inside D go
      // to the idle A/B ring (the tile's MMAs, which tfull waited for, consumed every fill).
      // Step 2: cluster barrier, which every thread of the cluster passes exactly once before
      // the final one, on the abort path too. Step 3: CTA s owns columns [s, s + 1) * BN /
      // KSPLIT of the tile: the KSPLIT partials summed in split order (fp32 adds, round to
      // nearest), times 1/scale, to bf16, 4 columns per task, read from each CTA's shared
      // memory, which stays valid until the final cluster barrier.
      int mb, nb;
      tile_coords(first_tile, p, mb, nb);
      const int m_cta = mb * C::TILE_M;
      const int n0 = nb * C::BN;
      const uint32_t part_s = ptx::smem_u32(smem + C::OFF_A);
      const bool ok = __all_sync(0xFFFFFFFFu, first_tile < num_tiles &&
                                                  ptx::mbar_wait<false>(&tfull_bar[0], 0, abort_flag,
                                                                        p.timeout_ns));
      if (ok && m_cta + ew * 32 < p.m) {
        ptx::tc_fence_after_sync();
        const uint32_t t_row = tmem_base + (uint32_t(ew * 32) << 16);
        const int row = ew * 32 + lane;
#pragma unroll
        for (int g = 0; g < C::BN / 64; ++g) {  // 64 columns per tcgen05.wait::ld
          uint32_t v[64];
          ptx::tmem_ld_32x32b_x32(t_row + g * 64, *reinterpret_cast<uint32_t(*)[32]>(v));
          ptx::tmem_ld_32x32b_x32(t_row + g * 64 + 32, *reinterpret_cast<uint32_t(*)[32]>(v + 32));
          ptx::tmem_wait_ld();
          if (m_cta + row < p.m) {
            const uint32_t dst_s = part_s + uint32_t((row * C::PART_STRIDE + g * 64) * 4);
#pragma unroll
            for (int k = 0; k < 16; ++k)
              ptx::st_shared_v4(dst_s + 16 * k,
                                make_uint4(v[4 * k], v[4 * k + 1], v[4 * k + 2], v[4 * k + 3]));
          }
        }
      }
      ptx::cluster_sync();
      // Every load and MMA of the cluster is over: the next kernel on the stream may launch (it
      // still waits for this grid's completion before reading memory).
      if (ew == 0 && lane == 0) ptx::griddep_launch_dependents();
      if (ok && !*abort_flag) {
        constexpr int kCols = C::BN / kSplit;
        constexpr int kQuads = kCols / 4;
        const int rows = min(kRowsPerCta, p.m - m_cta);
        const int tasks = rows * kQuads;
        constexpr int kStride = kNumEpiWarps * 32;
        // Two tasks per iteration, all 2 * KSPLIT cluster loads issued before the first add.
        for (int task = ew * 32 + lane; task < tasks; task += 2 * kStride) {
          uint4 part[2][kSplit];
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            const int tk = min(task + h * kStride, tasks - 1);
            const uint32_t src = part_s + uint32_t(((tk / kQuads) * C::PART_STRIDE +
                                                    split * kCols + (tk % kQuads) * 4) * 4);
#pragma unroll
            for (int t = 0; t < kSplit; ++t)
              part[h][t] = ptx::ld_dsmem_v4(ptx::map_addr_to_cta(src, uint32_t(t)));
          }
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            const int tk = task + h * kStride;
            const int col = split * kCols + (tk % kQuads) * 4;
            // N % 8 == 0: a quad lies wholly inside or outside D
            if (tk >= tasks || n0 + col >= p.n) continue;
            float s0 = __uint_as_float(part[h][0].x), s1 = __uint_as_float(part[h][0].y);
            float s2 = __uint_as_float(part[h][0].z), s3 = __uint_as_float(part[h][0].w);
#pragma unroll
            for (int t = 1; t < kSplit; ++t) {
              s0 = __fadd_rn(s0, __uint_as_float(part[h][t].x));
              s1 = __fadd_rn(s1, __uint_as_float(part[h][t].y));
              s2 = __fadd_rn(s2, __uint_as_float(part[h][t].z));
              s3 = __fadd_rn(s3, __uint_as_float(part[h][t].w));
            }
            const uint2 v =
                make_uint2(ptx::scaled_f32x2_to_bf16x2(__float_as_uint(s0), __float_as_uint(s1), alpha2),
                           ptx::scaled_f32x2_to_bf16x2(__float_as_uint(s2), __float_as_uint(s3), alpha2));
            const int64_t off = int64_t(m_cta + tk / kQuads) * p.ldd + n0 + col;
            // all-gather form: the same 8 bytes into every rank's D, local first, then the peers'
            // over NVLink (a warp's lanes write consecutive quads of a row)
#pragma unroll 1
            for (int i = 0; i < (NDST == 1 ? 1 : p.ndst); ++i)
              *reinterpret_cast<uint2*>(p.dsts[i] + off) = v;
          }
        }
        // stores into other GPUs' memory are complete and visible system-wide before the kernel
        // ends (the caller orders the ranks' reads after every rank's kernel)
        if constexpr (NDST > 1) __threadfence_system();
      }
    } else {
    int acc = 0;
    uint32_t acc_phase = 0;
    for (int tile = first_tile; tile < num_tiles; tile += tile_step) {
      int mb, nb;
      tile_coords(tile, p, mb, nb);
      const int m_cta = mb * C::TILE_M + int(rank) * kRowsPerCta;
      const int n0 = nb * C::BN;
      const bool ok = ptx::mbar_wait<kPair>(&tfull_bar[acc], acc_phase, abort_flag, p.timeout_ns);
      if (!__all_sync(0xFFFFFFFFu, ok)) break;
      // Single-CTA bf16 form: once the CTA's last accumulator is complete its loads and MMAs are
      // over, so the next kernel on the stream may launch now (onto SMs as they free up); it
      // still waits for this grid's completion before reading memory. Measured on decode
      // shapes, per call: 1.2-1.6 us for M = 16 and 32 (direct stores), 0.1-1.1 us for
      // M = 64 and 128 (ring-staged TMA stores).
      if constexpr (kRingStage)
        if (ew == 0 && lane == 0 && tile + tile_step >= num_tiles)
          ptx::griddep_launch_dependents();
      ptx::tc_fence_after_sync();
      const uint32_t t_row = tmem_base + (uint32_t(ew * 32) << 16) + uint32_t(acc * C::BN);
      // Drain this thread's accumulator row into registers as bf16 pairs, 64 columns per
      // tcgen05.wait::ld, then hand TMEM back to the MMA warp at once: the next tile's MMAs
      // overlap the shared-memory staging and TMA stores below.
      uint32_t pk[C::BN / 2];
#pragma unroll
      for (int g = 0; g < C::BN / 64; ++g) {
        uint32_t r0[32], r1[32];
        ptx::tmem_ld_32x32b_x32(t_row + g * 64, r0);
        ptx::tmem_ld_32x32b_x32(t_row + g * 64 + 32, r1);
        ptx::tmem_wait_ld();
#pragma unroll
        for (int i = 0; i < 16; ++i) {  // acc * (1/scale), two columns per multiply
          pk[g * 32 + i] = ptx::scaled_f32x2_to_bf16x2(r0[2 * i], r0[2 * i + 1], alpha2);
          pk[g * 32 + 16 + i] = ptx::scaled_f32x2_to_bf16x2(r1[2 * i], r1[2 * i + 1], alpha2);
        }
      }
      if constexpr (C::BN == 32) {  // one 32-column chunk
        uint32_t r0[32];
        ptx::tmem_ld_32x32b_x32(t_row, r0);
        ptx::tmem_wait_ld();
#pragma unroll
        for (int i = 0; i < 16; ++i)
          pk[i] = ptx::scaled_f32x2_to_bf16x2(r0[2 * i], r0[2 * i + 1], alpha2);
      }
      ptx::tc_fence_before_sync();
      __syncwarp();
      if (lane == 0) {
        if constexpr (kPair) ptx::mbar_arrive_cta(&tempty_bar[acc], 0);
        else ptx::mbar_arrive(&tempty_bar[acc]);
      }
      if constexpr (kRingStage) {
        if (p.m <= 32) {
          // At most 32 rows (one warp's worth): each thread stores its row straight from
          // registers, 16 bytes at a time, and the CTA can exit as soon as the stores are issued
          // (the grid's completion covers them) instead of waiting for TMA stores to read
          // shared memory. N % 8 == 0, so a 16-byte chunk lies wholly inside or outside D.
          const int r = m_cta + ew * 32 + lane;
          if (r < p.m) {
            uint16_t* drow = p.d + int64_t(r) * p.ldd + n0;
#pragma unroll
            for (int k = 0; k < C::BN / 8; ++k)
              if (n0 + 8 * k < p.n)
                ptx::st_global_v4(drow + 8 * k, make_uint4(pk[4 * k], pk[4 * k + 1],
                                                           pk[4 * k + 2], pk[4 * k + 3]));
          }
          if (++acc == C::ACC_STAGES) { acc = 0; acc_phase ^= 1; }
          continue;
        }
      }
      if (lane == 0) ptx::bulk_wait_group_read<0>();  // the previous tile's stores have read
      if constexpr (MODE == kEpiQuant) {
        // Codes: 128 bytes of this row per tile, staged EPI_ROW_BYTES at a time (each 16-byte
        // chunk = two 16-column blocks); the row's 16 scale bytes go straight to sf_out.
        const float s_out = __ldg(p.out_scale_ptr);
        const float* qtab = reinterpret_cast<const float*>(smem + C::OFF_QTAB);
        constexpr int kColsPerChunk = C::EPI_ROW_BYTES * 2;
        uint32_t sfw[4] = {0u, 0u, 0u, 0u};
#pragma unroll
        for (int c = 0; c < C::BN / kColsPerChunk; ++c) {
          if (m_cta + ew * 32 >= p.m || n0 + c * kColsPerChunk >= p.n) break;
          if (c >= 1 && lane == 0) ptx::bulk_wait_group_read<0>();
          __syncwarp();
          const uint32_t row = buf_s + uint32_t(lane) * C::EPI_ROW_BYTES;
#pragma unroll
          for (int k = 0; k < C::EPI_ROW_BYTES / 16; ++k) {
            const int blk = c * (kColsPerChunk / 16) + 2 * k;  // first of the two blocks
            uint32_t lo0, hi0, lo1, hi1;
            const int j = blk * 8;
            const uint8_t s0 = bq::quantize_block16_tab(pk[j], pk[j + 1], pk[j + 2], pk[j + 3],
                                                        pk[j + 4], pk[j + 5], pk[j + 6],
                                                        pk[j + 7], s_out, qtab, lo0, hi0);
            const uint8_t s1 = bq::quantize_block16_tab(pk[j + 8], pk[j + 9], pk[j + 10],
                                                        pk[j + 11], pk[j + 12], pk[j + 13],
                                                        pk[j + 14], pk[j + 15], s_out, qtab, lo1,
                                                        hi1);
            sfw[blk / 4] |= (uint32_t(s0) | (uint32_t(s1) << 8)) << (8 * (blk % 4));
            ptx::st_shared_v4(row + ((uint32_t(k) ^ swz) << 4), make_uint4(lo0, hi0, lo1, hi1));
          }
          ptx::fence_proxy_async_smem();
          __syncwarp();
          if (lane == 0) {
            ptx::tma_store_2d(&dst.map[0], buf, (n0 + c * kColsPerChunk) / 2, m_cta + ew * 32);
            ptx::bulk_commit_group();
          }
        }
        const int r = m_cta + ew * 32 + lane;
        const int nblk = min(16, (p.n - n0) / 16);  // scale bytes of this row inside D
        if (r < p.m && nblk > 0) {
          uint8_t* dst_sf = p.sf_out + int64_t(r) * p.sf_pitch + n0 / 16;
          if (nblk == 16 && (reinterpret_cast<uintptr_t>(dst_sf) & 15) == 0) {
            *reinterpret_cast<uint4*>(dst_sf) = make_uint4(sfw[0], sfw[1], sfw[2], sfw[3]);
          } else {
            for (int i = 0; i < nblk; ++i) dst_sf[i] = uint8_t(sfw[i / 4] >> (8 * (i % 4)));
          }
        }
      } else {
      int out_c0 = n0, out_w = p.n;  // output columns of this tile, output width
      constexpr int kOutCols = MODE == kEpiSwiglu ? C::BN / 2 : C::BN;
      if constexpr (MODE == kEpiSwiglu) {
#pragma unroll
        for (int j = 0; j < C::BN / 4; ++j) pk[j] = swiglu_bf16x2(pk[j], pk[j + C::BN / 4]);
        out_c0 = n0 / 2;
        out_w = p.n / 2;
      }
      // The CTA's last tile in the single-CTA bf16 form: the A/B ring is idle (this accumulator's
      // MMAs, which the epilogue waited for, consumed every fill the producer issued), so each
      // warp stages all its boxes there and issues their stores back to back instead of waiting
      // for each box's shared-memory read before refilling its one staging buffer.
      const bool ring = kRingStage && tile + tile_step >= num_tiles;
      const uint32_t ring_s = ptx::smem_u32(smem + C::OFF_A) +
                              uint32_t(ew * (kOutCols / C::EPI_COLS) * C::EPI_BUF_BYTES);
#pragma unroll
      for (int c = 0; c < kOutCols / C::EPI_COLS; ++c) {
        // Boxes entirely outside D (ragged M or N) end the loop — the issued store groups stay a
        // prefix, which the buffer-reuse wait below counts on; boxes that start inside D are
        // clipped by the TMA unit.
        if (m_cta + ew * 32 >= p.m || out_c0 + c * C::EPI_COLS >= out_w) break;
        const int b = c % C::EPI_BUFS;
        if (!ring && c >= C::EPI_BUFS && lane == 0)
          ptx::bulk_wait_group_read<C::EPI_BUFS - 1>();  // buffer b's previous store has read it
        __syncwarp();
        const uint32_t box_s = ring ? ring_s + uint32_t(c * C::EPI_BUF_BYTES)
                                    : buf_s + uint32_t(b * C::EPI_BUF_BYTES);
        const uint32_t row = box_s + uint32_t(lane) * C::EPI_ROW_BYTES;
        constexpr int kPairsPerChunk = C::EPI_COLS / 2;  // bf16 pairs of this row in the box
#pragma unroll
        for (int k = 0; k < C::EPI_COLS / 8; ++k) {
          const int j = c * kPairsPerChunk + 4 * k;
          ptx::st_shared_v4(row + ((uint32_t(k) ^ swz) << 4),
                            make_uint4(pk[j], pk[j + 1], pk[j + 2], pk[j + 3]));
        }
        ptx::fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) {
          // Peers' outputs are written over NVLink straight from this staging buffer; the tile
          // reaches every rank while the next tile's MMAs run.
          for (int i = 0; i < (NDST == 1 ? 1 : dst.count); ++i)
            ptx::tma_store_2d_s(&dst.map[i], box_s, out_c0 + c * C::EPI_COLS, m_cta + ew * 32);
          ptx::bulk_commit_group();
        }
      }
      }
      if (++acc == C::ACC_STAGES) { acc = 0; acc_phase ^= 1; }
    }
    if (lane == 0) {
      if constexpr (NDST > 1) {
        // Stores into other GPUs' memory must be complete and visible system-wide before the
        // kernel ends (the caller orders the ranks' reads after every rank's kernel).
        ptx::bulk_wait_group<0>();
        __threadfence_system();
      } else {
        // Local stores only need their shared-memory reads done before the CTA exits; the
        // grid's completion covers the global writes.
        ptx::bulk_wait_group_read<0>();
      }
    }
    }  // not split K
  }

  if constexpr (kSplit > 1) {
    // Split K: the epilogue warps pass the cluster's partials barrier inside their role; every
    // other warp passes it here, so that each thread of the cluster arrives exactly once.
    if (!(warp >= kFirstEpiWarp && warp < kFirstEpiWarp + kNumEpiWarps)) ptx::cluster_sync();
  }
  ptx::tc_fence_before_sync();
  // Pairs and split-K clusters: no CTA exits (releasing its shared memory) while a peer may
  // still read it.
  if constexpr (kPair || kSplit > 1) ptx::cluster_sync(); else __syncthreads();
  if (threadIdx.x == 0 && *abort_flag) atomicCAS(&g_nvfp4_device_status, 0, NVFP4_ERR_DEVICE_TIMEOUT);
  if (warp == kMmaWarp) {
    __syncwarp();
    ptx::tc_fence_after_sync();
    ptx::tmem_dealloc_g<kGroup>(tmem_base, C::TMEM_COLS);
  }
}

// K == 0: the sum is empty; D = bf16(0 / scale), as the reference epilogue would produce.
// D is rows x cols with a row pitch of ld elements.
__global__ void fill_empty_k_kernel(uint16_t* __restrict__ d, int64_t rows, int64_t cols,
                                    int64_t ld, const float* scale_ptr, float scale_val) {
  const float scale = scale_ptr ? __ldg(scale_ptr) : scale_val;
  const uint32_t v = ptx::f32x2_to_bf16x2(__fdiv_rn(0.0f, scale), 0.0f) & 0xFFFFu;
  const int64_t n = rows * cols;
  for (int64_t i = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; i < n;
       i += int64_t(gridDim.x) * blockDim.x)
    d[(i / cols) * ld + i % cols] = static_cast<uint16_t>(v);
}

// Self-test of the bounded wait: nothing ever arrives on this barrier.
__global__ void wait_timeout_selftest_kernel(uint64_t timeout_ns) {
  __shared__ uint64_t bar;
  __shared__ int abort_flag;
  if (threadIdx.x == 0) {
    ptx::mbar_init(&bar, 1);
    abort_flag = 0;
    ptx::fence_mbar_init();
  }
  __syncthreads();
  const bool ok = ptx::mbar_wait(&bar, 0, &abort_flag, timeout_ns);
  if (!__all_sync(0xFFFFFFFFu, ok) && threadIdx.x == 0)
    atomicCAS(&g_nvfp4_device_status, 0, NVFP4_ERR_DEVICE_TIMEOUT);
}

// ------------------------------------------------------------------------------------------
// Host side
// ------------------------------------------------------------------------------------------
typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                  const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                  const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                  CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = []() -> EncodeTiledFn {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &ptr, 12000, cudaEnableDefault,
                                         &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess)
      return nullptr;
    return reinterpret_cast<EncodeTiledFn>(ptr);
  }();
  return fn;
}

bool make_map_2d(CUtensorMap* m, CUtensorMapDataType dt, const void* base, uint64_t inner,
                 uint64_t outer, uint64_t row_bytes, uint32_t box_inner, uint32_t box_outer,
                 CUtensorMapSwizzle swz) {
  EncodeTiledFn enc = encode_fn();
  if (!enc) return false;
  cuuint64_t dims[2] = {inner, outer};
  cuuint64_t strides[1] = {row_bytes};
  cuuint32_t box[2] = {box_inner, box_outer};
  cuuint32_t estr[2] = {1, 1};
  return enc(m, dt, 2, const_cast<void*>(base), dims, strides, box, estr,
             CU_TENSOR_MAP_INTERLEAVE_NONE, swz, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
             CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

constexpr int kMaxDevices = 64;

// Per device, once: raise the dynamic shared-memory limit and find how many CTAs (single) or
// CTA pairs (clusters of 2) can be resident at once — the persistent grid size.
template <class C, int NDST, int MODE>
int resident_units(int dev) {
  static std::once_flag flags[kMaxDevices];
  static int units[kMaxDevices];
  static cudaError_t errs[kMaxDevices];
  if (dev < 0 || dev >= kMaxDevices) return -NVFP4_ERR_NO_DEVICE;
  std::call_once(flags[dev], [&] {
    errs[dev] = cudaFuncSetAttribute(gemm_kernel<C, NDST, MODE>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     C::SMEM_ALLOC);
    if (errs[dev] != cudaSuccess) return;
    int sms = 0;
    errs[dev] = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    if (errs[dev] != cudaSuccess) return;
    if constexpr (C::PAIR) {
      cudaLaunchConfig_t cfg = {};
      cudaLaunchAttribute attr[1];
      attr[0].id = cudaLaunchAttributeClusterDimension;
      attr[0].val.clusterDim.x = 2;
      attr[0].val.clusterDim.y = 1;
      attr[0].val.clusterDim.z = 1;
      cfg.gridDim = dim3(sms & ~1);
      cfg.blockDim = dim3(kThreads);
      cfg.dynamicSmemBytes = C::SMEM_ALLOC;
      cfg.attrs = attr;
      cfg.numAttrs = 1;
      int clusters = 0;
      errs[dev] = cudaOccupancyMaxActiveClusters(&clusters, gemm_kernel<C, NDST, MODE>, &cfg);
      units[dev] = clusters > 0 ? clusters : sms / 2;
    } else {
      units[dev] = sms;
    }
  });
  if (errs[dev] != cudaSuccess) return -NVFP4_ERR_CUDA;
  return units[dev];
}

// 128 x 256 tiles, one CTA: 4-stage A/B ring, scale factors one k-block per shared-memory slot
// (4 slots).
using CfgSingle = Cfg<256, 4, 1, false, 1, 4>;
// 256 x 256 tiles, CTA pair: 5-stage A/B ring per CTA (160 KiB), scale factors four k-blocks
// per shared-memory slot (64-byte rows, 2 slots), one 32 x 64 staging box per epilogue warp;
// tensor memory 256 + 5 x 48 columns.
using CfgPair = Cfg<256, 5, 1, true, 4, 2, 64, 1>;
// Narrower single-CTA tiles for N too small to give half the SMs a 256-column tile (decode
// shapes sharded along N: 28672 / 8 ranks = 14 tiles). More, narrower tiles put more SMs on the
// weight stream; the ring is deeper (A/B stages are smaller) to keep enough bytes in flight per
// SM. Each output element is still one chain of MMAs over K in the same order.
using CfgSingle128 = Cfg<128, 6, 1, false, 1, 4>;
using CfgSingle64 = Cfg<64, 8, 1, false, 1, 4>;
using CfgSingle32 = Cfg<32, 10, 1, false, 1, 4>;
// K split over a cluster of KSPLIT CTAs (decode shapes whose 256-column tiles fill less than
// half the SMs, K a multiple of KSPLIT k-blocks): 128 x 128 tiles over 4 or 2 CTAs, 128 x 256
// tiles over 4. The narrower tile halves the partials each CTA exchanges in the cluster sum.
using CfgSplit4N128 = Cfg<128, 6, 1, false, 1, 4, 32, 1, 4>;
using CfgSplit2N128 = Cfg<128, 6, 1, false, 1, 4, 32, 1, 2>;
using CfgSplit4 = Cfg<256, 4, 1, false, 1, 4, 32, 1, 4>;

// D of this launch: `count` destinations, each [M, N] with its own base and row pitch.
struct DstDesc {
  void* base[kMaxRanks];
  uint64_t row_bytes;
  int count;
};

// Quantized output of a launch (kEpiQuant): per-tensor scale, scale-byte destination, pitch.
struct QOutDesc {
  const float* out_scale = nullptr;
  uint8_t* sf = nullptr;
  int64_t sf_pitch = 0;
};

template <class C, int NDST, int MODE = kEpiBf16>
int launch(const void* A, const void* B, const void* A_sf, const void* B_sf,
           const float* scale_ptr, float scale_val, const DstDesc& dd, int64_t M, int64_t N,
           int64_t K, cudaStream_t stream, const QOutDesc& qd = QOutDesc()) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return NVFP4_ERR_NO_DEVICE;
  const int units = resident_units<C, NDST, MODE>(dev);
  if (units <= 0) return units == 0 ? NVFP4_ERR_NO_DEVICE : -units;
  if (dd.count < 1 || dd.count > NDST) return NVFP4_ERR_INVALID_VALUE;
  if ((K / kBK) % C::KSPLIT != 0) return NVFP4_ERR_INVALID_VALUE;

  CUtensorMap tm_a, tm_b, tm_sfa, tm_sfb;
  DstMaps<NDST> dst;
  dst.count = dd.count;
  const uint64_t kb = uint64_t(K) / 2, ks = uint64_t(K) / 16;
  // Scale-factor rows of 16/32/64 bytes per slot; the wider ones swizzled (see sf_chunk_addr).
  const CUtensorMapSwizzle sf_swizzle = C::SF_ROW_BYTES == 64   ? CU_TENSOR_MAP_SWIZZLE_64B
                                        : C::SF_ROW_BYTES == 32 ? CU_TENSOR_MAP_SWIZZLE_32B
                                                                : CU_TENSOR_MAP_SWIZZLE_NONE;
  // A single-CTA launch with M < kRowsPerCta (decode shapes) loads only the M rows of A and of
  // its scale factors that exist: a 128-row box would have the TMA unit fill the missing rows
  // with zeros on every fill. The MMA still runs 128 rows; the shared-memory rows past M hold
  // stale bytes, and their results (TMEM lanes past M) are never stored.
  const uint32_t a_rows = (!C::PAIR && M < kRowsPerCta) ? uint32_t(M) : uint32_t(kRowsPerCta);
  bool ok = make_map_2d(&tm_a, CU_TENSOR_MAP_DATA_TYPE_UINT8, A, kb, M, kb, kBKBytes, a_rows,
                        CU_TENSOR_MAP_SWIZZLE_128B) &&
            make_map_2d(&tm_b, CU_TENSOR_MAP_DATA_TYPE_UINT8, B, kb, N, kb, kBKBytes, C::B_ROWS,
                        CU_TENSOR_MAP_SWIZZLE_128B) &&
            make_map_2d(&tm_sfa, CU_TENSOR_MAP_DATA_TYPE_UINT8, A_sf, ks, M, ks, C::SF_ROW_BYTES,
                        a_rows, sf_swizzle) &&
            make_map_2d(&tm_sfb, CU_TENSOR_MAP_DATA_TYPE_UINT8, B_sf, ks, N, ks, C::SF_ROW_BYTES,
                        C::BN, sf_swizzle);
  const CUtensorMapSwizzle epi_swizzle =
      C::EPI_ROW_BYTES == 128 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_64B;
  for (int i = 0; ok && i < dd.count; ++i) {
    if constexpr (MODE == kEpiQuant)  // packed codes [M, N/2]
      ok = make_map_2d(&dst.map[i], CU_TENSOR_MAP_DATA_TYPE_UINT8, dd.base[i], uint64_t(N) / 2, M,
                       dd.row_bytes, C::EPI_ROW_BYTES, 32, epi_swizzle);
    else if constexpr (MODE == kEpiSwiglu)  // bf16 [M, N/2]
      ok = make_map_2d(&dst.map[i], CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, dd.base[i], uint64_t(N) / 2,
                       M, dd.row_bytes, C::EPI_COLS, 32, epi_swizzle);
    else
      ok = make_map_2d(&dst.map[i], CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, dd.base[i], N, M,
                       dd.row_bytes, C::EPI_COLS, 32, epi_swizzle);
  }
  if (!ok) return encode_fn() ? NVFP4_ERR_INVALID_VALUE : NVFP4_ERR_NO_DEVICE;

  Params p;
  p.scale_ptr = scale_ptr;
  p.scale_val = scale_val;
  p.m = int(M);
  p.n = int(N);
  p.m_blocks = int((M + C::TILE_M - 1) / C::TILE_M);
  p.n_blocks = int((N + C::BN - 1) / C::BN);
  p.k_stages = int(K / kBK);
  p.ab_tx = uint32_t(C::CTAS) * (a_rows * kBKBytes + C::B_STAGE);
  p.sf_tx = a_rows * C::SF_ROW_BYTES + C::SFB_SLOT;
  p.timeout_ns = 2000000000ull;  // 2 s per wait: far above any legitimate stall
  p.out_scale_ptr = qd.out_scale;
  p.sf_out = qd.sf;
  p.sf_pitch = qd.sf_pitch;
  p.d = static_cast<uint16_t*>(dd.base[0]);
  p.ldd = int64_t(dd.row_bytes / 2);
  static_assert(kMaxRanks <= 8, "Params::dsts");
  for (int i = 0; i < kMaxRanks; ++i)
    p.dsts[i] = i < dd.count ? static_cast<uint16_t*>(dd.base[i]) : nullptr;
  p.ndst = dd.count;
  const int64_t tiles = int64_t(p.m_blocks) * p.n_blocks;
  if (tiles > 0x7FFFFFFF / 16) return NVFP4_ERR_TOO_LARGE;
  // Split K: one cluster of KSPLIT CTAs per tile (clusters beyond what fits at once run as
  // earlier ones finish; each cluster only waits on its own CTAs). Otherwise a persistent grid.
  const int grid_units = C::KSPLIT > 1 ? int(tiles) : int(tiles < units ? tiles : units);
  cudaLaunchConfig_t cfg = {};
  cudaLaunchAttribute attr[2];
  int na = 0;
  if constexpr (C::PAIR || C::KSPLIT > 1) {
    attr[na].id = cudaLaunchAttributeClusterDimension;
    attr[na].val.clusterDim.x = C::PAIR ? 2 : C::KSPLIT;
    attr[na].val.clusterDim.y = 1;
    attr[na].val.clusterDim.z = 1;
    ++na;
  }
  if constexpr (NDST == 1) {
    // The grid may launch once the previous kernel's CTAs have exited and set up while that
    // kernel completes; the kernel waits for the completion before touching global memory.
    attr[na].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[na].val.programmaticStreamSerializationAllowed = 1;
    ++na;
  }
  cfg.gridDim = dim3(C::CTAS * C::KSPLIT * grid_units);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = C::SMEM_ALLOC;
  cfg.stream = stream;
  cfg.attrs = attr;
  cfg.numAttrs = na;
  return status_from_cuda(cudaLaunchKernelEx(&cfg, gemm_kernel<C, NDST, MODE>, tm_a, tm_b, tm_sfa,
                                             tm_sfb, dst, p));
}

// The kernel form of a plain bf16 GEMM, M x N x K (K > 0, a multiple of 256) on `sms` SMs.
enum class Plan { kPair, kSingle, kSingle128, kSingle64, kSingle32, kSplit4N128, kSplit2N128, kSplit4 };

Plan select_plan(int64_t M, int64_t N, int64_t K, int sms) {
  // A CTA pair covers 256 rows; for M <= 128 a single CTA per tile wastes no tensor work.
  if (M > kRowsPerCta) return Plan::kPair;
  const auto tiles = [N](int64_t bn) { return (N + bn - 1) / bn; };
  if (sms <= 0 || 2 * tiles(256) > sms) return Plan::kSingle;
  // 256-column tiles give less than half the SMs a tile. Split K when every tile's cluster fits
  // on the SMs at once (measured on 28672 / 8 and / 4 column shards of a 28672 x 8192 weight):
  // 128-column tiles over 4 CTAs where they fit; else, above 32 rows, 128-column tiles over 2;
  // else 256-column tiles over 4. Otherwise the widest single-CTA tile that still gives at least
  // half the SMs a tile.
  const int64_t kblocks = K / kBK;
  const auto fits = [&](int64_t bn, int64_t s) { return tiles(bn) * s <= sms && kblocks % s == 0; };
  if (fits(128, 4)) return Plan::kSplit4N128;
  if (M > 32 && fits(128, 2)) return Plan::kSplit2N128;
  if (fits(256, 4)) return Plan::kSplit4;
  if (2 * tiles(128) > sms) return Plan::kSingle128;
  if (2 * tiles(64) > sms) return Plan::kSingle64;
  return Plan::kSingle32;
}

int check_shape(int64_t M, int64_t N, int64_t K) {
  if (M < 0 || N < 0 || K < 0) return NVFP4_ERR_INVALID_VALUE;
  if (K % kBK != 0 || N % 8 != 0) return NVFP4_ERR_UNSUPPORTED_SHAPE;
  if (M > 0x7FFFFFFF || N > 0x7FFFFFFF || K > 0x7FFFFFFF) return NVFP4_ERR_TOO_LARGE;
  return NVFP4_OK;
}

int run(const void* A, const void* B, const void* A_sf, const void* B_sf, const float* scale_ptr,
        float scale_val, void* D, int64_t M, int64_t N, int64_t K, cudaStream_t stream) {
  if (const int st = check_shape(M, N, K); st != NVFP4_OK) return st;
  if (M == 0 || N == 0) return NVFP4_OK;
  if (!D) return NVFP4_ERR_INVALID_VALUE;
  if (!aligned_to(D, 16)) return NVFP4_ERR_MISALIGNED;
  if (K == 0) {
    fill_empty_k_kernel<<<148, 256, 0, stream>>>(static_cast<uint16_t*>(D), M, N, N, scale_ptr,
                                                 scale_val);
    return status_from_cuda(cudaGetLastError());
  }
  if (!A || !B || !A_sf || !B_sf) return NVFP4_ERR_INVALID_VALUE;
  if (!aligned_to(A, 16) || !aligned_to(B, 16) || !aligned_to(A_sf, 16) || !aligned_to(B_sf, 16))
    return NVFP4_ERR_MISALIGNED;
  DstDesc dd = {};
  dd.base[0] = D;
  dd.row_bytes = uint64_t(N) * 2;
  dd.count = 1;
  const int sms = M > kRowsPerCta ? 0 : current_device_sm_count(nullptr);
#define NVFP4_LAUNCH(CFG) launch<CFG, 1>(A, B, A_sf, B_sf, scale_ptr, scale_val, dd, M, N, K, stream)
  switch (select_plan(M, N, K, sms)) {
    case Plan::kPair: return NVFP4_LAUNCH(CfgPair);
    case Plan::kSplit4N128: return NVFP4_LAUNCH(CfgSplit4N128);
    case Plan::kSplit2N128: return NVFP4_LAUNCH(CfgSplit2N128);
    case Plan::kSplit4: return NVFP4_LAUNCH(CfgSplit4);
    case Plan::kSingle128: return NVFP4_LAUNCH(CfgSingle128);
    case Plan::kSingle64: return NVFP4_LAUNCH(CfgSingle64);
    case Plan::kSingle32: return NVFP4_LAUNCH(CfgSingle32);
    case Plan::kSingle: break;
  }
  return NVFP4_LAUNCH(CfgSingle);
#undef NVFP4_LAUNCH
}

// Column-parallel GEMM with the all-gather fused into the epilogue. Every rank holds the same
// A, its own column shard of B ([N_local, K/2]) and a full output D_r [M, world * N_local];
// `outputs[r]` is rank r's D_r as mapped in this process. This rank's tile results are stored
// into columns [rank * N_local, (rank + 1) * N_local) of every D_r.
int run_allgather(const void* A, const void* B, const void* A_sf, const void* B_sf,
                  const float* scale_ptr, float scale_val, void* const* outputs, int world,
                  int rank, int64_t M, int64_t N_local, int64_t K, cudaStream_t stream) {
  if (M < 0 || N_local < 0 || K < 0) return NVFP4_ERR_INVALID_VALUE;
  if (world < 1 || world > kMaxRanks || rank < 0 || rank >= world || !outputs)
    return NVFP4_ERR_INVALID_VALUE;
  if (K % kBK != 0 || N_local % 8 != 0) return NVFP4_ERR_UNSUPPORTED_SHAPE;
  if (M > 0x7FFFFFFF || K > 0x7FFFFFFF || N_local * world > 0x7FFFFFFF) return NVFP4_ERR_TOO_LARGE;
  if (M == 0 || N_local == 0) return NVFP4_OK;
  DstDesc dd = {};
  dd.row_bytes = uint64_t(N_local) * uint64_t(world) * 2;
  dd.count = world;
  for (int i = 0; i < world; ++i) {
    const int r = (rank + i) % world;  // local output first, then the next ranks in turn
    if (!outputs[r]) return NVFP4_ERR_INVALID_VALUE;
    if (!aligned_to(outputs[r], 16)) return NVFP4_ERR_MISALIGNED;
    dd.base[i] = static_cast<uint8_t*>(outputs[r]) + uint64_t(rank) * uint64_t(N_local) * 2;
  }
  if (K == 0) {
    for (int i = 0; i < world; ++i) {
      fill_empty_k_kernel<<<148, 256, 0, stream>>>(static_cast<uint16_t*>(dd.base[i]), M,
                                                   N_local, int64_t(dd.row_bytes / 2), scale_ptr,
                                                   scale_val);
      const cudaError_t e = cudaGetLastError();
      if (e != cudaSuccess) return status_from_cuda(e);
    }
    return NVFP4_OK;
  }
  if (!A || !B || !A_sf || !B_sf) return NVFP4_ERR_INVALID_VALUE;
  if (!aligned_to(A, 16) || !aligned_to(B, 16) || !aligned_to(A_sf, 16) || !aligned_to(B_sf, 16))
    return NVFP4_ERR_MISALIGNED;
  // Decode shapes take the split-K forms of the plain GEMM (their epilogue stores each sum into
  // every rank's D); other shapes the 256-column tiles, whose epilogue TMA-stores each staged box.
  const int sms = M > kRowsPerCta ? 0 : current_device_sm_count(nullptr);
#define NVFP4_LAUNCH_AG(CFG) \
  launch<CFG, kMaxRanks>(A, B, A_sf, B_sf, scale_ptr, scale_val, dd, M, N_local, K, stream)
  switch (select_plan(M, N_local, K, sms)) {
    case Plan::kPair: return NVFP4_LAUNCH_AG(CfgPair);
    case Plan::kSplit4N128: return NVFP4_LAUNCH_AG(CfgSplit4N128);
    case Plan::kSplit2N128: return NVFP4_LAUNCH_AG(CfgSplit2N128);
    case Plan::kSplit4: return NVFP4_LAUNCH_AG(CfgSplit4);
    default: break;
  }
  return NVFP4_LAUNCH_AG(CfgSingle);
#undef NVFP4_LAUNCH_AG
}

// GEMM with the output quantized to NVFP4 in the epilogue: the bytes of
// quantize(bf16(A.B^T / scale), out_scale) without writing or re-reading bf16 D.
int run_quantized(const void* A, const void* B, const void* A_sf, const void* B_sf,
                  const float* scale_ptr, const float* out_scale, void* q_out, void* sf_out,
                  int64_t M, int64_t N, int64_t K, cudaStream_t stream) {
  if (M < 0 || N < 0 || K < 0) return NVFP4_ERR_INVALID_VALUE;
  // N % 32: the packed output's rows (N/2 bytes) must be a multiple of 16 bytes for TMA stores
  if (K % kBK != 0 || N % 32 != 0 || K == 0) return NVFP4_ERR_UNSUPPORTED_SHAPE;
  if (M > 0x7FFFFFFF || N > 0x7FFFFFFF || K > 0x7FFFFFFF) return NVFP4_ERR_TOO_LARGE;
  if (M == 0 || N == 0) return NVFP4_OK;
  if (!A || !B || !A_sf || !B_sf || !scale_ptr || !out_scale || !q_out || !sf_out)
    return NVFP4_ERR_INVALID_VALUE;
  if (!aligned_to(A, 16) || !aligned_to(B, 16) || !aligned_to(A_sf, 16) || !aligned_to(B_sf, 16) ||
      !aligned_to(q_out, 16))
    return NVFP4_ERR_MISALIGNED;
  DstDesc dd = {};
  dd.base[0] = q_out;
  dd.row_bytes = uint64_t(N) / 2;
  dd.count = 1;
  QOutDesc qd;
  qd.out_scale = out_scale;
  qd.sf = static_cast<uint8_t*>(sf_out);
  qd.sf_pitch = N / 16;
  if (M > kRowsPerCta)
    return launch<CfgPair, 1, kEpiQuant>(A, B, A_sf, B_sf, scale_ptr, 0.0f, dd, M, N, K, stream, qd);
  return launch<CfgSingle, 1, kEpiQuant>(A, B, A_sf, B_sf, scale_ptr, 0.0f, dd, M, N, K, stream,
                                         qd);
}

// Gate+up GEMM with SwiGLU in the epilogue: B holds 2*I rows interleaved in groups of 128 (for
// each t: gate rows 128t..128t+127, then up rows 128t..128t+127), so every 256-row tile of B
// carries the gate and up columns of the same 128 features; out [M, I] bf16 =
// bf16(silu(D_gate) * D_up) with D = bf16(A.B^T / scale) computed in fp32.
int run_swiglu(const void* A, const void* B, const void* A_sf, const void* B_sf,
               const float* scale_ptr, float scale_val, void* out, int64_t M, int64_t N,
               int64_t K, cudaStream_t stream) {
  if (M < 0 || N < 0 || K < 0) return NVFP4_ERR_INVALID_VALUE;
  if (K % kBK != 0 || N % 256 != 0 || K == 0) return NVFP4_ERR_UNSUPPORTED_SHAPE;
  if (M > 0x7FFFFFFF || N > 0x7FFFFFFF || K > 0x7FFFFFFF) return NVFP4_ERR_TOO_LARGE;
  if (M == 0 || N == 0) return NVFP4_OK;
  if (!A || !B || !A_sf || !B_sf || !out) return NVFP4_ERR_INVALID_VALUE;
  if (!aligned_to(A, 16) || !aligned_to(B, 16) || !aligned_to(A_sf, 16) || !aligned_to(B_sf, 16) ||
      !aligned_to(out, 16))
    return NVFP4_ERR_MISALIGNED;
  DstDesc dd = {};
  dd.base[0] = out;
  dd.row_bytes = uint64_t(N / 2) * 2;
  dd.count = 1;
  if (M > kRowsPerCta)
    return launch<CfgPair, 1, kEpiSwiglu>(A, B, A_sf, B_sf, scale_ptr, scale_val, dd, M, N, K,
                                          stream);
  return launch<CfgSingle, 1, kEpiSwiglu>(A, B, A_sf, B_sf, scale_ptr, scale_val, dd, M, N, K,
                                          stream);
}

}  // namespace gemm

int current_device_sm_count(int* device_out) {
  static int cache[gemm::kMaxDevices] = {0};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= gemm::kMaxDevices) return -1;
  if (device_out) *device_out = dev;
  if (cache[dev] == 0) {
    int n = 0;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) return -1;
    cache[dev] = n;
  }
  return cache[dev];
}

}  // namespace nvfp4

extern "C" {

int nvfp4_gemm(const void* A, const void* B, const void* A_sf, const void* B_sf, const float* scale,
               void* D, int64_t M, int64_t N, int64_t K, cudaStream_t stream) {
  if (!scale) return NVFP4_ERR_INVALID_VALUE;
  return nvfp4::gemm::run(A, B, A_sf, B_sf, scale, 0.0f, D, M, N, K, stream);
}

int nvfp4_gemm_host_scale(const void* A, const void* B, const void* A_sf, const void* B_sf,
                          float scale, void* D, int64_t M, int64_t N, int64_t K,
                          cudaStream_t stream) {
  return nvfp4::gemm::run(A, B, A_sf, B_sf, nullptr, scale, D, M, N, K, stream);
}

int nvfp4_gemm_plan(int64_t M, int64_t N, int64_t K, int sms, int* tile_m, int* tile_n,
                    int* k_split) {
  using nvfp4::gemm::Plan;
  if (!tile_m || !tile_n || !k_split || K == 0) return NVFP4_ERR_INVALID_VALUE;
  if (const int st = nvfp4::gemm::check_shape(M, N, K); st != NVFP4_OK) return st;
  if (sms <= 0) {
    sms = nvfp4::current_device_sm_count(nullptr);
    if (sms <= 0) return NVFP4_ERR_NO_DEVICE;
  }
  int tm = 128, tn = 256, ks = 1;
  switch (nvfp4::gemm::select_plan(M, N, K, sms)) {
    case Plan::kPair: tm = 256; break;
    case Plan::kSingle: break;
    case Plan::kSingle128: tn = 128; break;
    case Plan::kSingle64: tn = 64; break;
    case Plan::kSingle32: tn = 32; break;
    case Plan::kSplit4N128: tn = 128; ks = 4; break;
    case Plan::kSplit2N128: tn = 128; ks = 2; break;
    case Plan::kSplit4: ks = 4; break;
  }
  *tile_m = tm;
  *tile_n = tn;
  *k_split = ks;
  return NVFP4_OK;
}

int nvfp4_gemm_quantized(const void* A, const void* B, const void* A_sf, const void* B_sf,
                         const float* scale, const float* out_scale, void* q_out, void* sf_out,
                         int64_t M, int64_t N, int64_t K, cudaStream_t stream) {
  return nvfp4::gemm::run_quantized(A, B, A_sf, B_sf, scale, out_scale, q_out, sf_out, M, N, K,
                                    stream);
}

int nvfp4_gemm_swiglu(const void* A, const void* B_gate_up, const void* A_sf,
                      const void* B_gate_up_sf, const float* scale, void* out, int64_t M,
                      int64_t N, int64_t K, cudaStream_t stream) {
  if (!scale) return NVFP4_ERR_INVALID_VALUE;
  return nvfp4::gemm::run_swiglu(A, B_gate_up, A_sf, B_gate_up_sf, scale, 0.0f, out, M, N, K,
                                 stream);
}

int nvfp4_gemm_allgather(const void* A, const void* B_shard, const void* A_sf,
                         const void* B_sf_shard, const float* scale, void* const* outputs,
                         int world, int rank, int64_t M, int64_t N_local, int64_t K,
                         cudaStream_t stream) {
  if (!scale) return NVFP4_ERR_INVALID_VALUE;
  return nvfp4::gemm::run_allgather(A, B_shard, A_sf, B_sf_shard, scale, 0.0f, outputs, world,
                                    rank, M, N_local, K, stream);
}

int nvfp4_device_status(int* status_out, cudaStream_t stream) {
  if (!status_out) return NVFP4_ERR_INVALID_VALUE;
  int v = 0;
  cudaError_t e = cudaMemcpyFromSymbolAsync(&v, g_nvfp4_device_status, sizeof(int), 0,
                                            cudaMemcpyDeviceToHost, stream);
  if (e == cudaSuccess) e = cudaStreamSynchronize(stream);
  if (e != cudaSuccess) return NVFP4_ERR_CUDA;
  *status_out = v;
  return NVFP4_OK;
}

int nvfp4_clear_device_status(cudaStream_t stream) {
  static const int zero = 0;
  cudaError_t e = cudaMemcpyToSymbolAsync(g_nvfp4_device_status, &zero, sizeof(int), 0,
                                          cudaMemcpyHostToDevice, stream);
  if (e == cudaSuccess) e = cudaStreamSynchronize(stream);
  return nvfp4::status_from_cuda(e);
}

int nvfp4_selftest_wait_timeout(uint64_t timeout_ns, cudaStream_t stream) {
  nvfp4::gemm::wait_timeout_selftest_kernel<<<1, 32, 0, stream>>>(timeout_ns);
  return nvfp4::status_from_cuda(cudaGetLastError());
}

const char* nvfp4_status_string(int status) {
  switch (status) {
    case NVFP4_OK: return "NVFP4_OK";
    case NVFP4_ERR_INVALID_VALUE: return "NVFP4_ERR_INVALID_VALUE";
    case NVFP4_ERR_UNSUPPORTED_SHAPE: return "NVFP4_ERR_UNSUPPORTED_SHAPE";
    case NVFP4_ERR_MISALIGNED: return "NVFP4_ERR_MISALIGNED";
    case NVFP4_ERR_CUDA: return "NVFP4_ERR_CUDA";
    case NVFP4_ERR_NO_DEVICE: return "NVFP4_ERR_NO_DEVICE";
    case NVFP4_ERR_DEVICE_TIMEOUT: return "NVFP4_ERR_DEVICE_TIMEOUT";
    case NVFP4_ERR_TOO_LARGE: return "NVFP4_ERR_TOO_LARGE";
    default: return "NVFP4_ERR_UNKNOWN";
  }
}

int nvfp4_version(void) { return 0x000100; }

}  // extern "C"
