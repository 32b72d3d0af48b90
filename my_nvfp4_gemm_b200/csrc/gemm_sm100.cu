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
//   * warp-specialised (320 threads per CTA):
//       warp 8  TMA producer: A/B tiles (128B-swizzled) and scale-factor tiles into a
//               STAGES-deep shared-memory ring, guarded by full and empty mbarriers;
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
constexpr int kProducerWarp = 8;          // TMA producer
constexpr int kMmaWarp = 9;               // MMA issuer, owns the TMEM allocation
constexpr int kThreads = 32 * 10;
constexpr int kEpiCols = 32;              // accumulator columns per epilogue store
constexpr int kEpiBufBytes = 32 * kEpiCols * 2;  // 32 rows x 32 bf16 per epilogue warp

template <int BN_, int STAGES_, int ACC_STAGES_, bool PAIR_>
struct Cfg {
  static constexpr int BN = BN_;
  static constexpr int STAGES = STAGES_;
  static constexpr int ACC_STAGES = ACC_STAGES_;
  static constexpr bool PAIR = PAIR_;
  static constexpr int CTAS = PAIR ? 2 : 1;
  static constexpr int TILE_M = kRowsPerCta * CTAS;        // output rows per tile
  static constexpr int B_ROWS = BN / CTAS;                 // B rows each CTA loads
  static_assert(BN % 128 == 0 && BN <= 256, "BN must be 128 or 256");

  static constexpr int A_STAGE = kRowsPerCta * kBKBytes;   // 16 KiB
  static constexpr int B_STAGE = B_ROWS * kBKBytes;
  static constexpr int SFA_STAGE = kRowsPerCta * kSfBytesPerRow;   // 2 KiB
  static constexpr int SFB_STAGE = BN * kSfBytesPerRow;    // every CTA holds all BN rows
  static constexpr uint32_t AB_TX = uint32_t(CTAS) * (A_STAGE + B_STAGE);  // pair total
  static constexpr uint32_t SF_TX = SFA_STAGE + SFB_STAGE;                 // per CTA

  static constexpr int OFF_A = 0;
  static constexpr int OFF_B = OFF_A + STAGES * A_STAGE;
  static constexpr int OFF_SFA = OFF_B + STAGES * B_STAGE;
  static constexpr int OFF_SFB = OFF_SFA + STAGES * SFA_STAGE;
  static constexpr int OFF_EPI = OFF_SFB + STAGES * SFB_STAGE;
  static constexpr int OFF_BAR = OFF_EPI + kNumEpiWarps * kEpiBufBytes;
  static constexpr int NUM_BARS = 4 * STAGES + 2 * ACC_STAGES + 1;
  static constexpr int OFF_MISC = OFF_BAR + NUM_BARS * 8;
  static constexpr int SMEM_BYTES = OFF_MISC + 16;
  static constexpr int SMEM_ALLOC = SMEM_BYTES + 1024;     // slack to align the base to 1 KiB
  static_assert(SMEM_ALLOC <= 232448, "shared memory budget exceeded");

  // Tensor memory columns: accumulators, then one scale-factor slot per pipeline stage, so the
  // factors of stage s+1 are written while the MMAs of stage s still read theirs. Within a slot:
  // B's factors for K-steps 0..3 (BN/32 columns each), then A's (4 columns each).
  static constexpr uint32_t SFB_COLS_PER_STEP = BN / 32;
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
  uint64_t timeout_ns;
};

// Scale-factor writer (one warp per TMEM lane quarter q). The block-scaled MMA of sub-partition
// q reads the scale factors of A row 32q+r from TMEM lane 32q+r, column sfa+q, and those of B
// row n from lane 32q+(n%32), column sfb+n/32 (B's factors are needed by every quarter). The
// warp reads its rows' row-major factors from the stage's shared-memory tile (16 bytes per row
// = K-steps 0..3) and writes its quarter of the stage's TMEM slot with tcgen05.st:
//   slot + j*(BN/32) + i   <- step-j word of B row 32i + lane     (BN/8 columns)
//   slot + BN/8 + 4j + k   <- step-j word of A row 32q + lane     (16 columns, k = 0..3)
template <class C>
__device__ __forceinline__ void write_sf_slot(uint32_t slot, uint32_t sfa_s, uint32_t sfb_s, int q,
                                              int lane) {
  constexpr int kChunksB = C::BN / 32;
  uint32_t vb[C::BN / 8];
#pragma unroll
  for (int i = 0; i < kChunksB; ++i) {
    const uint4 w = ptx::ld_shared_v4(sfb_s + uint32_t(32 * i + lane) * 16);
    vb[0 * kChunksB + i] = w.x;
    vb[1 * kChunksB + i] = w.y;
    vb[2 * kChunksB + i] = w.z;
    vb[3 * kChunksB + i] = w.w;
  }
  const uint4 a = ptx::ld_shared_v4(sfa_s + uint32_t(32 * q + lane) * 16);
  uint32_t va[16];
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    va[0 + k] = a.x;
    va[4 + k] = a.y;
    va[8 + k] = a.z;
    va[12 + k] = a.w;
  }
  if constexpr (C::BN == 256) {
    ptx::tmem_st_32x32b_x32(slot, vb);
  } else {
    ptx::tmem_st_32x32b_x16(slot, vb);
  }
  ptx::tmem_st_32x32b_x16(slot + C::BN / 8, va);
}

template <class C>
__global__ void __launch_bounds__(kThreads, 1)
gemm_kernel(const __grid_constant__ CUtensorMap tm_a, const __grid_constant__ CUtensorMap tm_b,
            const __grid_constant__ CUtensorMap tm_sfa, const __grid_constant__ CUtensorMap tm_sfb,
            const __grid_constant__ CUtensorMap tm_d, const Params p) {
  constexpr bool kPair = C::PAIR;
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
  uint64_t* full_bar = bars;                        // A/B landed (leader's counts the pair)
  uint64_t* sfload_bar = bars + C::STAGES;          // this CTA's scale-factor tiles landed
  uint64_t* sf_bar = bars + 2 * C::STAGES;          // scale factors in TMEM (leader's, all CTAs)
  uint64_t* empty_bar = bars + 3 * C::STAGES;       // MMA done with the stage -> producer
  uint64_t* tfull_bar = bars + 4 * C::STAGES;       // accumulator ready -> epilogue
  uint64_t* tempty_bar = tfull_bar + C::ACC_STAGES; // accumulator drained -> MMA (leader's)
  uint64_t* drain_bar = tempty_bar + C::ACC_STAGES; // MMA drain before TMEM free
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + C::OFF_MISC);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + C::OFF_MISC + 4);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t rank = kPair ? ptx::cluster_ctarank() : 0u;
  const int num_tiles = p.m_blocks * p.n_blocks;
  const int first_tile = kPair ? int(blockIdx.x >> 1) : int(blockIdx.x);
  const int tile_step = kPair ? int(gridDim.x >> 1) : int(gridDim.x);

  if (threadIdx.x == 0) {
    for (int i = 0; i < C::STAGES; ++i) {
      ptx::mbar_init(&full_bar[i], 1);
      ptx::mbar_init(&sfload_bar[i], 1);
      ptx::mbar_init(&sf_bar[i], kNumSfWarps * C::CTAS);
      ptx::mbar_init(&empty_bar[i], 1);
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
    ptx::tma_prefetch_desc(&tm_d);
  }
  if (warp == kMmaWarp) {
    ptx::tmem_alloc_g<kGroup>(tmem_slot, C::TMEM_COLS);
    ptx::tmem_relinquish_g<kGroup>();
  }
  ptx::tc_fence_before_sync();
  if constexpr (kPair) ptx::cluster_sync(); else __syncthreads();
  ptx::tc_fence_after_sync();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == kProducerWarp) {
    // ------------------------------------------------------------------ TMA producer
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      int64_t fills = 0;
      for (int tile = first_tile; tile < num_tiles; tile += tile_step) {
        const int m_cta = (tile % p.m_blocks) * C::TILE_M + int(rank) * kRowsPerCta;
        const int n0 = (tile / p.m_blocks) * C::BN;
        const int n_cta = n0 + int(rank) * C::B_ROWS;
        for (int kb = 0; kb < p.k_stages; ++kb) {
          if (!ptx::mbar_wait<kPair>(&empty_bar[stage], phase ^ 1, abort_flag, p.timeout_ns))
            goto producer_done;
          if (rank == 0) ptx::mbar_arrive_expect_tx(&full_bar[stage], C::AB_TX);
          if constexpr (kPair) {
            ptx::tma_load_2d_pair(sA + stage * C::A_STAGE, &tm_a, &full_bar[stage], kb * kBKBytes, m_cta);
            ptx::tma_load_2d_pair(sB + stage * C::B_STAGE, &tm_b, &full_bar[stage], kb * kBKBytes, n_cta);
          } else {
            ptx::tma_load_2d(sA + stage * C::A_STAGE, &tm_a, &full_bar[stage], kb * kBKBytes, m_cta);
            ptx::tma_load_2d(sB + stage * C::B_STAGE, &tm_b, &full_bar[stage], kb * kBKBytes, n_cta);
          }
          ptx::mbar_arrive_expect_tx(&sfload_bar[stage], C::SF_TX);
          ptx::tma_load_2d(sSFA + stage * C::SFA_STAGE, &tm_sfa, &sfload_bar[stage], kb * kSfBytesPerRow, m_cta);
          ptx::tma_load_2d(sSFB + stage * C::SFB_STAGE, &tm_sfb, &sfload_bar[stage], kb * kSfBytesPerRow, n0);
          ++fills;
          if (++stage == C::STAGES) { stage = 0; phase ^= 1; }
        }
      }
    producer_done:
      // Never leave a TMA write in flight into shared memory of an exiting CTA: wait (bounded,
      // ignoring the abort flag) until the most recent fill of every slot has landed. In a pair
      // the A/B bytes of both CTAs are counted on the leader's barriers; the follower waits a
      // fixed bounded time after an abort instead.
      {
        int no_abort = 0;
        const int64_t last = fills < C::STAGES ? fills : C::STAGES;
        for (int64_t i = 0; i < last; ++i) {
          const int64_t f = fills - 1 - i;
          const uint32_t par = uint32_t((f / C::STAGES) & 1);
          ptx::mbar_wait<kPair>(&sfload_bar[f % C::STAGES], par, &no_abort, p.timeout_ns);
          if (rank == 0)
            ptx::mbar_wait<kPair>(&full_bar[f % C::STAGES], par, &no_abort, p.timeout_ns);
        }
        if (kPair && rank != 0 && *abort_flag) {
          const uint64_t t0 = ptx::globaltimer_ns();
          while (ptx::globaltimer_ns() - t0 < 1000000ull) {
          }
        }
      }
    }
  } else if (warp == kMmaWarp) {
    // ------------------------------------------------------------------ MMA issuer
    if (lane == 0 && rank == 0) {
      constexpr uint32_t idesc = ptx::make_idesc_mxf4nvf4(C::TILE_M, C::BN);
      int stage = 0;
      uint32_t phase = 0;
      int acc = 0;
      uint32_t acc_phase = 0;
      for (int tile = first_tile; tile < num_tiles; tile += tile_step) {
        if (!ptx::mbar_wait<kPair>(&tempty_bar[acc], acc_phase ^ 1, abort_flag, p.timeout_ns))
          goto mma_done;
        ptx::tc_fence_after_sync();
        const uint32_t d_tmem = tmem_base + uint32_t(acc * C::BN);
        for (int kb = 0; kb < p.k_stages; ++kb) {
          if (!ptx::mbar_wait<kPair>(&sf_bar[stage], phase, abort_flag, p.timeout_ns)) goto mma_done;
          if (!ptx::mbar_wait<kPair>(&full_bar[stage], phase, abort_flag, p.timeout_ns)) goto mma_done;
          ptx::tc_fence_after_sync();
          const uint32_t t_sfb = tmem_base + C::COL_SF + uint32_t(stage) * C::SF_SLOT_COLS;
          const uint32_t t_sfa = t_sfb + C::BN / 8;
          const uint32_t a_s = ptx::smem_u32(sA + stage * C::A_STAGE);
          const uint32_t b_s = ptx::smem_u32(sB + stage * C::B_STAGE);
#pragma unroll
          for (int j = 0; j < kKSteps; ++j) {
            // K-step j starts 32 bytes further along the 128-byte swizzled rows.
            const uint64_t a_desc = ptx::make_smem_desc(a_s + j * 32, 0, 1024, ptx::kLayoutSW128);
            const uint64_t b_desc = ptx::make_smem_desc(b_s + j * 32, 0, 1024, ptx::kLayoutSW128);
            if constexpr (kPair)
              ptx::tc_mma_mxf4nvf4_pair(d_tmem, a_desc, b_desc, idesc, t_sfa + 4 * j,
                                        t_sfb + j * (C::BN / 32), (kb | j) != 0 ? 1u : 0u);
            else
              ptx::tc_mma_mxf4nvf4(d_tmem, a_desc, b_desc, idesc, t_sfa + 4 * j,
                                   t_sfb + j * (C::BN / 32), (kb | j) != 0 ? 1u : 0u);
          }
          // frees the stage's smem and TMEM scale slot (in both CTAs of a pair)
          if constexpr (kPair) ptx::tc_commit_pair(&empty_bar[stage], 0x3);
          else ptx::tc_commit(&empty_bar[stage]);
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
    // Stage s's TMEM slot is rewritten only after sfload[s] of its next fill, which the
    // producer issues after empty[s]: the MMAs that read the slot's previous contents are done.
    const int q = warp;
    const uint32_t lane_base = uint32_t(q * 32) << 16;
    int stage = 0;
    uint32_t phase = 0;
    for (int tile = first_tile; tile < num_tiles; tile += tile_step) {
      for (int kb = 0; kb < p.k_stages; ++kb) {
        const bool ok = ptx::mbar_wait<kPair>(&sfload_bar[stage], phase, abort_flag, p.timeout_ns);
        if (!__all_sync(0xFFFFFFFFu, ok)) goto sf_done;
        write_sf_slot<C>(tmem_base + lane_base + C::COL_SF + uint32_t(stage) * C::SF_SLOT_COLS,
                         ptx::smem_u32(sSFA + stage * C::SFA_STAGE),
                         ptx::smem_u32(sSFB + stage * C::SFB_STAGE), q, lane);
        ptx::tmem_wait_st();
        ptx::tc_fence_before_sync();
        __syncwarp();
        if (lane == 0) {
          if constexpr (kPair) ptx::mbar_arrive_cta(&sf_bar[stage], 0);
          else ptx::mbar_arrive(&sf_bar[stage]);
        }
        if (++stage == C::STAGES) { stage = 0; phase ^= 1; }
      }
    }
  sf_done:;
  } else if (warp >= kFirstEpiWarp && warp < kFirstEpiWarp + kNumEpiWarps) {
    // ------------------------------------------------------------------ epilogue
    const int ew = warp - kFirstEpiWarp;  // == warp % 4: TMEM lanes 32*ew .. 32*ew+31
    const float scale = p.scale_ptr ? __ldg(p.scale_ptr) : p.scale_val;
    const float alpha = __frcp_rn(scale);
    uint8_t* buf = sEPI + ew * kEpiBufBytes;
    const uint32_t buf_s = ptx::smem_u32(buf);
    const uint32_t swz = uint32_t((lane >> 1) & 3);  // 64-byte TMA swizzle of row `lane`
    int acc = 0;
    uint32_t acc_phase = 0;
    for (int tile = first_tile; tile < num_tiles; tile += tile_step) {
      const int m_cta = (tile % p.m_blocks) * C::TILE_M + int(rank) * kRowsPerCta;
      const int n0 = (tile / p.m_blocks) * C::BN;
      const bool ok = ptx::mbar_wait<kPair>(&tfull_bar[acc], acc_phase, abort_flag, p.timeout_ns);
      if (!__all_sync(0xFFFFFFFFu, ok)) break;
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
        for (int i = 0; i < 16; ++i) {
          pk[g * 32 + i] = ptx::f32x2_to_bf16x2(__uint_as_float(r0[2 * i]) * alpha,
                                                __uint_as_float(r0[2 * i + 1]) * alpha);
          pk[g * 32 + 16 + i] = ptx::f32x2_to_bf16x2(__uint_as_float(r1[2 * i]) * alpha,
                                                     __uint_as_float(r1[2 * i + 1]) * alpha);
        }
      }
      ptx::tc_fence_before_sync();
      __syncwarp();
      if (lane == 0) {
        if constexpr (kPair) ptx::mbar_arrive_cta(&tempty_bar[acc], 0);
        else ptx::mbar_arrive(&tempty_bar[acc]);
      }
#pragma unroll
      for (int c = 0; c < C::BN / kEpiCols; ++c) {
        if (lane == 0) ptx::bulk_wait_group_read<0>();  // previous store has read the buffer
        __syncwarp();
        const uint32_t row = buf_s + uint32_t(lane) * 64;
#pragma unroll
        for (int k = 0; k < 4; ++k)
          ptx::st_shared_v4(row + ((uint32_t(k) ^ swz) << 4),
                            make_uint4(pk[c * 16 + 4 * k], pk[c * 16 + 4 * k + 1],
                                       pk[c * 16 + 4 * k + 2], pk[c * 16 + 4 * k + 3]));
        ptx::fence_proxy_async_smem();
        __syncwarp();
        // Boxes that start inside D are clipped by the TMA unit; boxes entirely outside
        // (ragged M or N) are skipped.
        if (lane == 0 && m_cta + ew * 32 < p.m && n0 + c * kEpiCols < p.n) {
          ptx::tma_store_2d(&tm_d, buf, n0 + c * kEpiCols, m_cta + ew * 32);
          ptx::bulk_commit_group();
        }
      }
      if (++acc == C::ACC_STAGES) { acc = 0; acc_phase ^= 1; }
    }
    if (lane == 0) ptx::bulk_wait_group<0>();
  }

  ptx::tc_fence_before_sync();
  if constexpr (kPair) ptx::cluster_sync(); else __syncthreads();
  if (threadIdx.x == 0 && *abort_flag) atomicCAS(&g_nvfp4_device_status, 0, NVFP4_ERR_DEVICE_TIMEOUT);
  if (warp == kMmaWarp) {
    __syncwarp();
    ptx::tc_fence_after_sync();
    ptx::tmem_dealloc_g<kGroup>(tmem_base, C::TMEM_COLS);
  }
}

// K == 0: the sum is empty; D = bf16(0 / scale), as the reference epilogue would produce.
__global__ void fill_empty_k_kernel(uint16_t* __restrict__ d, int64_t n, const float* scale_ptr,
                                    float scale_val) {
  const float scale = scale_ptr ? __ldg(scale_ptr) : scale_val;
  const uint32_t v = ptx::f32x2_to_bf16x2(__fdiv_rn(0.0f, scale), 0.0f) & 0xFFFFu;
  for (int64_t i = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; i < n;
       i += int64_t(gridDim.x) * blockDim.x)
    d[i] = static_cast<uint16_t>(v);
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
template <class C>
int resident_units(int dev) {
  static std::once_flag flags[kMaxDevices];
  static int units[kMaxDevices];
  static cudaError_t errs[kMaxDevices];
  if (dev < 0 || dev >= kMaxDevices) return -NVFP4_ERR_NO_DEVICE;
  std::call_once(flags[dev], [&] {
    errs[dev] = cudaFuncSetAttribute(gemm_kernel<C>, cudaFuncAttributeMaxDynamicSharedMemorySize,
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
      errs[dev] = cudaOccupancyMaxActiveClusters(&clusters, gemm_kernel<C>, &cfg);
      units[dev] = clusters > 0 ? clusters : sms / 2;
    } else {
      units[dev] = sms;
    }
  });
  if (errs[dev] != cudaSuccess) return -NVFP4_ERR_CUDA;
  return units[dev];
}

using CfgSingle = Cfg<256, 4, 1, false>;  // 128 x 256 tiles, one CTA, 4-stage ring
using CfgPair = Cfg<256, 5, 1, true>;     // 256 x 256 tiles, CTA pair, 5-stage ring per CTA

template <class C>
int launch(const void* A, const void* B, const void* A_sf, const void* B_sf,
           const float* scale_ptr, float scale_val, void* D, int64_t M, int64_t N, int64_t K,
           cudaStream_t stream) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return NVFP4_ERR_NO_DEVICE;
  const int units = resident_units<C>(dev);
  if (units <= 0) return units == 0 ? NVFP4_ERR_NO_DEVICE : -units;

  CUtensorMap tm_a, tm_b, tm_sfa, tm_sfb, tm_d;
  const uint64_t kb = uint64_t(K) / 2, ks = uint64_t(K) / 16;
  bool ok = make_map_2d(&tm_a, CU_TENSOR_MAP_DATA_TYPE_UINT8, A, kb, M, kb, kBKBytes, kRowsPerCta,
                        CU_TENSOR_MAP_SWIZZLE_128B) &&
            make_map_2d(&tm_b, CU_TENSOR_MAP_DATA_TYPE_UINT8, B, kb, N, kb, kBKBytes, C::B_ROWS,
                        CU_TENSOR_MAP_SWIZZLE_128B) &&
            make_map_2d(&tm_sfa, CU_TENSOR_MAP_DATA_TYPE_UINT8, A_sf, ks, M, ks, kSfBytesPerRow,
                        kRowsPerCta, CU_TENSOR_MAP_SWIZZLE_NONE) &&
            make_map_2d(&tm_sfb, CU_TENSOR_MAP_DATA_TYPE_UINT8, B_sf, ks, N, ks, kSfBytesPerRow,
                        C::BN, CU_TENSOR_MAP_SWIZZLE_NONE) &&
            make_map_2d(&tm_d, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, D, N, M, uint64_t(N) * 2,
                        kEpiCols, 32, CU_TENSOR_MAP_SWIZZLE_64B);
  if (!ok) return encode_fn() ? NVFP4_ERR_INVALID_VALUE : NVFP4_ERR_NO_DEVICE;

  Params p;
  p.scale_ptr = scale_ptr;
  p.scale_val = scale_val;
  p.m = int(M);
  p.n = int(N);
  p.m_blocks = int((M + C::TILE_M - 1) / C::TILE_M);
  p.n_blocks = int((N + C::BN - 1) / C::BN);
  p.k_stages = int(K / kBK);
  p.timeout_ns = 2000000000ull;  // 2 s per wait: far above any legitimate stall
  const int64_t tiles = int64_t(p.m_blocks) * p.n_blocks;
  const int grid_units = int(tiles < units ? tiles : units);
  if constexpr (C::PAIR) {
    cudaLaunchConfig_t cfg = {};
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 2;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.gridDim = dim3(2 * grid_units);
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = C::SMEM_ALLOC;
    cfg.stream = stream;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return status_from_cuda(cudaLaunchKernelEx(&cfg, gemm_kernel<C>, tm_a, tm_b, tm_sfa, tm_sfb,
                                               tm_d, p));
  } else {
    gemm_kernel<C><<<grid_units, kThreads, C::SMEM_ALLOC, stream>>>(tm_a, tm_b, tm_sfa, tm_sfb,
                                                                   tm_d, p);
    return status_from_cuda(cudaGetLastError());
  }
}

int run(const void* A, const void* B, const void* A_sf, const void* B_sf, const float* scale_ptr,
        float scale_val, void* D, int64_t M, int64_t N, int64_t K, cudaStream_t stream) {
  if (M < 0 || N < 0 || K < 0) return NVFP4_ERR_INVALID_VALUE;
  if (K % kBK != 0 || N % 8 != 0) return NVFP4_ERR_UNSUPPORTED_SHAPE;
  if (M > 0x7FFFFFFF || N > 0x7FFFFFFF || K > 0x7FFFFFFF) return NVFP4_ERR_TOO_LARGE;
  if (M == 0 || N == 0) return NVFP4_OK;
  if (!D) return NVFP4_ERR_INVALID_VALUE;
  if (!aligned_to(D, 16)) return NVFP4_ERR_MISALIGNED;
  if (K == 0) {
    fill_empty_k_kernel<<<148, 256, 0, stream>>>(static_cast<uint16_t*>(D), M * N, scale_ptr,
                                                 scale_val);
    return status_from_cuda(cudaGetLastError());
  }
  if (!A || !B || !A_sf || !B_sf) return NVFP4_ERR_INVALID_VALUE;
  if (!aligned_to(A, 16) || !aligned_to(B, 16) || !aligned_to(A_sf, 16) || !aligned_to(B_sf, 16))
    return NVFP4_ERR_MISALIGNED;
  // A CTA pair covers 256 rows; for M <= 128 a single CTA per tile wastes no tensor work.
  if (M > kRowsPerCta)
    return launch<CfgPair>(A, B, A_sf, B_sf, scale_ptr, scale_val, D, M, N, K, stream);
  return launch<CfgSingle>(A, B, A_sf, B_sf, scale_ptr, scale_val, D, M, N, K, stream);
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
