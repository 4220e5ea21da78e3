// CTA-pair tcgen05 GEMM for sm_100a:  C[M,N] = A[M,K] * B[N,K]^T with 256 x 256 output tiles.
//
// Same job and epilogues as gemm.cu (one CTA, 128 x BN tiles), for the large block linears.
// A cluster of two CTAs on neighbouring SMs computes each 256 x 256 tile with
// tcgen05.mma.cta_group::2: the even CTA holds A rows 0-127 and B rows (output columns)
// 0-127 of every k-block, the odd CTA rows 128-255 of both, and each CTA's Tensor Memory
// receives its own 128 accumulator rows for all 256 columns.  Per SM and k-block that is
// 32 KB of operands for a 128 x 256 x K share of the tile instead of the 48 KB a one-CTA
// 128 x 256 tile loads, so six pipeline stages fit and the operand stream per flop is a third
// lower.
//
// Roles (both CTAs, 320 threads):
//   warp 0      TMA producer: this CTA's A and B halves of each k-block into its own ring; the
//               loads complete on the even CTA's `full` barrier (cta_group::2 loads).
//   warp 1      even CTA: the single MMA issuer for the pair (4 x K16 pair MMAs per k-block),
//               committing each stage to both CTAs' `empty` barriers and each finished tile to
//               both CTAs' `tfull`; both CTAs: Tensor Memory allocation / release for the pair.
//   warps 2..9  epilogue of this CTA's 128 rows (as in gemm.cu); releasing an accumulator
//               arrives on the even CTA's `tempty` (512 arrivals: both CTAs' epilogues).
// Every wait is bounded; on a timeout the CTA records a status code and unwinds.
#include "../../include/fastworld_b200.h"
#include "fw_gemm_epi.cuh"
#include "fw_internal.h"
#include "fw_ptx.cuh"

namespace fw {

namespace g2 {
constexpr int BM = 256, BN = 256, HALF = 128;
constexpr int A_BYTES = HALF * 128;          // 128 rows x 128 bytes of K (64 bf16 / 128 e4m3)
constexpr int B_BYTES = HALF * 128;
constexpr int STAGE = A_BYTES + B_BYTES;     // 32 KB per CTA
constexpr int STAGES = 6;
constexpr uint32_t TMEM_COLS = 512;          // two 256-column accumulators
constexpr int BAR_OFF = STAGES * STAGE;
constexpr int EPI_OFF = BAR_OFF + 1024;
constexpr int EPI_BOX = 32 * 32 * 4;
constexpr int SMEM = EPI_OFF + 8 * EPI_BOX + 1024;
}  // namespace g2

template <bool F8>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(320, 1)
    gemm2_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                 const __grid_constant__ CUtensorMap tmC, const GemmArgs args) {
  using namespace g2;
  constexpr int KE = F8 ? 128 : 64;   // K elements per stage
  pdl_trigger();
  extern __shared__ uint8_t smem_raw[];
  const uint32_t pad = (1024u - (smem_u32(smem_raw) & 1023u)) & 1023u;
  uint8_t* smem = smem_raw + pad;
  uint8_t* sA = smem;
  uint8_t* sB = smem + STAGES * A_BYTES;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + BAR_OFF);
  uint64_t* empty = full + STAGES;
  uint64_t* tfull = empty + STAGES;
  uint64_t* tempty = tfull + 2;
  uint64_t* drain = tempty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();
  const bool leader = rank == 0;
  const int pair = blockIdx.x >> 1, npairs = gridDim.x >> 1;
  const int M = args.M, N = args.N, K = args.K;
  const int num_m = (M + BM - 1) / BM, num_n = (N + BN - 1) / BN;
  const int num_tiles = num_m * num_n, num_kb = (K + KE - 1) / KE;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(full + s, 1);
      mbar_init(empty + s, 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(tfull + a, 1);
      mbar_init(tempty + a, 512);
    }
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch(&tmA);
    tma_prefetch(&tmB);
  }
  if (warp == 1) {
    tmem_alloc_pair(tmem_slot, TMEM_COLS);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  cluster_sync();   // both CTAs' barriers initialised and the pair's Tensor Memory allocated
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  pdl_wait();

  if (warp == 0) {
    if (lane == 0) {
      const uint32_t full0 = mapa_cluster(full, 0);   // the even CTA's full[0]
      int stage = 0;
      uint32_t phase = 0, used = 0, last_par = 0;
      bool ok = true;
      for (int t = pair; t < num_tiles && ok; t += npairs) {
        const int mb = t % num_m, nb = t / num_m;
        for (int kb = 0; kb < num_kb; ++kb) {
          if (!mbar_wait(empty + stage, phase ^ 1u, abort_flag, args.status, DEV_TIMEOUT_PRODUCER)) {
            ok = false;
            break;
          }
          if (leader) mbar_arrive_expect_tx(full + stage, 2 * STAGE);
          const uint32_t fb = full0 + 8u * (uint32_t)stage;
          tma_load_2d_pair(sA + stage * A_BYTES, &tmA, fb, kb * KE, mb * BM + (int)rank * HALF);
          tma_load_2d_pair(sB + stage * B_BYTES, &tmB, fb, kb * KE, nb * BN + (int)rank * HALF);
          used |= 1u << stage;
          last_par = (last_par & ~(1u << stage)) | (phase << stage);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
      // bounded wait until the MMAs consumed every stage this thread filled (the loads of both
      // CTAs have then landed), so no copy into this CTA's memory is in flight at exit
      volatile int no_abort = 0;
      for (int s = 0; s < STAGES; ++s)
        if (used >> s & 1u) mbar_wait(empty + s, last_par >> s & 1u, &no_abort, args.status, DEV_TIMEOUT_DRAIN);
    }
  } else if (warp == 1) {
    if (lane == 0 && leader) {
      constexpr uint32_t idesc = F8 ? idesc_e4m3(BM, BN) : idesc_bf16(BM, BN, false, false);
      const uint32_t empty_peer = mapa_cluster(empty, 1), tfull_peer = mapa_cluster(tfull, 1);
      int stage = 0, acc = 0;
      uint32_t phase = 0, acc_phase = 0;
      bool ok = true;
      for (int t = pair; t < num_tiles && ok; t += npairs) {
        if (!mbar_wait(tempty + acc, acc_phase ^ 1u, abort_flag, args.status, DEV_TIMEOUT_MMA)) break;
        tc_fence_after();
        const uint32_t d = tmem_base + (uint32_t)(acc * BN);
        for (int kb = 0; kb < num_kb; ++kb) {
          if (!mbar_wait(full + stage, phase, abort_flag, args.status, DEV_TIMEOUT_MMA)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a0 = smem_u32(sA + stage * A_BYTES), b0 = smem_u32(sB + stage * B_BYTES);
#pragma unroll
          for (int k = 0; k < 4; ++k)
            if constexpr (F8)
              umma_f8_pair(d, sdesc_sw128(a0 + k * 32, 16, 1024), sdesc_sw128(b0 + k * 32, 16, 1024), idesc,
                           (kb | k) != 0);
            else
              umma_bf16_pair(d, sdesc_sw128(a0 + k * 32, 16, 1024), sdesc_sw128(b0 + k * 32, 16, 1024), idesc,
                             (kb | k) != 0);
          umma_commit_pair(smem_u32(empty + stage));                  // both CTAs may refill the stage
          umma_commit_pair(empty_peer + 8u * (uint32_t)stage);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (!ok) break;
        umma_commit_pair(smem_u32(tfull + acc));                      // both CTAs' epilogues may read
        umma_commit_pair(tfull_peer + 8u * (uint32_t)acc);
        acc ^= 1;
        if (acc == 0) acc_phase ^= 1u;
      }
      umma_commit_pair(smem_u32(drain));   // all pair MMAs complete before the Tensor Memory is released
      volatile int no_abort = 0;
      mbar_wait(drain, 0, &no_abort, args.status, DEV_TIMEOUT_DRAIN);
    }
  } else {
    // 8 epilogue warps per CTA: warp w reads lane quarter (w % 4) and column half (w - 2) / 4
    // of this CTA's 128 accumulator rows (4 chunks of 32 columns per thread).
    constexpr int NC = 4;
    const int q = warp & 3, h = (warp - 2) >> 2;
    const uint32_t tempty0 = mapa_cluster(tempty, 0);
    uint8_t* box = smem + EPI_OFF + (warp - 2) * EPI_BOX;
    int acc = 0;
    uint32_t acc_phase = 0;
    for (int t = pair; t < num_tiles; t += npairs) {
      const int mb = t % num_m, nb = t / num_m;
      const int row0 = mb * BM + (int)rank * HALF + q * 32;
      const int row = row0 + lane;
      const int colh = nb * BN + h * (BN / 2);
      if (args.epi.mode == EPI_RESID_F32 && row < M && colh < N) {
        const char* p = reinterpret_cast<const char*>(args.epi.resid + (size_t)row * args.epi.ld_resid + colh);
#pragma unroll
        for (int b = 0; b < BN * 2; b += 128) asm volatile("prefetch.global.L2 [%0];" ::"l"(p + b));
      }
      const bool ok = mbar_wait(tfull + acc, acc_phase, abort_flag, args.status, DEV_TIMEOUT_EPILOGUE);
      if (!__all_sync(0xffffffffu, ok)) break;
      tc_fence_after();
      const uint32_t tb = tmem_base + ((uint32_t)(q * 32) << 16) + (uint32_t)(acc * BN + h * (BN / 2));
      uint32_t r[NC][32];
#pragma unroll
      for (int c = 0; c < NC; ++c) tmem_ld32(tb + (uint32_t)(c * 32), r[c]);
      tmem_ld_wait();
      tc_fence_before();
      mbar_arrive_cluster(tempty0 + 8u * (uint32_t)acc);   // this CTA's half of the accumulator is free
      if (args.epi.mode == EPI_RESID_TMA) {
#pragma unroll
        for (int c = 0; c < NC; ++c) {
          const int col0 = colh + c * 32;
          if (col0 < N)
            epilogue_chunk_tma(args.epi, &tmC, min(row, M - 1), row0, col0, r[c], F8 ? args.sa : nullptr, args.sw,
                               box, lane);
        }
      } else if (row < M) {
#pragma unroll
        for (int c = 0; c < NC; ++c) {
          const int col0 = colh + c * 32;
          if (col0 < N) epilogue_chunk(args.epi, row, col0, r[c], F8 ? args.sa : nullptr, args.sw);
        }
      }
      acc ^= 1;
      if (acc == 0) acc_phase ^= 1u;
    }
    if (args.epi.mode == EPI_RESID_TMA && lane == 0) bulk_wait0();
  }
  tc_fence_before();
  __syncthreads();
  cluster_sync();   // neither CTA releases the pair's Tensor Memory or exits while the other uses it
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc_pair(tmem_base, TMEM_COLS);
  }
}

template <bool F8>
static int launch_pair(const CUtensorMap& tmA, const CUtensorMap& tmB, const CUtensorMap& tmC, const GemmArgs& a,
                       cudaStream_t s, int grid) {
  cudaError_t err = cudaFuncSetAttribute(gemm2_kernel<F8>, cudaFuncAttributeMaxDynamicSharedMemorySize, g2::SMEM);
  if (err != cudaSuccess) return FW_ECUDA;
  launch_k(gemm2_kernel<F8>, grid, 320, g2::SMEM, s, tmA, tmB, tmC, a);
  return cudaGetLastError() == cudaSuccess ? 0 : FW_ECUDA;
}

int gemm_pair_launch(const CUtensorMap& tmA, const CUtensorMap& tmB, const GemmArgs& a, cudaStream_t s,
                     const CUtensorMap* tmC) {
  int rc = gemm_check(a, g2::BN);
  if (rc) return rc;
  if (a.epi.mode == EPI_BF16_PUSH || a.groups != 1) return FW_EINVAL;   // one-CTA kernel only
  if (a.epi.mode == EPI_RESID_TMA && !tmC) return FW_EINVAL;
  const CUtensorMap& mc = tmC ? *tmC : tmA;
  const int tiles = ((a.M + g2::BM - 1) / g2::BM) * ((a.N + g2::BN - 1) / g2::BN);
  int pairs = num_sms() / 2;
  if (pairs > tiles) pairs = tiles;
  return a.sa ? launch_pair<true>(tmA, tmB, mc, a, s, 2 * pairs) : launch_pair<false>(tmA, tmB, mc, a, s, 2 * pairs);
}

}  // namespace fw
