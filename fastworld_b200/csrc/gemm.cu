// tcgen05 / TMEM GEMM for sm_100a:  C[M,N] = A[M,K] * B[N,K]^T  (bf16 in, fp32 accumulate).
//
// Replaces the cuBLAS Linear calls of the reference forward (fastworld/models/mg2/static.py:
// 198, 208-210, 219, 189-192, 224 and the action-module Linears 150-185).
//
// Design (one CTA per SM, persistent over output tiles):
//   warp 0      TMA producer: A tile [128 x 64] and B tile [BN x 64] per stage, 128-byte swizzle
//   warp 1      MMA issuer: 4 x tcgen05.mma (K = 16 each) per stage into a TMEM accumulator;
//               tcgen05.commit releases the smem stage and, per tile, signals the epilogue
//   warps 2..9  epilogue (thread = output row, two warps per TMEM lane quarter splitting the
//               tile's columns): all accumulator columns loaded with tcgen05.ld, TMEM released,
//               then fused bias / GELU / scales in registers; bf16 outputs go through a
//               per-warp shared-memory box so that each store instruction writes whole
//               128-byte rows, gated fp32 residual updates are TMA reduce-adds of such boxes
// The TMEM accumulator is double-buffered (two BN-column buffers; 256 columns apart for BN = 224)
// so the epilogue of tile i overlaps the main loop of tile i + 1.  BN is 64, 128, 224 or 256.  Tile order is M-fastest so consecutive CTAs share a weight
// tile in L2.  M, N and K tails are zero-filled by TMA and masked in the epilogue.
#include "../../include/fastworld_b200.h"
#include "fw_internal.h"
#include "fw_ptx.cuh"
#include "fw_gemm_epi.cuh"

namespace fw {

// BN = 224 (7 chunks of 32 columns) exists for the N = 1536 residual linears of 2640-row chunks:
// 21 x 7 = 147 tiles fill one wave of 148 SMs, where 256-wide tiles leave 22 SMs idle (126
// tiles).  Measured on B200 it gains only 1-2 % (2640 x 1536 x 1536: 15.35 -> 15.1 us; K = 8960:
// 62.1 -> 61.4 us): a tile's time barely follows its width, so the one-CTA main loop is not
// bound by the MMA's N (the extra SMs also re-read A: 7 column tiles instead of 6).  Its two
// accumulators sit 256 columns apart.
template <int BN>
struct GemmCfg {
  static constexpr int BM = 128, BK = 64;
  static constexpr int A_BYTES = BM * BK * 2;
  static constexpr int B_BYTES = BN * BK * 2;
  static constexpr int STAGE = A_BYTES + B_BYTES;
  static constexpr int STAGES = BN > 128 ? 4 : (BN == 128 ? 6 : 8);
  static constexpr int ACC = BN == 224 ? 256 : BN;   // TMEM column stride of the two accumulators
  static constexpr int TMEM_COLS = 2 * ACC;
  // epilogue: 32-column chunks per tile, and the first warp of a lane quarter takes the first H0
  static constexpr int NCT = BN / 32, H0 = (NCT + 1) / 2;
  // staging for EPI_RESID_TMA: one [32 rows x 32 fp32] 128-byte-swizzled box per epilogue warp,
  // 1024-aligned after the barrier block
  static constexpr int EPI_OFF = STAGES * STAGE + 1024;
  static constexpr int EPI_BOX = 32 * 32 * 4;
  static constexpr int SMEM = EPI_OFF + 8 * EPI_BOX + 1024;
};

// F8 = false: bf16 operands, kind::f16, 64 elements (128 bytes) of K per stage.
// F8 = true:  e4m3 operands, kind::f8f6f4, 128 elements (128 bytes) of K per stage; the same
//             128-byte-swizzled smem tiles and descriptors, 32 bytes of K per MMA instruction.
// Epilogue kinds, one kernel instantiation each, so that a launch carries only the code of its
// own epilogue (the in-chunk GEMMs are sensitive to instruction-cache misses):
enum : int {
  EK_BOX = 0,     // bf16 output modes, 64 columns per box stored with st.global (grouped launches)
  EK_RTMA = 1,    // EPI_RESID_TMA
  EK_RF32 = 2,    // EPI_RESID_F32
  EK_CHUNK = 3,   // EPI_F32, and the bf16 modes of 64-column tiles (epilogue_chunk)
  EK_PUSH = 4,    // EPI_BF16_PUSH
  EK_TMA = 8,     // bf16 output modes, 64 columns per box, TMA store; + the activation:
                  // EK_TMA + EPI_BF16, EK_TMA + EPI_GELU_BF16, EK_TMA + EPI_GELU_ERF_BF16
};

template <int BN, bool F8, int EK>
__global__ void __launch_bounds__(320, 1)
    gemm_bf16_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                     const __grid_constant__ CUtensorMap tmC, const __grid_constant__ CUtensorMap tmO0,
                     const __grid_constant__ CUtensorMap tmO1, const __grid_constant__ CUtensorMap tmO2,
                     const GemmArgs args) {
  using C = GemmCfg<BN>;
  constexpr int KE = F8 ? 128 : 64;   // K elements per stage
  pdl_trigger();
  extern __shared__ uint8_t smem_raw[];
  const uint32_t pad = (1024u - (smem_u32(smem_raw) & 1023u)) & 1023u;
  uint8_t* smem = smem_raw + pad;
  uint8_t* sA = smem;
  uint8_t* sB = smem + C::STAGES * C::A_BYTES;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + C::STAGES * C::STAGE);
  uint64_t* empty = full + C::STAGES;
  uint64_t* tfull = empty + C::STAGES;
  uint64_t* tempty = tfull + 2;
  uint64_t* drain = tempty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int M = args.M, N = args.N, K = args.K;
  const int num_m = (M + 127) / 128, num_n = (N + BN - 1) / BN;
  const int tpg = num_m * num_n;   // tiles per group
  const int num_tiles = tpg * args.groups, num_kb = (K + KE - 1) / KE;

  if (threadIdx.x == 0) {
    for (int s = 0; s < C::STAGES; ++s) {
      mbar_init(full + s, 1);
      mbar_init(empty + s, 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(tfull + a, 1);
      mbar_init(tempty + a, 256);
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
    tmem_alloc(tmem_slot, C::TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  // Weights that no kernel of the stream writes (args.b_static) are fetched for the CTA's first
  // tile before the dependency wait: their loads overlap the previous kernel's tail.  The stages
  // are still free at this point (first pass over the ring), so no empty-barrier wait is needed.
  const int pre = (args.b_static && args.groups == 1 && blockIdx.x < num_tiles)
                      ? (num_kb < C::STAGES ? num_kb : C::STAGES) : 0;
  if (warp == 0 && lane == 0 && pre > 0) {
    const int nb0 = (blockIdx.x % tpg) / num_m;
    for (int kb = 0; kb < pre; ++kb) {
      mbar_arrive_expect_tx(full + kb, C::STAGE);   // both halves of the stage: B now, A after the wait
      tma_load_2d(sB + kb * C::B_BYTES, &tmB, full + kb, kb * KE, nb0 * BN);
    }
  }
  pdl_wait();   // everything below reads or writes data of earlier kernels

  if (warp == 0) {
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0, used = 0, last_par = 0;
      bool ok = true;
      for (int t = blockIdx.x; t < num_tiles && ok; t += gridDim.x) {
        const int g = t / tpg, mb = (t - g * tpg) % num_m, nb = (t - g * tpg) / num_m;
        const CUtensorMap* mB = args.groups > 1 ? args.tmB_grp + g : &tmB;
        for (int kb = 0; kb < num_kb; ++kb) {
          if (t == (int)blockIdx.x && kb < pre) {   // B already in flight; only A is left
            tma_load_2d(sA + stage * C::A_BYTES, &tmA, full + stage, kb * KE, mb * 128);
          } else {
            if (!mbar_wait(empty + stage, phase ^ 1u, abort_flag, args.status, DEV_TIMEOUT_PRODUCER)) {
              ok = false;
              break;
            }
            mbar_arrive_expect_tx(full + stage, C::STAGE);
            tma_load_2d(sA + stage * C::A_BYTES, &tmA, full + stage, kb * KE, mb * 128);
            tma_load_2d(sB + stage * C::B_BYTES, mB, full + stage, kb * KE, nb * BN);
          }
          used |= 1u << stage;
          last_par = (last_par & ~(1u << stage)) | (phase << stage);
          if (++stage == C::STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
      // wait (bounded) for every load this thread issued to land before the CTA exits
      volatile int no_abort = 0;
      for (int s = 0; s < C::STAGES; ++s)
        if (used >> s & 1u) mbar_wait(full + s, last_par >> s & 1u, &no_abort, args.status, DEV_TIMEOUT_DRAIN);
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t idesc = F8 ? idesc_e4m3(128, BN) : idesc_bf16(128, BN, false, false);
      int stage = 0, acc = 0;
      uint32_t phase = 0, acc_phase = 0;
      bool ok = true;
      for (int t = blockIdx.x; t < num_tiles && ok; t += gridDim.x) {
        if (!mbar_wait(tempty + acc, acc_phase ^ 1u, abort_flag, args.status, DEV_TIMEOUT_MMA)) break;
        tc_fence_after();
        const uint32_t d = tmem_base + (uint32_t)(acc * C::ACC);
        for (int kb = 0; kb < num_kb; ++kb) {
          if (!mbar_wait(full + stage, phase, abort_flag, args.status, DEV_TIMEOUT_MMA)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a0 = smem_u32(sA + stage * C::A_BYTES), b0 = smem_u32(sB + stage * C::B_BYTES);
#pragma unroll
          for (int k = 0; k < 4; ++k)
            if constexpr (F8)
              umma_f8(d, sdesc_sw128(a0 + k * 32, 16, 1024), sdesc_sw128(b0 + k * 32, 16, 1024), idesc,
                      (kb | k) != 0);
            else
              umma_bf16(d, sdesc_sw128(a0 + k * 32, 16, 1024), sdesc_sw128(b0 + k * 32, 16, 1024), idesc,
                      (kb | k) != 0);
          umma_commit(empty + stage);
          if (++stage == C::STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (!ok) break;
        umma_commit(tfull + acc);
        acc ^= 1;
        if (acc == 0) acc_phase ^= 1u;
      }
      // all MMAs issued by this thread must complete before TMEM is released
      umma_commit(drain);
      volatile int no_abort = 0;
      mbar_wait(drain, 0, &no_abort, args.status, DEV_TIMEOUT_DRAIN);
    }
  } else {
    // 8 epilogue warps: warp w reads TMEM lane quarter (w % 4) and column half (w - 2) / 4 of
    // the tile (chunks [0, H0) or [H0, NCT) of 32 columns; the halves are equal except for
    // BN = 224, 4 + 3 chunks).  All of a thread's accumulator columns are loaded at once, the
    // TMEM buffer is released, and the bias / activation / residual math and the stores run from
    // registers.
    constexpr int NC = BN / 64;                   // 64-column boxes per thread are NC / 2
    static_assert(8 * C::H0 * C::EPI_BOX <= C::STAGES * C::STAGE, "last-tile staging must fit in the pipeline stages");
    const int q = warp & 3, h = (warp - 2) >> 2;
    const int c_lo = h ? C::H0 : 0, n_ch = h ? C::NCT - C::H0 : C::H0;
    int acc = 0;
    uint32_t acc_phase = 0;
    for (int t = blockIdx.x; t < num_tiles; t += gridDim.x) {
      const int g = t / tpg, mb = (t - g * tpg) % num_m, nb = (t - g * tpg) / num_m;
      const int row = mb * 128 + q * 32 + lane;
      const int colh = nb * BN + c_lo * 32;
      if (EK == EK_RF32 && row < M && colh < N) {   // warm L2 with this thread's residual row part
        const char* p = reinterpret_cast<const char*>(args.epi.resid + (size_t)row * args.epi.ld_resid + colh);
#pragma unroll
        for (int b = 0; b < n_ch * 128; b += 128) asm volatile("prefetch.global.L2 [%0];" ::"l"(p + b));
      }
      const bool ok = mbar_wait(tfull + acc, acc_phase, abort_flag, args.status, DEV_TIMEOUT_EPILOGUE);
      if (!__all_sync(0xffffffffu, ok)) break;   // keep the warp converged for tcgen05.ld
      tc_fence_after();
      const uint32_t tb = tmem_base + ((uint32_t)(q * 32) << 16) + (uint32_t)(acc * C::ACC + c_lo * 32);
      // Accumulator chunks are read from TMEM as each is needed (tcgen05.ld is warp-collective:
      // every lane executes it) and the buffer is released after the last one: the next tile's
      // main loop outlasts this epilogue, so holding TMEM costs nothing and frees the registers.
      uint8_t* box = smem + C::EPI_OFF + (warp - 2) * C::EPI_BOX;
      const int rowc = min(row, M - 1), row0 = mb * 128 + q * 32;
      const float* sa = F8 ? args.sa : nullptr;
      if constexpr (EK == EK_PUSH || EK == EK_BOX || EK >= EK_TMA) {   // 64 columns per box
        // not unrolled: one box's code is already long, and warps that miss in the instruction
        // cache stall the epilogue (the main stall of an epilogue-bound GEMM, measured)
#pragma unroll 1
        for (int b = 0; b < NC / 2; ++b) {
          uint32_t r[2][32];
          tmem_ld32(tb + (uint32_t)(b * 64), r[0]);
          tmem_ld32(tb + (uint32_t)(b * 64 + 32), r[1]);
          tmem_ld_wait();
          const int colb = colh + b * 64;
          if (colb < N) {
            if constexpr (EK == EK_PUSH) {
              epilogue_push64(args.epi, rowc, row0, colb, M, N, r[0], r[1], box, lane);
            } else if constexpr (EK >= EK_TMA) {
              const int seg = colb / args.epi.seg_w;
              epilogue_bf16_tma<2, EK - EK_TMA>(args.epi, seg == 0 ? &tmO0 : (seg == 1 ? &tmO1 : &tmO2), rowc, row0,
                                                colb, N, r, sa, args.sw, box, lane);
            } else
              epilogue_bf16_box<2>(args.epi, args.groups > 1 ? args.bias_grp[g] : args.epi.bias,
                                   (size_t)g * (size_t)args.out_grp_stride, rowc, row0, colb, M, N, r, sa,
                                   args.sw, box, lane);
          }
        }
      } else {   // 32 columns at a time
        // EPI_RESID_TMA in the CTA's last tile: every MMA has completed (tfull) and no load is
        // pending, so the pipeline stages are idle and each warp stages all its chunks at once
        // (NC boxes in flight, one wait at the end).  Earlier tiles overlap the next tile's main
        // loop and reuse the warp's one box.
        const bool last = EK == EK_RTMA && t + (int)gridDim.x >= num_tiles;
#pragma unroll 1
        for (int c = 0; c < n_ch; ++c) {
          uint32_t r[32];
          tmem_ld32(tb + (uint32_t)(c * 32), r);
          tmem_ld_wait();
          const int col0 = colh + c * 32;
          if (col0 >= N) continue;
          if constexpr (EK == EK_RTMA)
            epilogue_chunk_tma(args.epi, &tmC, rowc, row0, col0, r, sa, args.sw,
                               last ? smem + ((warp - 2) * C::H0 + c) * C::EPI_BOX : box, lane, !last);
          else if constexpr (EK == EK_RF32)
            epilogue_resid_box(args.epi, rowc, row0, col0, M, r, sa, args.sw, box, lane);
          else if (row < M)
            epilogue_chunk(args.epi, row, col0, r, sa, args.sw);
        }
      }
      tc_fence_before();
      mbar_arrive(tempty + acc);                 // the accumulator buffer is free again
      acc ^= 1;
      if (acc == 0) acc_phase ^= 1u;
    }
    if ((EK == EK_RTMA || EK >= EK_TMA) && lane == 0)
      bulk_wait0();   // residual adds / output stores performed before exit
  }
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, C::TMEM_COLS);
  }
}

int gemm_check(const GemmArgs& a, int bn) {
  const GemmEpi& e = a.epi;
  if (a.M <= 0 || a.N <= 0 || a.K <= 0) return FW_EINVAL;
  if (a.groups < 1) return FW_EINVAL;
  if (a.groups > 1) {   // grouped launches take the bf16 box epilogue only
    if (bn < 128 || !a.tmB_grp || !a.bias_grp || (reinterpret_cast<uintptr_t>(a.tmB_grp) & 63u) || a.out_grp_stride < 0)
      return FW_EINVAL;
    if (e.mode != EPI_BF16 && e.mode != EPI_GELU_BF16 && e.mode != EPI_GELU_ERF_BF16) return FW_EINVAL;
  }
  if (bn != 64 && bn != 128 && bn != 224 && bn != 256) return FW_EINVAL;
  if (bn == 224 && (a.sa || a.groups != 1 ||
                    (e.mode != EPI_RESID_TMA && e.mode != EPI_RESID_F32 && e.mode != EPI_F32)))
    return FW_EINVAL;
  if (a.N % 32 || a.K % (a.sa ? 16 : 8)) return FW_ESHAPE;
  if (a.sa && (!a.sw || (reinterpret_cast<uintptr_t>(a.sw) & 15u))) return FW_EALIGN;
  auto al16 = [](const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; };
  if (e.bias && !al16(e.bias)) return FW_EALIGN;
  if (e.fbias && (!al16(e.fbias) || e.fbias_stride % 4)) return FW_EALIGN;
  if (e.rows_per_frame <= 0) return FW_EINVAL;
  switch (e.mode) {
    case EPI_BF16:
    case EPI_GELU_BF16:
    case EPI_GELU_ERF_BF16: {
      if (e.seg_w <= 0 || e.seg_w % bn || e.ld_out % 8) return FW_ESHAPE;
      const int nseg = (a.N + e.seg_w - 1) / e.seg_w;
      if (nseg > 3) return FW_ESHAPE;
      for (int i = 0; i < nseg; ++i)
        if (!e.out[i] || !al16(e.out[i])) return FW_EALIGN;
      break;
    }
    case EPI_F32:
      if (!e.out[0] || !al16(e.out[0]) || e.ld_out % 4) return FW_EALIGN;
      break;
    case EPI_BF16_PUSH:
      if (bn < 128 || !e.out[0] || !al16(e.out[0]) || e.ld_out % 8) return FW_EINVAL;
      if (e.push_tp > 2) {
        if (e.push_tp > 8 || e.push_ls <= 0 || e.push_rank < 0 || e.push_rank >= e.push_tp || e.peer_out)
          return FW_EINVAL;
        for (int j = 0; j < e.push_tp; ++j)
          if (j != e.push_rank && (!e.push_base[j] || !al16(e.push_base[j]))) return FW_EALIGN;
      } else if (!e.peer_out || !al16(e.peer_out)) {
        return FW_EINVAL;
      }
      break;
    case EPI_RESID_TMA:
      if (e.mirror) return FW_EINVAL;   // the mirror needs the updated residual in registers
      if (!e.resid || !al16(e.resid) || e.ld_resid % 4) return FW_EALIGN;
      if (e.gate && (!al16(e.gate) || e.gate_stride % 4)) return FW_EALIGN;
      break;
    case EPI_RESID_F32:
      if (!e.resid || !al16(e.resid) || e.ld_resid % 4) return FW_EALIGN;
      if (e.gate && (!al16(e.gate) || e.gate_stride % 4)) return FW_EALIGN;
      if (e.mirror && (!al16(e.mirror) || e.ld_mirror % 8)) return FW_EALIGN;
      break;
    default:
      return FW_EINVAL;
  }
  return 0;
}

template <int BN, bool F8, int EK>
static int launch_bn(const CUtensorMap& tmA, const CUtensorMap& tmB, const CUtensorMap& tmC, const CUtensorMap* o,
                     const GemmArgs& a, cudaStream_t s, int grid) {
  using C = GemmCfg<BN>;
  cudaError_t err =
      cudaFuncSetAttribute(gemm_bf16_kernel<BN, F8, EK>, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM);
  if (err != cudaSuccess) return FW_ECUDA;
  launch_k(gemm_bf16_kernel<BN, F8, EK>, grid, 320, C::SMEM, s, tmA, tmB, tmC, o[0], o[1], o[2], a);
  return cudaGetLastError() == cudaSuccess ? 0 : FW_ECUDA;
}

static int epi_kind(const GemmEpi& e, int bn) {
  switch (e.mode) {
    case EPI_BF16_PUSH: return EK_PUSH;
    case EPI_BF16:
    case EPI_GELU_BF16:
    case EPI_GELU_ERF_BF16: return bn < 128 ? EK_CHUNK : (e.tma_store ? EK_TMA + e.mode : EK_BOX);
    case EPI_RESID_TMA: return EK_RTMA;
    case EPI_RESID_F32: return EK_RF32;
    default: return EK_CHUNK;
  }
}

template <int BN, bool F8>
static int launch_kind(const CUtensorMap& tmA, const CUtensorMap& tmB, const CUtensorMap& tmC, const CUtensorMap* o,
                       const GemmArgs& a, cudaStream_t s, int grid) {
  switch (epi_kind(a.epi, BN)) {
    case EK_RTMA: return launch_bn<BN, F8, EK_RTMA>(tmA, tmB, tmC, o, a, s, grid);
    case EK_RF32: return launch_bn<BN, F8, EK_RF32>(tmA, tmB, tmC, o, a, s, grid);
    case EK_CHUNK: return launch_bn<BN, F8, EK_CHUNK>(tmA, tmB, tmC, o, a, s, grid);
    default: break;
  }
  if constexpr (BN >= 128) {   // the box kinds need two 32-column chunks per thread
    switch (epi_kind(a.epi, BN)) {
      case EK_BOX: return launch_bn<BN, F8, EK_BOX>(tmA, tmB, tmC, o, a, s, grid);
      case EK_TMA + EPI_BF16: return launch_bn<BN, F8, EK_TMA + EPI_BF16>(tmA, tmB, tmC, o, a, s, grid);
      case EK_TMA + EPI_GELU_BF16: return launch_bn<BN, F8, EK_TMA + EPI_GELU_BF16>(tmA, tmB, tmC, o, a, s, grid);
      case EK_TMA + EPI_GELU_ERF_BF16:
        return launch_bn<BN, F8, EK_TMA + EPI_GELU_ERF_BF16>(tmA, tmB, tmC, o, a, s, grid);
      case EK_PUSH:
        if constexpr (!F8) return launch_bn<BN, false, EK_PUSH>(tmA, tmB, tmC, o, a, s, grid);
        break;
      default: break;
    }
  }
  return FW_EINVAL;
}

int make_out_tmaps(GemmArgs& a, CUtensorMap (&o)[3]) {
  GemmEpi& e = a.epi;
  e.tma_store = false;
  if (a.groups != 1 || (e.mode != EPI_BF16 && e.mode != EPI_GELU_BF16 && e.mode != EPI_GELU_ERF_BF16)) return 0;
  if (e.seg_w <= 0 || e.ld_out % 8) return FW_ESHAPE;
  const int nseg = (a.N + e.seg_w - 1) / e.seg_w;
  if (nseg > 3) return FW_ESHAPE;
  for (int i = 0; i < nseg; ++i) {
    const int cols = a.N - i * e.seg_w < e.seg_w ? a.N - i * e.seg_w : e.seg_w;
    const int rc = make_tmap_2d(&o[i], e.out[i], 2, a.M, cols, e.ld_out, 32, 64, true);
    if (rc) return rc;
  }
  for (int i = nseg; i < 3; ++i) o[i] = o[0];
  e.tma_store = true;
  return 0;
}

int gemm_resid_bn(int M, int N) {
  if (N < 256) return N >= 128 ? 128 : 64;
  // waves x tile width: the time of the busiest SM, up to the per-tile constant
  const int sms = num_sms(), mt = (M + 127) / 128;
  const long c256 = (long)((mt * ((N + 255) / 256) + sms - 1) / sms) * 256;
  const long c224 = (long)((mt * ((N + 223) / 224) + sms - 1) / sms) * 224;
  return c224 < c256 ? 224 : 256;
}

int gemm_bf16_launch(const CUtensorMap& tmA, const CUtensorMap& tmB, int bn, const GemmArgs& a, cudaStream_t s,
                     int ctas, const CUtensorMap* tmC, const CUtensorMap* tmO) {
  int rc = gemm_check(a, bn);
  if (rc) return rc;
  if (a.epi.mode == EPI_RESID_TMA && !tmC) return FW_EINVAL;
  if (a.epi.tma_store && (!tmO || a.groups != 1)) return FW_EINVAL;
  const CUtensorMap& mc = tmC ? *tmC : tmA;   // unused unless EPI_RESID_TMA
  const CUtensorMap none[3] = {tmA, tmA, tmA};   // unused unless epi.tma_store
  const CUtensorMap* o = a.epi.tma_store ? tmO : none;
  const int tiles = ((a.M + 127) / 128) * ((a.N + bn - 1) / bn) * a.groups;
  int grid = ctas > 0 ? ctas : num_sms();
  if (grid > tiles) grid = tiles;
  GemmArgs b = a;
  switch (bn) {
    case 256:
      return a.sa ? launch_kind<256, true>(tmA, tmB, mc, o, b, s, grid) : launch_kind<256, false>(tmA, tmB, mc, o, b, s, grid);
    case 224:   // bf16 operands, 32-column epilogue kinds (gemm_check)
      switch (epi_kind(a.epi, 224)) {
        case EK_RTMA: return launch_bn<224, false, EK_RTMA>(tmA, tmB, mc, o, b, s, grid);
        case EK_RF32: return launch_bn<224, false, EK_RF32>(tmA, tmB, mc, o, b, s, grid);
        case EK_CHUNK: return launch_bn<224, false, EK_CHUNK>(tmA, tmB, mc, o, b, s, grid);
        default: return FW_EINVAL;
      }
    case 128:
      return a.sa ? launch_kind<128, true>(tmA, tmB, mc, o, b, s, grid) : launch_kind<128, false>(tmA, tmB, mc, o, b, s, grid);
    default:
      return a.sa ? launch_kind<64, true>(tmA, tmB, mc, o, b, s, grid) : launch_kind<64, false>(tmA, tmB, mc, o, b, s, grid);
  }
}

}  // namespace fw
