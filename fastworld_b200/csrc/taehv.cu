// TAEHV streaming video decoder on tcgen05 for sm_100a (the reference's optional lossy decoder,
// fastworld/models/mg2/vae.py:95-124 `TinyVAE`, which runs the third-party TAEHV `taew2_1`
// decoder through its StreamingTAEHV wrapper).
//
// The decoder, per latent chunk of F0 frames [lat_ch, F0, h, w]:
//   clamp 3 tanh(x / 3) -> conv3x3(lat_ch -> C0) + bias, ReLU
//   stage s = 0, 1, 2 at (h, w) * 2^s with C_s channels and F_s frames:
//     3 x MemBlock:  y = ReLU(conv3x3(ReLU(conv3x3(ReLU(conv3x3(cat[x, past]))))) + x), where
//                    past = the block's input one frame earlier (the last frame of the previous
//                    chunk for the first frame: the streaming state);
//     nearest 2x upsample, TGrow (1x1 conv C_s -> C_s * r_s, output frame f * r_s + j takes
//     channels [j C_s, (j + 1) C_s)), conv3x3(C_s -> C_{s+1}) without bias
//   ReLU, conv3x3(C_3 -> 3) + bias, clamp to [0, 1], x 2 - 1 (vae.py:109).
//
// Layout: activations fp16 NHWC, one [F, H, W, C] tensor per layer output; weights fp16
// [Cout, taps * Cin] with K ordered (tap, input channel), biases fp32.
//
// One kernel, `conv_kernel<BN, EK>`, runs every layer as an implicit GEMM (persistent, one CTA
// per SM, warp-specialised like the engine's linear GEMM):
//   M = output pixels in tiles of 8 rows x 16 columns of one frame (128 TMEM lanes),
//   N = output channels in tiles of BN, K = taps x input channels in blocks of 64.
//   warp 0     TMA producer: per K block one 4-D box {64 channels, 16 x, 8 y, 1 frame} of the
//              input at the tap's offset; TMA's zero fill outside the image is the conv's
//              zero padding, so there is no im2col buffer and no halo logic.  The concatenated
//              past input of a MemBlock is a second source: frame f - 1 of the same tensor,
//              or the state frame for f = 0.
//   warp 1     MMA issuer: 4 x tcgen05.mma kind::f16 (fp16 A and B, fp32 accumulate in TMEM)
//              per K block; double-buffered TMEM accumulator.
//   warps 2-9  two epilogue groups of four warps, alternating tiles (group g drains TMEM buffer
//              g), thread = output pixel:
//                EK_STORE  (+bias) (+residual, rounded to fp16 first as the eager module
//                          sums two fp16 tensors) (ReLU) -> fp16 box -> 4-D TMA store
//                EK_UP     TGrow + nearest 2x upsample: each 64-channel box is written to
//                          both output rows of its pixel row pair, each pixel twice along x,
//                          by TMA stores of [32 pixels x 64 channels] rows
// The first conv's input has 16 channels: a prep kernel applies the clamp and writes its
// 3 x 3 neighbourhoods as 144 (padded to 192) channels, and that conv runs as a 1-tap conv.
// The last conv (64 -> 3) runs in `rgb_kernel`, transposed (all taps' products per input pixel,
// then a 3 x 3 gather), with the bias, fp16 rounding, clamp and x 2 - 1 in its epilogue.
#include <cuda_fp16.h>

#include <cstring>
#include <string>
#include <vector>

#include "../../include/fastworld_b200.h"
#include "fw_internal.h"
#include "fw_ptx.cuh"

namespace fw {

namespace taehv {

enum : int { EK_STORE = 0, EK_UP = 1 };

constexpr int kSmemLimit = 232448;   // opt-in dynamic shared memory per CTA

// How the A operand (and B) reach shared memory:
//   LM_TAP    one pipeline unit per (tap, 64-channel block): A = the 128 pixels at the tap's
//             offset (4-D box {64, 16, 8, 1}), B = the tap's weight block; a 3 x 3 conv reads
//             every input byte 9 times from L2
//   LM_HALO   one unit per (64-channel block, dx): A = the tile's 10 input rows (8 + halo) at
//             x offset dx (box {64, 16, 10, 1}, 20 KB), from which the three taps dy = -1, 0, 1
//             are the 1024-byte-aligned windows at rows 0, 1, 2 (2048 bytes apart); B = those
//             three taps' weight blocks.  Input bytes are read 3 times (x halo copies).
//   LM_HALO_RES  LM_HALO with all weights resident in shared memory (loaded once per CTA)
enum : int { LM_TAP = 0, LM_HALO = 1, LM_HALO_RES = 2 };

template <int BN, int EK, int LM>
struct Cfg {
  static constexpr int A_BYTES = LM == LM_TAP ? 128 * 128 : 160 * 128;
  static constexpr int B_BYTES = LM == LM_TAP ? BN * 128 : (LM == LM_HALO ? 3 * BN * 128 : 0);
  static constexpr int STAGE = A_BYTES + B_BYTES;
  // resident weights: 9 taps x one 64-channel block
  static constexpr int RES = LM == LM_HALO_RES ? 9 * BN * 128 : 0;
  // per epilogue warp: EK_STORE one [32 pixels x 128 B] box; EK_UP two upsampled rows
  static constexpr int BOX = EK == EK_STORE ? 4096 : 8192;
  static constexpr int EPI = 8 * BOX;
  static constexpr int FIT = (kSmemLimit - 2048 - EPI - RES) / STAGE;
  static constexpr int STAGES = FIT > 8 ? 8 : FIT;
  static constexpr int RES_OFF = STAGES * STAGE;
  static constexpr int BAR_OFF = RES_OFF + RES;
  static constexpr int EPI_OFF = BAR_OFF + 1024;
  static constexpr int SMEM = EPI_OFF + EPI + 1024;
  static constexpr uint32_t TMEM_COLS = 2 * BN;
  static_assert(STAGES >= 3, "pipeline too shallow");
  static_assert(SMEM <= kSmemLimit, "shared memory");
  static_assert(STAGE % 1024 == 0 && RES % 1024 == 0, "1024-byte aligned operands");
};

struct ConvArgs {
  int T, H, W;        // frames and size of the (input = output) grid
  int taps;           // 9 (3 x 3, padding 1) or 1
  int ch0, ch1;       // 64-channel blocks of the input and of the past input (0: none)
  int N;              // output channels
  const float* bias;  // [N] or null
  const __half* resid;   // [T, H, W, N] or null (EK_STORE)
  int relu;
  int up_stride, up_C;   // EK_UP: output frames per input frame, channels per output frame
  float* rgb;            // rgb_kernel: [T, 3, H, W]
  int* status;
};

__device__ __forceinline__ float round_h(float v) { return __half2float(__float2half_rn(v)); }
__device__ __forceinline__ uint32_t pack_h2(float a, float b) {
  __half2 h = __floats2half2_rn(a, b);
  return *reinterpret_cast<uint32_t*>(&h);
}
// AND of `pred` over the 128 threads that use named barrier `id` (a barrier for all of them).
__device__ __forceinline__ bool bar_and128(int id, bool pred) {
  uint32_t r;
  asm volatile(
      "{\n\t.reg .pred p, q;\n\t"
      "setp.ne.u32 p, %1, 0;\n\t"
      "barrier.red.and.pred q, %2, 128, p;\n\t"
      "selp.u32 %0, 1, 0, q;\n\t}\n"
      : "=r"(r)
      : "r"((uint32_t)pred), "r"(id)
      : "memory");
  return r != 0;
}

template <int BN, int EK, int LM>
__global__ void __launch_bounds__(320, 1)
    conv_kernel(const __grid_constant__ CUtensorMap tmX, const __grid_constant__ CUtensorMap tmM,
                const __grid_constant__ CUtensorMap tmW, const __grid_constant__ CUtensorMap tmY, const ConvArgs a) {
  using C = Cfg<BN, EK, LM>;
  constexpr bool HALO = LM != LM_TAP;
  pdl_trigger();
  extern __shared__ uint8_t smem_raw[];
  const uint32_t pad = (1024u - (smem_u32(smem_raw) & 1023u)) & 1023u;
  uint8_t* smem = smem_raw + pad;
  uint8_t* sA = smem;
  uint8_t* sB = smem + C::STAGES * C::A_BYTES;
  uint8_t* sR = smem + C::RES_OFF;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + C::BAR_OFF);
  uint64_t* empty = full + C::STAGES;
  uint64_t* tfull = empty + C::STAGES;
  uint64_t* tempty = tfull + 2;
  uint64_t* drain = tempty + 2;
  uint64_t* res_full = drain + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(res_full + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nxb = a.W >> 4, nyb = (a.H + 7) >> 3;
  const int num_m = a.T * nyb * nxb, num_n = (a.N + BN - 1) / BN;
  const int num_tiles = num_m * num_n;
  const int cpt = a.ch0 + a.ch1;
  // pipeline units per tile: (tap, block) or (block, dx)
  const int num_kb = HALO ? 3 * cpt : a.taps * cpt;

  if (threadIdx.x == 0) {
    for (int s = 0; s < C::STAGES; ++s) {
      mbar_init(full + s, 1);
      mbar_init(empty + s, 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(tfull + b, 1);
      mbar_init(tempty + b, 128);   // the four warps of epilogue group b
    }
    mbar_init(drain, 1);
    mbar_init(res_full, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch(&tmX);
    tma_prefetch(&tmW);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, C::TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  // The weights are static: they are requested before the wait on the previous kernel (the
  // resident copy, or the first tile's blocks while the ring's stages are still free).
  int pre = 0;
  if (warp == 0 && lane == 0 && blockIdx.x < num_tiles) {
    if constexpr (LM == LM_HALO_RES) {
      mbar_arrive_expect_tx(res_full, C::RES);
      for (int p = 0; p < 9; ++p) tma_load_2d(sR + p * BN * 128, &tmW, res_full, p * 64, 0);
    } else if constexpr (LM == LM_TAP) {
      pre = num_kb < C::STAGES ? num_kb : C::STAGES;
      const int nb0 = blockIdx.x / num_m;
      for (int kb = 0; kb < pre; ++kb) {
        mbar_arrive_expect_tx(full + kb, C::STAGE);
        tma_load_2d(sB + kb * C::B_BYTES, &tmW, full + kb, kb * 64, nb0 * BN);
      }
    }
  }
  pdl_wait();

  if (warp == 0) {
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0, used = 0, last_par = 0;
      bool ok = true;
      for (int t = blockIdx.x; t < num_tiles && ok; t += gridDim.x) {
        const int m = t % num_m, nb = t / num_m;
        const int xb = m % nxb, r = m / nxb, yb = r % nyb, f = r / nyb;
        const int x0 = xb * 16, y0 = yb * 8;
        for (int kb = 0; kb < num_kb; ++kb) {
          // unit kb: LM_TAP (tap p, block j); halo modes (block j, x offset dx)
          const int p = HALO ? 0 : kb / cpt, j = HALO ? kb / 3 : kb - p * cpt;
          const int dy = HALO ? -1 : (a.taps == 9 ? p / 3 - 1 : 0);
          const int dx = HALO ? kb % 3 - 1 : (a.taps == 9 ? p % 3 - 1 : 0);
          if (!(t == (int)blockIdx.x && kb < pre)) {
            if (!mbar_wait(empty + stage, phase ^ 1u, abort_flag, a.status, DEV_TIMEOUT_PRODUCER)) {
              ok = false;
              break;
            }
            mbar_arrive_expect_tx(full + stage, C::STAGE);
            if constexpr (LM == LM_TAP) {
              tma_load_2d(sB + stage * C::B_BYTES, &tmW, full + stage, kb * 64, nb * BN);
            } else if constexpr (LM == LM_HALO) {   // weight blocks of taps (dy, dx), dy = -1, 0, 1
              for (int d = 0; d < 3; ++d)
                tma_load_2d(sB + stage * C::B_BYTES + d * BN * 128, &tmW, full + stage,
                            ((d * 3 + dx + 1) * cpt + j) * 64, nb * BN);
            }
          }
          uint8_t* dst = sA + stage * C::A_BYTES;
          if (j < a.ch0)
            tma_load_4d(dst, &tmX, full + stage, j * 64, x0 + dx, y0 + dy, f);
          else if (f == 0)   // past of the chunk's first frame: the state frame
            tma_load_4d(dst, &tmM, full + stage, (j - a.ch0) * 64, x0 + dx, y0 + dy, 0);
          else
            tma_load_4d(dst, &tmX, full + stage, (j - a.ch0) * 64, x0 + dx, y0 + dy, f - 1);
          used |= 1u << stage;
          last_par = (last_par & ~(1u << stage)) | (phase << stage);
          if (++stage == C::STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
      volatile int no_abort = 0;
      for (int s = 0; s < C::STAGES; ++s)
        if (used >> s & 1u) mbar_wait(full + s, last_par >> s & 1u, &no_abort, a.status, DEV_TIMEOUT_DRAIN);
      if (LM == LM_HALO_RES && blockIdx.x < num_tiles)
        mbar_wait(res_full, 0, &no_abort, a.status, DEV_TIMEOUT_DRAIN);
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t idesc = idesc_f16(128, BN);
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      int i = 0;
      if (LM == LM_HALO_RES && blockIdx.x < num_tiles)
        ok = mbar_wait(res_full, 0, abort_flag, a.status, DEV_TIMEOUT_MMA);
      for (int t = blockIdx.x; t < num_tiles && ok; t += gridDim.x, ++i) {
        const int acc = i & 1;
        const uint32_t acc_phase = (uint32_t)(i >> 1) & 1u;
        if (!mbar_wait(tempty + acc, acc_phase ^ 1u, abort_flag, a.status, DEV_TIMEOUT_MMA)) break;
        tc_fence_after();
        const uint32_t d = tmem_base + (uint32_t)(acc * BN);
        for (int kb = 0; kb < num_kb; ++kb) {
          if (!mbar_wait(full + stage, phase, abort_flag, a.status, DEV_TIMEOUT_MMA)) {
            ok = false;
            break;
          }
          tc_fence_after();
          // Descriptors are built once per unit; operand offsets are added to their 14-bit
          // start-address field (byte offset / 16; every offset stays inside shared memory).
          // kind::f16; the instruction descriptor selects fp16 operands.
          const uint64_t ad = sdesc_sw128(smem_u32(sA + stage * C::A_BYTES), 16, 1024);
          if constexpr (LM == LM_TAP) {
            const uint64_t bd = sdesc_sw128(smem_u32(sB + stage * C::B_BYTES), 16, 1024);
#pragma unroll
            for (int k = 0; k < 4; ++k) umma_bf16(d, ad + 2 * k, bd + 2 * k, idesc, (kb | k) != 0);
          } else {
            const int dxi = kb % 3;
            const uint64_t bd = LM == LM_HALO ? sdesc_sw128(smem_u32(sB + stage * C::B_BYTES), 16, 1024)
                                              : sdesc_sw128(smem_u32(sR) + (uint32_t)(dxi * BN * 128), 16, 1024);
#pragma unroll
            for (int dyi = 0; dyi < 3; ++dyi) {
              // tap (dy, dx): the window at input row dyi of the unit's 10 rows (2048 bytes apart);
              // its weight block: dyi-th of the unit's three, or tap dyi * 3 + dxi of the resident copy
              const uint64_t aw = ad + (uint64_t)(dyi * 128);
              const uint64_t bw = bd + (uint64_t)(dyi * (LM == LM_HALO ? BN * 8 : 3 * BN * 8));
#pragma unroll
              for (int k = 0; k < 4; ++k) umma_bf16(d, aw + 2 * k, bw + 2 * k, idesc, (kb | dyi | k) != 0);
            }
          }
          umma_commit(empty + stage);
          if (++stage == C::STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (!ok) break;
        umma_commit(tfull + acc);
      }
      umma_commit(drain);
      volatile int no_abort = 0;
      mbar_wait(drain, 0, &no_abort, a.status, DEV_TIMEOUT_DRAIN);
    }
  } else {
    // epilogue group g = tiles i with i % 2 == g; warp quarter q = TMEM lanes 32q .. 32q + 31
    const int g = (warp - 2) >> 2, q = warp & 3;
    uint8_t* box = smem + C::EPI_OFF + (warp - 2) * C::BOX;
    const int pr = q * 32 + lane;              // pixel of the tile
    const int yl = pr >> 4, xl = pr & 15;
    int i = 0;
    for (int t = blockIdx.x; t < num_tiles; t += gridDim.x, ++i) {
      if ((i & 1) != g) continue;
      const int m = t % num_m, nb = t / num_m;
      const int xb = m % nxb, r = m / nxb, yb = r % nyb, f = r / nyb;
      const int x0 = xb * 16, y0 = yb * 8;
      const int y = y0 + yl, x = x0 + xl;
      const bool inside = y < a.H;
      const bool ok = mbar_wait(tfull + g, (uint32_t)(i >> 1) & 1u, abort_flag, a.status, DEV_TIMEOUT_EPILOGUE);
      if (!__all_sync(0xffffffffu, ok)) break;
      tc_fence_after();
      const uint32_t tb = tmem_base + ((uint32_t)(q * 32) << 16) + (uint32_t)(g * BN);
      {
#pragma unroll 1
        for (int b = 0; b < BN / 64; ++b) {
          uint32_t v[2][32];
          tmem_ld32(tb + (uint32_t)(b * 64), v[0]);
          tmem_ld32(tb + (uint32_t)(b * 64 + 32), v[1]);
          tmem_ld_wait();
          const int n0 = nb * BN + b * 64;
          if (n0 >= a.N) break;
          uint32_t h2[32];
          if constexpr (EK == EK_STORE) {
            uint4 res[8];
            if (a.resid && inside) {
              const uint4* rp =
                  reinterpret_cast<const uint4*>(a.resid + ((((size_t)f * a.H + y) * a.W + x) * a.N + n0));
#pragma unroll
              for (int c = 0; c < 8; ++c) res[c] = __ldg(rp + c);
            }
#pragma unroll
            for (int c = 0; c < 8; ++c) {
              float4 bb = make_float4(0.f, 0.f, 0.f, 0.f), bh = bb;
              if (a.bias) {
                bb = __ldg(reinterpret_cast<const float4*>(a.bias + n0 + c * 8));
                bh = __ldg(reinterpret_cast<const float4*>(a.bias + n0 + c * 8 + 4));
              }
              float e[8] = {bb.x, bb.y, bb.z, bb.w, bh.x, bh.y, bh.z, bh.w};
#pragma unroll
              for (int k = 0; k < 8; ++k) e[k] += __uint_as_float(v[c >> 2][(c & 3) * 8 + k]);
              if (a.resid && inside) {
                const __half* rh = reinterpret_cast<const __half*>(&res[c]);
#pragma unroll
                for (int k = 0; k < 8; ++k) e[k] = round_h(e[k]) + __half2float(rh[k]);
              }
              if (a.relu) {
#pragma unroll
                for (int k = 0; k < 8; ++k) e[k] = fmaxf(e[k], 0.f);
              }
#pragma unroll
              for (int k = 0; k < 4; ++k) h2[c * 4 + k] = pack_h2(e[2 * k], e[2 * k + 1]);
            }
            // the box of the previous tile must have been read by its TMA store
            if (lane == 0) bulk_wait_read0();
            __syncwarp();
#pragma unroll
            for (int c = 0; c < 8; ++c)
              *reinterpret_cast<uint4*>(box + lane * 128 + ((c ^ (lane & 7)) << 4)) =
                  make_uint4(h2[c * 4], h2[c * 4 + 1], h2[c * 4 + 2], h2[c * 4 + 3]);
            fence_proxy_async_smem();
            __syncwarp();
            if (lane == 0 && y0 + q * 2 < a.H) {   // rows past the image are not stored
              tma_store_4d(&tmY, box, n0, x0, y0 + q * 2, f);
              bulk_commit();
            }
          } else {   // EK_UP: no bias, no activation
#pragma unroll
            for (int c = 0; c < 32; ++c)
              h2[c] = pack_h2(__uint_as_float(v[c >> 4][(c & 15) * 2]), __uint_as_float(v[c >> 4][(c & 15) * 2 + 1]));
            if (lane == 0) bulk_wait_read0();
            __syncwarp();
            uint8_t* row = box + (lane >> 4) * 4096;   // this pixel row's upsampled row
#pragma unroll
            for (int d = 0; d < 2; ++d) {
              const int px = 2 * (lane & 15) + d;
#pragma unroll
              for (int c = 0; c < 8; ++c)
                *reinterpret_cast<uint4*>(row + px * 128 + ((c ^ (px & 7)) << 4)) =
                    make_uint4(h2[c * 4], h2[c * 4 + 1], h2[c * 4 + 2], h2[c * 4 + 3]);
            }
            fence_proxy_async_smem();
            __syncwarp();
            if (lane == 0) {
              const int s = n0 / a.up_C, c0 = n0 - s * a.up_C, fo = f * a.up_stride + s;
#pragma unroll
              for (int hl = 0; hl < 2; ++hl) {
                const int ylo = y0 + q * 2 + hl;
                if (ylo < a.H) {
                  tma_store_4d(&tmY, box + hl * 4096, c0, 2 * x0, 2 * ylo, fo);
                  tma_store_4d(&tmY, box + hl * 4096, c0, 2 * x0, 2 * ylo + 1, fo);
                }
              }
              bulk_commit();
            }
          }
        }
      }
      tc_fence_before();
      mbar_arrive(tempty + g);
    }
    if (lane == 0) bulk_wait0();
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) tmem_dealloc(tmem_base, C::TMEM_COLS);
}

// Clamp (3 tanh(x / 3) of the fp16 latent, each step rounded to fp16 as the eager fp16 module
// computes it) and
// writes the first conv's 3 x 3 neighbourhoods: im[f, y, x, tap * 16 + c] for tap < 9, zeros for
// the 48 padding channels (taps 9..11).
__global__ void __launch_bounds__(256) prep_kernel(const __half* __restrict__ lat, __half* __restrict__ im,
                                                   int T, int H, int W) {
  pdl_trigger();
  pdl_wait();
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  const int total = T * H * W * 12;
  if (i >= total) return;
  const int tap = i % 12, pix = i / 12;
  const int x = pix % W, y = (pix / W) % H, f = pix / (W * H);
  uint32_t o[8] = {0, 0, 0, 0, 0, 0, 0, 0};
  if (tap < 9) {
    const int yy = y + tap / 3 - 1, xx = x + tap % 3 - 1;
    if (yy >= 0 && yy < H && xx >= 0 && xx < W) {
      const size_t cs = (size_t)T * H * W;   // channel stride of [16, T, H, W]
      const size_t base = ((size_t)f * H + yy) * W + xx;
      float v[16];
#pragma unroll
      for (int c = 0; c < 16; ++c) {
        const float d = round_h(__half2float(lat[c * cs + base]) / 3.f);
        v[c] = round_h(round_h(tanhf(d)) * 3.f);
      }
#pragma unroll
      for (int k = 0; k < 8; ++k) o[k] = pack_h2(v[2 * k], v[2 * k + 1]);
    }
  }
  uint4* dst = reinterpret_cast<uint4*>(im + (size_t)pix * 192 + tap * 16);
  dst[0] = make_uint4(o[0], o[1], o[2], o[3]);
  dst[1] = make_uint4(o[4], o[5], o[6], o[7]);
}

// State update: the last frame of each MemBlock's input becomes that block's past for the next
// chunk.  Up to 16 segments, 16-byte copies.
struct SegCopy {
  const uint4* src[16];
  uint4* dst[16];
  long long n16[16];
  int nseg;
};
__global__ void __launch_bounds__(256) seg_copy_kernel(const SegCopy c) {
  pdl_trigger();
  pdl_wait();
  for (int s = 0; s < c.nseg; ++s)
    for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < c.n16[s];
         i += (long long)gridDim.x * blockDim.x)
      c.dst[s][i] = c.src[s][i];
}

// fp16 tensor map: 4-D [F, H, W, C] NHWC, box {64 channels, bx, by, 1}, 128-byte swizzle.
int make_map_nhwc(CUtensorMap* out, const void* base, int F, int H, int W, int Cc, int bx, int by) {
  PFN_encodeTiled enc = get_encode_fn();
  if (!enc) return FW_ENODRIVER;
  if (!base || (reinterpret_cast<uintptr_t>(base) & 15u) || Cc % 64) return FW_EINVAL;
  cuuint64_t dims[4] = {(cuuint64_t)Cc, (cuuint64_t)W, (cuuint64_t)H, (cuuint64_t)F};
  cuuint64_t strides[3] = {(cuuint64_t)Cc * 2, (cuuint64_t)W * Cc * 2, (cuuint64_t)H * W * Cc * 2};
  cuuint32_t box[4] = {64, (cuuint32_t)bx, (cuuint32_t)by, 1};
  cuuint32_t estr[4] = {1, 1, 1, 1};
  CUresult r = enc(out, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 4, const_cast<void*>(base), dims, strides, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? 0 : FW_EINVAL;
}
// fp16 weights [rows, K], box {64, box_rows}, 128-byte swizzle.
int make_map_w(CUtensorMap* out, const void* base, int rows, int K, int box_rows) {
  PFN_encodeTiled enc = get_encode_fn();
  if (!enc) return FW_ENODRIVER;
  if (!base || (reinterpret_cast<uintptr_t>(base) & 15u) || K % 64) return FW_EINVAL;
  cuuint64_t dims[2] = {(cuuint64_t)K, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)K * 2};
  cuuint32_t box[2] = {64, (cuuint32_t)box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = enc(out, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void*>(base), dims, strides, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? 0 : FW_EINVAL;
}

template <int BN, int EK, int LM>
int launch_conv(const CUtensorMap& x, const CUtensorMap& m, const CUtensorMap& w, const CUtensorMap& y,
                const ConvArgs& a, cudaStream_t s) {
  using C = Cfg<BN, EK, LM>;
  if (cudaFuncSetAttribute(conv_kernel<BN, EK, LM>, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM) !=
      cudaSuccess)
    return FW_ECUDA;
  const int tiles = a.T * ((a.H + 7) / 8) * (a.W / 16) * ((a.N + BN - 1) / BN);
  const int grid = tiles < num_sms() ? tiles : num_sms();
  launch_k(conv_kernel<BN, EK, LM>, grid, 320, C::SMEM, s, x, m, w, y, a);
  return cudaGetLastError() == cudaSuccess ? 0 : FW_ECUDA;
}

// The last conv (64 -> 3 channels) in the transposed arrangement: a 3-channel conv on the
// per-tap form would spend 36 tensor-core MMAs per 128 pixels (each MMA of M = 128 costs about
// as much at N = 32 as at N = 64, and only 3 of the columns are used).  Instead, per tile of
// 8 x 16 output pixels, the input region with its halo (10 rows x 18 columns = 180 pixels, one
// TMA box) is multiplied by all 27 (tap, channel) weight rows at once: D[r, t * 3 + c] =
// in[r] . W[c, t] for every region pixel r (two M = 128 blocks, K = 64: 8 MMAs).  The epilogue
// writes D to shared memory and each output pixel sums its 9 neighbours' entries:
// out[y, x, c] = sum_t D[(y + dy_t + 1) * 18 + x + dx_t + 1, t * 3 + c], then bias, fp16
// rounding, clamp to [0, 1], x 2 - 1.
namespace rgbk {
constexpr int REGION = 180, A_BYTES = 256 * 128, BOX_BYTES = REGION * 128;
constexpr int STAGES = 4;
constexpr int W_OFF = STAGES * A_BYTES;          // resident weights [32 rows (t * 3 + c), 64]
constexpr int T_OFF = W_OFF + 32 * 128;          // per epilogue group: D table [256][27] fp32
constexpr int T_BYTES = 256 * 27 * 4;
constexpr int BAR_OFF = T_OFF + 2 * T_BYTES;
constexpr int SMEM = BAR_OFF + 1024 + 1024;
static_assert(SMEM <= kSmemLimit, "shared memory");
}  // namespace rgbk

__global__ void __launch_bounds__(320, 1)
    rgb_kernel(const __grid_constant__ CUtensorMap tmX, const __grid_constant__ CUtensorMap tmW, const ConvArgs a) {
  using namespace rgbk;
  pdl_trigger();
  extern __shared__ uint8_t smem_raw[];
  const uint32_t pad = (1024u - (smem_u32(smem_raw) & 1023u)) & 1023u;
  uint8_t* smem = smem_raw + pad;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + BAR_OFF);
  uint64_t* empty = full + STAGES;
  uint64_t* tfull = empty + STAGES;
  uint64_t* tempty = tfull + 2;
  uint64_t* drain = tempty + 2;
  uint64_t* res_full = drain + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(res_full + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nxb = a.W >> 4, nyb = (a.H + 7) >> 3;
  const int num_tiles = a.T * nyb * nxb;
  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(full + s, 1);
      mbar_init(empty + s, 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(tfull + b, 1);
      mbar_init(tempty + b, 128);
    }
    mbar_init(drain, 1);
    mbar_init(res_full, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, 128);   // 2 buffers x (2 region blocks x 32 columns)
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  if (warp == 0 && lane == 0 && blockIdx.x < num_tiles) {   // static weights: before the wait
    mbar_arrive_expect_tx(res_full, 32 * 128);
    tma_load_2d(smem + W_OFF, &tmW, res_full, 0, 0);
  }
  pdl_wait();
  if (warp == 0) {
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0, used = 0, last_par = 0;
      for (int t = blockIdx.x; t < num_tiles; t += gridDim.x) {
        const int xb = t % nxb, r = t / nxb, yb = r % nyb, f = r / nyb;
        if (!mbar_wait(empty + stage, phase ^ 1u, abort_flag, a.status, DEV_TIMEOUT_PRODUCER)) break;
        mbar_arrive_expect_tx(full + stage, BOX_BYTES);
        tma_load_4d(smem + stage * A_BYTES, &tmX, full + stage, 0, xb * 16 - 1, yb * 8 - 1, f);
        used |= 1u << stage;
        last_par = (last_par & ~(1u << stage)) | (phase << stage);
        if (++stage == STAGES) {
          stage = 0;
          phase ^= 1u;
        }
      }
      volatile int no_abort = 0;
      for (int s = 0; s < STAGES; ++s)
        if (used >> s & 1u) mbar_wait(full + s, last_par >> s & 1u, &no_abort, a.status, DEV_TIMEOUT_DRAIN);
      if (blockIdx.x < num_tiles) mbar_wait(res_full, 0, &no_abort, a.status, DEV_TIMEOUT_DRAIN);
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t idesc = idesc_f16(128, 32);
      int stage = 0;
      uint32_t phase = 0;
      bool ok = blockIdx.x >= num_tiles || mbar_wait(res_full, 0, abort_flag, a.status, DEV_TIMEOUT_MMA);
      const uint64_t bd = sdesc_sw128(smem_u32(smem + W_OFF), 16, 1024);
      int i = 0;
      for (int t = blockIdx.x; t < num_tiles && ok; t += gridDim.x, ++i) {
        const int acc = i & 1;
        if (!mbar_wait(tempty + acc, ((uint32_t)(i >> 1) & 1u) ^ 1u, abort_flag, a.status, DEV_TIMEOUT_MMA)) break;
        if (!mbar_wait(full + stage, phase, abort_flag, a.status, DEV_TIMEOUT_MMA)) break;
        tc_fence_after();
        const uint64_t ad = sdesc_sw128(smem_u32(smem + stage * A_BYTES), 16, 1024);
#pragma unroll
        for (int blk = 0; blk < 2; ++blk)   // region pixels 0-127 and 128-255 (180-255 unused)
#pragma unroll
          for (int k = 0; k < 4; ++k)       // kind::f16, fp16 operands
            umma_bf16(tmem_base + (uint32_t)(acc * 64 + blk * 32), ad + (uint64_t)(blk * 1024) + 2 * k, bd + 2 * k,
                      idesc, k != 0);
        umma_commit(empty + stage);
        umma_commit(tfull + acc);
        if (++stage == STAGES) {
          stage = 0;
          phase ^= 1u;
        }
      }
      umma_commit(drain);
      volatile int no_abort = 0;
      mbar_wait(drain, 0, &no_abort, a.status, DEV_TIMEOUT_DRAIN);
    }
  } else {
    const int g = (warp - 2) >> 2, q = warp & 3;
    float* tab = reinterpret_cast<float*>(smem + T_OFF + g * T_BYTES);
    const int bar_id = 1 + g;
    const int p = q * 32 + lane, yl = p >> 4, xl = p & 15;
    const size_t plane = (size_t)a.H * a.W;
    float bias[3];
#pragma unroll
    for (int c = 0; c < 3; ++c) bias[c] = a.bias ? __ldg(a.bias + c) : 0.f;
    int i = 0;
    for (int t = blockIdx.x; t < num_tiles; t += gridDim.x, ++i) {
      if ((i & 1) != g) continue;
      const int xb = t % nxb, r = t / nxb, yb = r % nyb, f = r / nyb;
      const bool ok = mbar_wait(tfull + g, (uint32_t)(i >> 1) & 1u, abort_flag, a.status, DEV_TIMEOUT_EPILOGUE);
      // the group's four warps leave together (they meet at named barriers below); this is also
      // the point after which the group's previous tile has finished reading the table
      if (!bar_and128(bar_id, ok)) break;
      tc_fence_after();
      uint32_t v0[32], v1[32];
      const uint32_t tb = tmem_base + ((uint32_t)(q * 32) << 16) + (uint32_t)(g * 64);
      tmem_ld32(tb, v0);
      tmem_ld32(tb + 32, v1);
      tmem_ld_wait();
      tc_fence_before();
      mbar_arrive(tempty + g);
#pragma unroll
      for (int j = 0; j < 27; ++j) tab[p * 27 + j] = __uint_as_float(v0[j]);
      if (p + 128 < REGION) {
#pragma unroll
        for (int j = 0; j < 27; ++j) tab[(p + 128) * 27 + j] = __uint_as_float(v1[j]);
      }
      asm volatile("bar.sync %0, 128;" ::"r"(bar_id) : "memory");
      const int y = yb * 8 + yl, x = xb * 16 + xl;
      if (y < a.H) {
        float o[3] = {0.f, 0.f, 0.f};
#pragma unroll
        for (int tap = 0; tap < 9; ++tap) {
          const int rr = (yl + tap / 3) * 18 + xl + tap % 3;
#pragma unroll
          for (int c = 0; c < 3; ++c) o[c] += tab[rr * 27 + tap * 3 + c];
        }
        float* out = a.rgb + (size_t)f * 3 * plane + (size_t)y * a.W + x;
#pragma unroll
        for (int c = 0; c < 3; ++c) {
          const float u = fminf(fmaxf(round_h(o[c] + bias[c]), 0.f), 1.f);
          out[c * plane] = u * 2.f - 1.f;
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) tmem_dealloc(tmem_base, 128);
}

int launch_rgb(const CUtensorMap& x, const CUtensorMap& w, const ConvArgs& a, cudaStream_t s) {
  if (cudaFuncSetAttribute(rgb_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, rgbk::SMEM) != cudaSuccess)
    return FW_ECUDA;
  const int tiles = a.T * ((a.H + 7) / 8) * (a.W / 16);
  launch_k(rgb_kernel, tiles < num_sms() ? tiles : num_sms(), 320, rgbk::SMEM, s, x, w, a);
  return cudaGetLastError() == cudaSuccess ? 0 : FW_ECUDA;
}

// One launch of the decoder's plan.
constexpr int EK_RGB = 2;   // the plan's last conv: rgb_kernel
struct Conv {
  int bn = 0, ek = EK_STORE, lm = LM_TAP;
  CUtensorMap x{}, m{}, w{}, y{};
  ConvArgs a{};
};

}  // namespace taehv

}  // namespace fw

// ------------------------------------------------------------------------------- handle
struct fw_taehv {
  fw_taehv_config cfg{};
  int device = 0;
  struct Tensor {
    std::string name;
    int kind, dtype, ndim;
    int64_t shape[5];
    size_t bytes;
    void* ptr = nullptr;
  };
  std::vector<Tensor> tensors;
  bool finalized = false;
  void* work = nullptr;   // activations (the bound "work" tensor)
  int* status = nullptr;
  // plan
  int T0 = 0, h = 0, w = 0;
  int C[4] = {0, 0, 0, 0}, F[4] = {0, 0, 0, 0};
  __half* im = nullptr;
  std::vector<fw::taehv::Conv> convs;
  fw::taehv::SegCopy mem_update{};
  int mem_blocks = 0;
};

namespace {

using fw::taehv::Conv;

// Activation buffers, in order: the first conv's neighbourhood tensor, per stage 3 block inputs,
// 2 temporaries and the stage output, the three upsampled TGrow outputs, the last conv's input.
std::vector<size_t> work_layout(const fw_taehv* h, size_t* total) {
  std::vector<size_t> sizes, off;
  sizes.push_back((size_t)h->T0 * h->h * h->w * 192 * 2);
  auto stage_bytes = [&](int s, int Cc) { return (size_t)h->F[s] * (h->h << s) * (h->w << s) * Cc * 2; };
  for (int s = 0; s < 3; ++s)
    for (int k = 0; k < 6; ++k) sizes.push_back(stage_bytes(s, h->C[s]));
  for (int s = 0; s < 3; ++s) sizes.push_back(stage_bytes(s + 1, h->C[s]));
  sizes.push_back(stage_bytes(3, h->C[3]));
  size_t t = 0;
  for (size_t b : sizes) {
    off.push_back(t);
    t += (b + 1023) & ~(size_t)1023;
  }
  *total = t;
  return off;
}

int find(const fw_taehv* h, const char* name) {
  for (size_t i = 0; i < h->tensors.size(); ++i)
    if (h->tensors[i].name == name) return (int)i;
  return -1;
}

void add(fw_taehv* h, const std::string& name, int kind, int dtype, std::initializer_list<int64_t> shape) {
  fw_taehv::Tensor t;
  t.name = name;
  t.kind = kind;
  t.dtype = dtype;
  t.ndim = (int)shape.size();
  size_t n = 1;
  int i = 0;
  for (int64_t d : shape) {
    t.shape[i++] = d;
    n *= (size_t)d;
  }
  for (; i < 5; ++i) t.shape[i] = 0;
  t.bytes = n * (dtype == FW_F32 || dtype == FW_I32 ? 4 : (dtype == FW_U8 ? 1 : 2));
  h->tensors.push_back(t);
}

void* ptr(fw_taehv* h, const std::string& name) { return h->tensors[find(h, name.c_str())].ptr; }

}  // namespace

extern "C" {

int fw_taehv_create(const fw_taehv_config* cfg, fw_taehv** out) {
  if (!cfg || !out) return FW_EINVAL;
  *out = nullptr;
  const fw_taehv_config& c = *cfg;
  if (c.lat_ch != 16 || c.lat_frames < 1 || c.lat_h < 8 || c.lat_w < 16 || c.lat_w % 16) return FW_ESHAPE;
  for (int s = 0; s < 4; ++s)
    if (c.channels[s] < 64 || c.channels[s] % 64 || c.channels[s] > 256) return FW_ESHAPE;
  for (int s = 0; s < 3; ++s) {   // TGrow widths: 64, 128, 256 or a multiple of 256
    const int n = c.channels[s] * c.time_up[s];
    if (c.time_up[s] < 1 || c.time_up[s] > 4 || (n > 256 && n % 256)) return FW_ESHAPE;
  }
  fw_taehv* h = new fw_taehv();
  h->cfg = c;
  cudaGetDevice(&h->device);
  h->T0 = c.lat_frames;
  h->h = c.lat_h;
  h->w = c.lat_w;
  for (int s = 0; s < 4; ++s) h->C[s] = c.channels[s];
  h->F[0] = c.lat_frames;
  for (int s = 0; s < 3; ++s) h->F[s + 1] = h->F[s] * c.time_up[s];
  // weights (fp16, [Cout, taps * Cin], K ordered (tap, input channel)) and fp32 biases
  add(h, "conv_in.w", FW_KIND_WEIGHT, FW_F16, {h->C[0], 192});
  add(h, "conv_in.b", FW_KIND_WEIGHT, FW_F32, {h->C[0]});
  for (int s = 0; s < 3; ++s) {
    const int Cs = h->C[s];
    for (int k = 0; k < 3; ++k) {
      const std::string p = "mb" + std::to_string(s * 3 + k);
      add(h, p + ".w0", FW_KIND_WEIGHT, FW_F16, {Cs, 9 * 2 * Cs});
      add(h, p + ".b0", FW_KIND_WEIGHT, FW_F32, {Cs});
      add(h, p + ".w1", FW_KIND_WEIGHT, FW_F16, {Cs, 9 * Cs});
      add(h, p + ".b1", FW_KIND_WEIGHT, FW_F32, {Cs});
      add(h, p + ".w2", FW_KIND_WEIGHT, FW_F16, {Cs, 9 * Cs});
      add(h, p + ".b2", FW_KIND_WEIGHT, FW_F32, {Cs});
    }
    add(h, "tgrow" + std::to_string(s) + ".w", FW_KIND_WEIGHT, FW_F16, {(int64_t)Cs * c.time_up[s], Cs});
    add(h, "conv" + std::to_string(s) + ".w", FW_KIND_WEIGHT, FW_F16, {h->C[s + 1], 9 * Cs});
  }
  add(h, "conv_out.wt", FW_KIND_WEIGHT, FW_F16, {32, h->C[3]});
  add(h, "conv_out.b", FW_KIND_WEIGHT, FW_F32, {32});
  add(h, "lat", FW_KIND_INPUT, FW_F16, {16, h->T0, h->h, h->w});
  add(h, "rgb", FW_KIND_OUTPUT, FW_F32, {h->F[3], 3, (int64_t)h->h * 8, (int64_t)h->w * 8});
  int64_t mem = 0;
  for (int s = 0; s < 3; ++s) mem += 3LL * h->C[s] * ((int64_t)h->h << s) * ((int64_t)h->w << s);
  add(h, "mem", FW_KIND_STATE, FW_F16, {mem});
  size_t work = 0;
  work_layout(h, &work);
  add(h, "work", FW_KIND_WORKSPACE, FW_U8, {(int64_t)work});
  add(h, "status", FW_KIND_STATUS, FW_I32, {4});
  *out = h;
  return FW_OK;
}

int fw_taehv_tensor_count(const fw_taehv* h) { return h ? (int)h->tensors.size() : FW_EINVAL; }

int fw_taehv_tensor_info_at(const fw_taehv* h, int index, fw_tensor_info* info) {
  if (!h || !info || index < 0 || index >= (int)h->tensors.size()) return FW_EINVAL;
  const auto& t = h->tensors[index];
  info->name = t.name.c_str();
  info->kind = t.kind;
  info->dtype = t.dtype;
  info->ndim = t.ndim;
  for (int i = 0; i < 5; ++i) info->shape[i] = t.shape[i];
  info->bytes = t.bytes;
  return FW_OK;
}

int fw_taehv_bind(fw_taehv* h, const char* name, void* p, size_t bytes) {
  if (!h || !name || !p || h->finalized) return FW_EINVAL;
  const int i = find(h, name);
  if (i < 0) return FW_EINVAL;
  if (bytes < h->tensors[i].bytes) return FW_ESIZE;
  if (reinterpret_cast<uintptr_t>(p) & 15u) return FW_EALIGN;
  h->tensors[i].ptr = p;
  return FW_OK;
}

int fw_taehv_finalize(fw_taehv* h) {
  using namespace fw::taehv;
  if (!h || h->finalized) return FW_EINVAL;
  for (const auto& t : h->tensors)
    if (!t.ptr) return FW_ENOTBOUND;
  size_t total = 0;
  const std::vector<size_t> off = work_layout(h, &total);
  const int T0 = h->T0;
  h->work = ptr(h, "work");
  h->status = static_cast<int*>(ptr(h, "status"));
  auto buf = [&](int i) { return static_cast<char*>(h->work) + off[i]; };
  h->im = reinterpret_cast<__half*>(buf(0));
  // buffers of stage s: in[k] = buf(1 + 6 s + k) (k < 3), tmp a / b = + 3 / + 4, out = + 5
  auto sb = [&](int s, int k) { return reinterpret_cast<__half*>(buf(1 + 6 * s + k)); };
  auto up = [&](int s) { return reinterpret_cast<__half*>(buf(19 + s)); };
  __half* z = reinterpret_cast<__half*>(buf(22));
  char* mem = static_cast<char*>(ptr(h, "mem"));
  int rc = 0;
  auto wmap = [&](CUtensorMap* m, const std::string& name, int rows, int K, int bn) {
    if (!rc) rc = make_map_w(m, ptr(h, name), rows, K, bn);
  };
  // input maps: 8-row boxes for per-tap loads, 10-row boxes (tile + halo) for the halo modes
  auto amap = [&](CUtensorMap* m, const void* p, int s, int Cc, int frames, int lm = LM_TAP) {
    if (!rc) rc = make_map_nhwc(m, p, frames, h->h << s, h->w << s, Cc, 16, lm == LM_TAP ? 8 : 10);
  };
  // 3 x 3 convs with at most 64 output channels are bound by operand traffic from L2: halo
  // loads, and resident weights when they fit (one 64-channel input block)
  auto lm_for = [](int bn, int cpt) { return bn <= 64 ? (cpt == 1 ? LM_HALO_RES : LM_HALO) : LM_TAP; };
  auto omap = [&](CUtensorMap* m, const void* p, int s, int Cc, int frames) {
    if (!rc) rc = make_map_nhwc(m, p, frames, h->h << s, h->w << s, Cc, 16, 2);
  };
  auto bn_for = [](int n) { return n >= 256 ? 256 : (n >= 128 ? 128 : 64); };
  h->convs.clear();
  // first conv: 1 tap over the 192-channel neighbourhood tensor
  {
    Conv c;
    c.bn = bn_for(h->C[0]);
    c.ek = EK_STORE;
    if (!rc) rc = make_map_nhwc(&c.x, h->im, T0, h->h, h->w, 192, 16, 8);
    c.m = c.x;
    wmap(&c.w, "conv_in.w", h->C[0], 192, c.bn);
    omap(&c.y, sb(0, 0), 0, h->C[0], T0);
    c.a = ConvArgs{T0, h->h, h->w, 1, 3, 0, h->C[0], (const float*)ptr(h, "conv_in.b"), nullptr, 1, 0, 0, nullptr,
                   h->status};
    h->convs.push_back(c);
  }
  size_t mem_off = 0;
  h->mem_update = SegCopy{};
  for (int s = 0; s < 3; ++s) {
    const int Cs = h->C[s], Fs = h->F[s], Hs = h->h << s, Ws = h->w << s;
    const size_t frame_bytes = (size_t)Hs * Ws * Cs * 2;
    for (int k = 0; k < 3; ++k) {
      const std::string p = "mb" + std::to_string(s * 3 + k);
      __half* xin = sb(s, k);
      __half* ta = sb(s, 3);
      __half* tbuf = sb(s, 4);
      __half* yout = k < 2 ? sb(s, k + 1) : sb(s, 5);
      const int bn = bn_for(Cs);
      Conv c0, c1, c2;
      // conv over cat[x, past]
      c0.bn = bn;
      c0.lm = lm_for(bn, 2 * Cs / 64);
      amap(&c0.x, xin, s, Cs, Fs, c0.lm);
      if (!rc) rc = make_map_nhwc(&c0.m, mem + mem_off, 1, Hs, Ws, Cs, 16, c0.lm == LM_TAP ? 8 : 10);
      wmap(&c0.w, p + ".w0", Cs, 9 * 2 * Cs, bn);
      omap(&c0.y, ta, s, Cs, Fs);
      c0.a = ConvArgs{Fs, Hs, Ws, 9, Cs / 64, Cs / 64, Cs, (const float*)ptr(h, p + ".b0"), nullptr, 1, 0, 0,
                      nullptr, h->status};
      c1.bn = bn;
      c1.lm = lm_for(bn, Cs / 64);
      amap(&c1.x, ta, s, Cs, Fs, c1.lm);
      c1.m = c1.x;
      wmap(&c1.w, p + ".w1", Cs, 9 * Cs, bn);
      omap(&c1.y, tbuf, s, Cs, Fs);
      c1.a = ConvArgs{Fs, Hs, Ws, 9, Cs / 64, 0, Cs, (const float*)ptr(h, p + ".b1"), nullptr, 1, 0, 0, nullptr,
                      h->status};
      c2.bn = bn;
      c2.lm = lm_for(bn, Cs / 64);
      amap(&c2.x, tbuf, s, Cs, Fs, c2.lm);
      c2.m = c2.x;
      wmap(&c2.w, p + ".w2", Cs, 9 * Cs, bn);
      omap(&c2.y, yout, s, Cs, Fs);
      c2.a = ConvArgs{Fs, Hs, Ws, 9, Cs / 64, 0, Cs, (const float*)ptr(h, p + ".b2"), xin, 1, 0, 0, nullptr,
                      h->status};
      h->convs.push_back(c0);
      h->convs.push_back(c1);
      h->convs.push_back(c2);
      // state update: the block input's last frame
      const int seg = h->mem_update.nseg++;
      h->mem_update.src[seg] = reinterpret_cast<const uint4*>(reinterpret_cast<char*>(xin) + (size_t)(Fs - 1) * frame_bytes);
      h->mem_update.dst[seg] = reinterpret_cast<uint4*>(mem + mem_off);
      h->mem_update.n16[seg] = (long long)(frame_bytes / 16);
      mem_off += frame_bytes;
    }
    // TGrow + 2x upsample into the next resolution, then the conv that changes the width
    {
      const int r = h->cfg.time_up[s], N = Cs * r;
      Conv c;
      c.bn = bn_for(N);
      c.ek = EK_UP;
      amap(&c.x, sb(s, 5), s, Cs, Fs);
      c.m = c.x;
      wmap(&c.w, "tgrow" + std::to_string(s) + ".w", N, Cs, c.bn);
      if (!rc) rc = make_map_nhwc(&c.y, up(s), Fs * r, Hs * 2, Ws * 2, Cs, 32, 1);
      c.a = ConvArgs{Fs, Hs, Ws, 1, Cs / 64, 0, N, nullptr, nullptr, 0, r, Cs, nullptr, h->status};
      h->convs.push_back(c);
    }
    {
      const int Cn = h->C[s + 1], Fn = h->F[s + 1];
      Conv c;
      c.bn = bn_for(Cn);
      c.lm = lm_for(c.bn, Cs / 64);
      amap(&c.x, up(s), s + 1, Cs, Fn, c.lm);
      c.m = c.x;
      wmap(&c.w, "conv" + std::to_string(s) + ".w", Cn, 9 * Cs, c.bn);
      __half* dst = s < 2 ? sb(s + 1, 0) : z;
      omap(&c.y, dst, s + 1, Cn, Fn);
      c.a = ConvArgs{Fn, h->h << (s + 1), h->w << (s + 1), 9, Cs / 64, 0, Cn, nullptr, nullptr, s == 2 ? 1 : 0, 0, 0,
                     nullptr, h->status};
      h->convs.push_back(c);
    }
  }
  {
    Conv c;
    c.bn = 32;
    c.ek = EK_RGB;
    if (h->C[3] != 64) return FW_ESHAPE;   // one 64-channel block of K
    if (!rc) rc = make_map_nhwc(&c.x, z, h->F[3], h->h << 3, h->w << 3, h->C[3], 18, 10);
    c.m = c.x;
    wmap(&c.w, "conv_out.wt", 32, 64, 32);
    c.y = c.x;
    c.a = ConvArgs{h->F[3], h->h << 3, h->w << 3, 9, 1, 0, 3, (const float*)ptr(h, "conv_out.b"), nullptr, 0, 0, 0,
                   (float*)ptr(h, "rgb"), h->status};
    h->convs.push_back(c);
  }
  if (rc) return rc;
  h->finalized = true;
  return FW_OK;
}

int fw_taehv_decode(fw_taehv* h, void* stream) {
  using namespace fw::taehv;
  if (!h || !h->finalized) return FW_EINVAL;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int n = h->T0 * h->h * h->w * 12;
  fw::launch_k(prep_kernel, (n + 255) / 256, 256, 0, s, (const __half*)ptr(h, "lat"), h->im, h->T0, h->h,
               h->w);
  if (cudaGetLastError() != cudaSuccess) return FW_ECUDA;
  for (const Conv& c : h->convs) {
    int rc;
    if (c.ek == EK_UP)
      rc = c.bn == 256 ? launch_conv<256, EK_UP, LM_TAP>(c.x, c.m, c.w, c.y, c.a, s)
           : c.bn == 128 ? launch_conv<128, EK_UP, LM_TAP>(c.x, c.m, c.w, c.y, c.a, s)
                         : launch_conv<64, EK_UP, LM_TAP>(c.x, c.m, c.w, c.y, c.a, s);
    else if (c.ek == EK_RGB)
      rc = launch_rgb(c.x, c.w, c.a, s);
    else if (c.lm == LM_HALO_RES)
      rc = launch_conv<64, EK_STORE, LM_HALO_RES>(c.x, c.m, c.w, c.y, c.a, s);
    else if (c.lm == LM_HALO)
      rc = launch_conv<64, EK_STORE, LM_HALO>(c.x, c.m, c.w, c.y, c.a, s);
    else
      rc = c.bn == 256 ? launch_conv<256, EK_STORE, LM_TAP>(c.x, c.m, c.w, c.y, c.a, s)
           : c.bn == 128 ? launch_conv<128, EK_STORE, LM_TAP>(c.x, c.m, c.w, c.y, c.a, s)
                         : launch_conv<64, EK_STORE, LM_TAP>(c.x, c.m, c.w, c.y, c.a, s);
    if (rc) return rc;
  }
  fw::launch_k(seg_copy_kernel, 2 * fw::num_sms(), 256, 0, s, h->mem_update);
  return cudaGetLastError() == cudaSuccess ? FW_OK : FW_ECUDA;
}

int fw_taehv_status(fw_taehv* h, int* out) {
  if (!h || !out || !h->finalized) return FW_EINVAL;
  return cudaMemcpy(out, h->status, sizeof(int), cudaMemcpyDeviceToHost) == cudaSuccess ? FW_OK : FW_ECUDA;
}

void fw_taehv_destroy(fw_taehv* h) { delete h; }

}  // extern "C"
