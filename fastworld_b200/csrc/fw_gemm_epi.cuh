// GEMM epilogue helpers shared by the one-CTA (gemm.cu) and CTA-pair (gemm2.cu) kernels: a
// thread holds 32 consecutive fp32 accumulator columns of one output row (one tcgen05.ld
// 32x32b.x32) and applies the fused epilogue of GemmEpi to them.
#pragma once
#include "fw_internal.h"
#include "fw_ptx.cuh"

namespace fw {

// bias[col0 .. col0 + 32) (bf16; null = none) and the per-frame fp32 bias of GemmEpi.
__device__ __forceinline__ void add_bias(const GemmEpi& e, const __nv_bfloat16* bias, int frame, int col0,
                                         float (&v)[32]) {
  if (bias) {
    const uint4* bp = reinterpret_cast<const uint4*>(bias + col0);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      uint4 u = __ldg(bp + j);
      float2 f0 = unpack_bf16(u.x), f1 = unpack_bf16(u.y), f2 = unpack_bf16(u.z), f3 = unpack_bf16(u.w);
      v[8 * j + 0] += f0.x; v[8 * j + 1] += f0.y; v[8 * j + 2] += f1.x; v[8 * j + 3] += f1.y;
      v[8 * j + 4] += f2.x; v[8 * j + 5] += f2.y; v[8 * j + 6] += f3.x; v[8 * j + 7] += f3.y;
    }
  }
  if (e.fbias) {
    const float4* fp = reinterpret_cast<const float4*>(e.fbias + (size_t)frame * e.fbias_stride + col0);
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      float4 b = __ldg(fp + j);
      v[4 * j + 0] += b.x; v[4 * j + 1] += b.y; v[4 * j + 2] += b.z; v[4 * j + 3] += b.w;
    }
  }
}

__device__ __forceinline__ void store_bf16x32(__nv_bfloat16* dst, const float (&v)[32]) {
  uint4* d4 = reinterpret_cast<uint4*>(dst);
#pragma unroll
  for (int j = 0; j < 4; ++j)
    d4[j] = make_uint4(pack_bf16(v[8 * j + 0], v[8 * j + 1]), pack_bf16(v[8 * j + 2], v[8 * j + 3]),
                       pack_bf16(v[8 * j + 4], v[8 * j + 5]), pack_bf16(v[8 * j + 6], v[8 * j + 7]));
}

__device__ __forceinline__ void epilogue_chunk(const GemmEpi& e, int row, int col0, const uint32_t (&r)[32],
                                               const float* __restrict__ sa, const float* __restrict__ sw) {
  float v[32];
#pragma unroll
  for (int j = 0; j < 32; ++j) v[j] = __uint_as_float(r[j]);
  if (sa) {   // e4m3 operands: dequantise with the row's activation scale and each column's weight scale
    const float ra = __ldg(sa + row);
    const float4* w4 = reinterpret_cast<const float4*>(sw + col0);
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const float4 w = __ldg(w4 + j);
      v[4 * j + 0] *= ra * w.x; v[4 * j + 1] *= ra * w.y; v[4 * j + 2] *= ra * w.z; v[4 * j + 3] *= ra * w.w;
    }
  }
  const int frame = row / e.rows_per_frame;
  add_bias(e, e.bias, frame, col0, v);
  if (e.mode == EPI_BF16 || e.mode == EPI_GELU_BF16 || e.mode == EPI_GELU_ERF_BF16) {
    if (e.mode == EPI_GELU_BF16) {
#pragma unroll
      for (int j = 0; j < 32; ++j) v[j] = gelu_tanh(v[j]);
    } else if (e.mode == EPI_GELU_ERF_BF16) {
#pragma unroll
      for (int j = 0; j < 32; ++j) v[j] = 0.5f * v[j] * (1.f + erff(v[j] * 0.7071067811865476f));
    }
    const int seg = col0 / e.seg_w;
    __nv_bfloat16* dst = reinterpret_cast<__nv_bfloat16*>(e.out[seg]) + (size_t)row * e.ld_out + (col0 - seg * e.seg_w);
    store_bf16x32(dst, v);
  } else if (e.mode == EPI_F32) {
    float4* d4 = reinterpret_cast<float4*>(reinterpret_cast<float*>(e.out[0]) + (size_t)row * e.ld_out + col0);
#pragma unroll
    for (int j = 0; j < 8; ++j) d4[j] = make_float4(v[4 * j], v[4 * j + 1], v[4 * j + 2], v[4 * j + 3]);
  } else {   // EPI_RESID_F32
    float4* rp = reinterpret_cast<float4*>(e.resid + (size_t)row * e.ld_resid + col0);
    const float4* gp = e.gate ? reinterpret_cast<const float4*>(e.gate + (size_t)frame * e.gate_stride + col0) : nullptr;
    float4 x[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) x[j] = rp[j];   // all eight loads in flight before the math
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const float4 g = gp ? __ldg(gp + j) : make_float4(1.f, 1.f, 1.f, 1.f);
      x[j].x += g.x * v[4 * j + 0]; x[j].y += g.y * v[4 * j + 1]; x[j].z += g.z * v[4 * j + 2]; x[j].w += g.w * v[4 * j + 3];
      rp[j] = x[j];
      v[4 * j + 0] = x[j].x; v[4 * j + 1] = x[j].y; v[4 * j + 2] = x[j].z; v[4 * j + 3] = x[j].w;
    }
    if (e.mirror) store_bf16x32(e.mirror + (size_t)row * e.ld_mirror + col0, v);
  }
}

// EPI_RESID_TMA: the warp's 32 rows x 32 columns of gate * (acc + bias) go through a
// 128-byte-swizzled staging box (16-byte chunk c of row l at chunk position c ^ (l % 8), the
// layout TMA expects, 4-way bank spread) and lane 0 adds the box into the fp32 residual with
// one TMA reduce-add; rows past M are dropped by TMA.  No residual read leaves the SM.  `row`
// is clamped to a valid row for the scale / bias / gate reads (its values are discarded).
// With wait = false the box is not reused by the caller, which waits for all its reduce-adds at
// the end (several boxes in flight at once).
__device__ __forceinline__ void epilogue_chunk_tma(const GemmEpi& e, const CUtensorMap* tmC, int row, int row0,
                                                   int col0, const uint32_t (&r)[32], const float* __restrict__ sa,
                                                   const float* __restrict__ sw, uint8_t* box, int lane,
                                                   bool wait = true) {
  float v[32];
#pragma unroll
  for (int j = 0; j < 32; ++j) v[j] = __uint_as_float(r[j]);
  if (sa) {
    const float ra = __ldg(sa + row);
    const float4* w4 = reinterpret_cast<const float4*>(sw + col0);
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const float4 w = __ldg(w4 + j);
      v[4 * j + 0] *= ra * w.x; v[4 * j + 1] *= ra * w.y; v[4 * j + 2] *= ra * w.z; v[4 * j + 3] *= ra * w.w;
    }
  }
  const int frame = row / e.rows_per_frame;
  add_bias(e, e.bias, frame, col0, v);
  if (e.gate) {
    const float4* gp = reinterpret_cast<const float4*>(e.gate + (size_t)frame * e.gate_stride + col0);
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const float4 g = __ldg(gp + j);
      v[4 * j + 0] *= g.x; v[4 * j + 1] *= g.y; v[4 * j + 2] *= g.z; v[4 * j + 3] *= g.w;
    }
  }
  uint8_t* myrow = box + lane * 128;
#pragma unroll
  for (int c = 0; c < 8; ++c)
    *reinterpret_cast<float4*>(myrow + ((c ^ (lane & 7)) << 4)) = make_float4(v[4 * c], v[4 * c + 1], v[4 * c + 2], v[4 * c + 3]);
  fence_proxy_async_smem();
  __syncwarp();
  if (lane == 0) {
    tma_reduce_add_2d(tmC, box, col0, row0);
    bulk_commit();
    if (wait) bulk_wait_read0();   // the box may be rewritten once TMA has read it
  }
  __syncwarp();
}

// Bias / activation / e4m3 scales of one 32-column accumulator chunk (bf16 output modes).
// ACT: the activation fixed at compile time (EPI_BF16 / EPI_GELU_BF16 / EPI_GELU_ERF_BF16), or
// -1 to read it from e.mode.
template <int ACT = -1>
__device__ __forceinline__ void epi_math_bf16(const GemmEpi& e, const __nv_bfloat16* bias, int row, int frame,
                                              int col0, const uint32_t (&r)[32],
                                              const float* __restrict__ sa, const float* __restrict__ sw,
                                              float (&v)[32]) {
  const int act = ACT >= 0 ? ACT : e.mode;
#pragma unroll
  for (int j = 0; j < 32; ++j) v[j] = __uint_as_float(r[j]);
  if (sa) {
    const float ra = __ldg(sa + row);
    const float4* w4 = reinterpret_cast<const float4*>(sw + col0);
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const float4 w = __ldg(w4 + j);
      v[4 * j + 0] *= ra * w.x; v[4 * j + 1] *= ra * w.y; v[4 * j + 2] *= ra * w.z; v[4 * j + 3] *= ra * w.w;
    }
  }
  add_bias(e, bias, frame, col0, v);
  if (act == EPI_GELU_BF16) {
#pragma unroll
    for (int j = 0; j < 32; ++j) v[j] = gelu_tanh(v[j]);
  } else if (act == EPI_GELU_ERF_BF16) {
#pragma unroll
    for (int j = 0; j < 32; ++j) v[j] = 0.5f * v[j] * (1.f + erff(v[j] * 0.7071067811865476f));
  }
}

// bf16 output modes (EPI_BF16 / EPI_GELU_BF16 / EPI_GELU_ERF_BF16): NCH (1 or 2) accumulator
// chunks of the warp's 32 rows become a bf16 box in shared memory (row l's 16-byte piece p at
// position p ^ (l % 8)), then the warp stores the box row-contiguously: with 64 columns, four
// whole 128-byte rows per instruction instead of 32 partial lines (one per thread's row).  `row`
// is clamped for the scale / bias reads; rows >= M and columns >= N are not stored.  The output
// segment (q / k / v of a fused projection) is that of colb: seg_w is a multiple of the tile width.
//
// bias / out_off: the group's bias vector and the element offset added to the output segments
// (a grouped launch); e.bias and 0 otherwise.
template <int NCH>
__device__ __forceinline__ void epilogue_bf16_box(const GemmEpi& e, const __nv_bfloat16* bias, size_t out_off,
                                                  int row, int row0, int colb, int M, int N,
                                                  const uint32_t (*r)[32], const float* __restrict__ sa,
                                                  const float* __restrict__ sw, uint8_t* box, int lane) {
  const int frame = row / e.rows_per_frame;
#pragma unroll
  for (int cc = 0; cc < NCH; ++cc) {
    float v[32];
    epi_math_bf16(e, bias, row, frame, min(colb + cc * 32, N - 32), r[cc], sa, sw, v);
#pragma unroll
    for (int pc = 0; pc < 4; ++pc)
      *reinterpret_cast<uint4*>(box + lane * 128 + (((cc * 4 + pc) ^ (lane & 7)) << 4)) =
          make_uint4(pack_bf16(v[8 * pc + 0], v[8 * pc + 1]), pack_bf16(v[8 * pc + 2], v[8 * pc + 3]),
                     pack_bf16(v[8 * pc + 4], v[8 * pc + 5]), pack_bf16(v[8 * pc + 6], v[8 * pc + 7]));
  }
  __syncwarp();
  constexpr int PPR = 4 * NCH;     // 16-byte pieces per row
  constexpr int RPI = 32 / PPR;    // rows per instruction
  const int seg = colb / e.seg_w, scol = colb - seg * e.seg_w;
  __nv_bfloat16* out = reinterpret_cast<__nv_bfloat16*>(e.out[seg]) + out_off;
#pragma unroll
  for (int it = 0; it < PPR; ++it) {
    const int rr = it * RPI + lane / PPR, p = lane % PPR;
    const uint4 u = *reinterpret_cast<const uint4*>(box + rr * 128 + ((p ^ (rr & 7)) << 4));
    const int grow = row0 + rr;
    if (grow < M && colb + p * 8 < N) *reinterpret_cast<uint4*>(out + (size_t)grow * e.ld_out + scol + p * 8) = u;
  }
  __syncwarp();
}

// The same bf16 box written by one TMA store (lane 0) through the output tensor map `om` of the
// column segment: the TMA engine carries the global writes, so the warp is free as soon as the
// store has read the box (an st.global epilogue is limited by the stores an SM keeps in flight:
// about 13 GB/s per SM, 2 TB/s for the whole GPU, measured).  Rows >= M and columns past the
// segment are clipped by TMA.  The box is reused only after the previous store read it.
template <int NCH, int ACT>
__device__ __forceinline__ void epilogue_bf16_tma(const GemmEpi& e, const CUtensorMap* om, int row, int row0,
                                                  int colb, int N, const uint32_t (*r)[32],
                                                  const float* __restrict__ sa, const float* __restrict__ sw,
                                                  uint8_t* box, int lane) {
  const int frame = row / e.rows_per_frame;
  if (lane == 0) bulk_wait_read0();   // this warp's previous store has read the box
  __syncwarp();
#pragma unroll
  for (int cc = 0; cc < NCH; ++cc) {
    float v[32];
    epi_math_bf16<ACT>(e, e.bias, row, frame, min(colb + cc * 32, N - 32), r[cc], sa, sw, v);
#pragma unroll
    for (int pc = 0; pc < 4; ++pc)
      *reinterpret_cast<uint4*>(box + lane * 128 + (((cc * 4 + pc) ^ (lane & 7)) << 4)) =
          make_uint4(pack_bf16(v[8 * pc + 0], v[8 * pc + 1]), pack_bf16(v[8 * pc + 2], v[8 * pc + 3]),
                     pack_bf16(v[8 * pc + 4], v[8 * pc + 5]), pack_bf16(v[8 * pc + 6], v[8 * pc + 7]));
  }
  fence_proxy_async_smem();
  __syncwarp();
  if (lane == 0) {
    const int seg = colb / e.seg_w;
    tma_store_2d(om, box, colb - seg * e.seg_w, row0);
    bulk_commit();
  }
}

// EPI_RESID_F32 (with or without a bf16 mirror): the warp's 32 rows x 32 columns of
// gate * (acc + bias) go through a swizzled fp32 box; then each instruction updates four whole
// 128-byte residual rows (8 lanes per row, 16 bytes each: coalesced read-modify-write, all eight
// loads issued before the epilogue math) and writes the matching 64-byte pieces of the bf16 mirror.
// `row` is clamped for the scale / bias / gate reads; rows >= M are not touched.
__device__ __forceinline__ void epilogue_resid_box(const GemmEpi& e, int row, int row0, int col0, int M,
                                                   const uint32_t (&r)[32], const float* __restrict__ sa,
                                                   const float* __restrict__ sw, uint8_t* box, int lane) {
  // the residual loads go out first: their latency overlaps the scale / bias / gate math
  const int p = lane & 7, gcol = col0 + p * 4;
  float4 x[8];
#pragma unroll
  for (int it = 0; it < 8; ++it) {
    const int grow = row0 + it * 4 + (lane >> 3);
    if (grow < M) x[it] = *reinterpret_cast<const float4*>(e.resid + (size_t)grow * e.ld_resid + gcol);
  }
  float v[32];
#pragma unroll
  for (int j = 0; j < 32; ++j) v[j] = __uint_as_float(r[j]);
  if (sa) {
    const float ra = __ldg(sa + row);
    const float4* w4 = reinterpret_cast<const float4*>(sw + col0);
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const float4 w = __ldg(w4 + j);
      v[4 * j + 0] *= ra * w.x; v[4 * j + 1] *= ra * w.y; v[4 * j + 2] *= ra * w.z; v[4 * j + 3] *= ra * w.w;
    }
  }
  const int frame = row / e.rows_per_frame;
  add_bias(e, e.bias, frame, col0, v);
  if (e.gate) {
    const float4* gp = reinterpret_cast<const float4*>(e.gate + (size_t)frame * e.gate_stride + col0);
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const float4 g = __ldg(gp + j);
      v[4 * j + 0] *= g.x; v[4 * j + 1] *= g.y; v[4 * j + 2] *= g.z; v[4 * j + 3] *= g.w;
    }
  }
#pragma unroll
  for (int c = 0; c < 8; ++c)
    *reinterpret_cast<float4*>(box + lane * 128 + ((c ^ (lane & 7)) << 4)) =
        make_float4(v[4 * c], v[4 * c + 1], v[4 * c + 2], v[4 * c + 3]);
  __syncwarp();
#pragma unroll
  for (int it = 0; it < 8; ++it) {
    const int rr = it * 4 + (lane >> 3), grow = row0 + rr;
    if (grow < M) {
      const float4 u = *reinterpret_cast<const float4*>(box + rr * 128 + ((p ^ (rr & 7)) << 4));
      x[it].x += u.x; x[it].y += u.y; x[it].z += u.z; x[it].w += u.w;
      *reinterpret_cast<float4*>(e.resid + (size_t)grow * e.ld_resid + gcol) = x[it];
      if (e.mirror)
        *reinterpret_cast<uint2*>(e.mirror + (size_t)grow * e.ld_mirror + gcol) =
            make_uint2(pack_bf16(x[it].x, x[it].y), pack_bf16(x[it].z, x[it].w));
    }
  }
  __syncwarp();
}

// EPI_BF16_PUSH: 64 columns (two accumulator chunks) of the warp's 32 rows become a 32 x 128-byte
// bf16 box in shared memory (16-byte piece p of row l at position p ^ (l % 8): conflict-free
// writes by row, conflict-free reads by 8 lanes per row), then the warp stores the box
// row-contiguously, four rows (512 bytes) per instruction, to out[0] and to the other GPUs
// (peer_out, or the row's owner for push_tp > 2), so the remote stores cross NVLink as whole
// 128-byte lines.  `row` is clamped for
// the bias read; rows >= M and columns >= N are not stored.
__device__ __forceinline__ void epilogue_push64(const GemmEpi& e, int row, int row0, int colb, int M, int N,
                                                const uint32_t (&r0)[32], const uint32_t (&r1)[32], uint8_t* box,
                                                int lane) {
  const int frame = row / e.rows_per_frame;
#pragma unroll
  for (int cc = 0; cc < 2; ++cc) {
    float v[32];
    const uint32_t (&r)[32] = cc ? r1 : r0;
#pragma unroll
    for (int j = 0; j < 32; ++j) v[j] = __uint_as_float(r[j]);
    if (colb + cc * 32 < N) add_bias(e, e.bias, frame, colb + cc * 32, v);
#pragma unroll
    for (int pc = 0; pc < 4; ++pc) {
      const int piece = cc * 4 + pc;
      *reinterpret_cast<uint4*>(box + lane * 128 + ((piece ^ (lane & 7)) << 4)) =
          make_uint4(pack_bf16(v[8 * pc + 0], v[8 * pc + 1]), pack_bf16(v[8 * pc + 2], v[8 * pc + 3]),
                     pack_bf16(v[8 * pc + 4], v[8 * pc + 5]), pack_bf16(v[8 * pc + 6], v[8 * pc + 7]));
    }
  }
  __syncwarp();
#pragma unroll
  for (int it = 0; it < 8; ++it) {
    const int rr = it * 4 + (lane >> 3), p = lane & 7;
    const uint4 u = *reinterpret_cast<const uint4*>(box + rr * 128 + ((p ^ (rr & 7)) << 4));
    const int grow = row0 + rr, gcol = colb + p * 8;
    if (grow < M && gcol < N) {
      const size_t off = (size_t)grow * e.ld_out + gcol;
      *reinterpret_cast<uint4*>(reinterpret_cast<__nv_bfloat16*>(e.out[0]) + off) = u;
      if (e.peer_out) {
        *reinterpret_cast<uint4*>(e.peer_out + off) = u;
      } else {   // reduce-scatter: the row's owner gets it in this rank's slot
        const int j = grow / e.push_ls;
        if (j != e.push_rank)
          *reinterpret_cast<uint4*>(e.push_base[j] + ((size_t)e.push_rank * e.push_ls + grow - j * e.push_ls) *
                                                         e.ld_out + gcol) = u;
      }
    }
  }
  __syncwarp();
}

}  // namespace fw
