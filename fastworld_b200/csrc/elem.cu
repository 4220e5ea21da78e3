// Fused memory-bound kernels of the chunk forward (sm_100a).  All are HBM/L2-bound row
// kernels: one warp per row (or per (token, head)), 16-byte vector access, fp32 math.
//
// Reference ops replaced (fastworld/models/mg2/static.py):
//   ln_kernel            norm1/norm2 + adaLN modulate (206, 224), norm3 (221), img_emb LNs (201),
//                        mouse_mlp LayerNorm (150)
//   rms_rope_kernel      norm_q / norm_k (208-209, 189-190) fused with the fp64 complex RoPE
//                        (_rope, 130-133; computed here in fp32 from an fp64-built table)
//   rope_table_kernel    the per-chunk RoPE table fi (113-118) and action RoPE acos/asin (120)
//   smallm_linear(8)_kernel time_embedding / time_projection (199-200), keyboard_embed and
//                        keyboard_attn_kv (165-168), the mouse-window part of mouse_mlp (150)
//   patchify_kernel      cat([x, cc]) + Conv3d(k = s = (1,2,2)) operand layout (197-198)
//   scheduler_kernel     unpatchify + _convert_flow_pred_to_x0 + add_noise (227-240)
//   mouse_attn_kernel    mouse branch of _action: RMSNorm + rotate-half RoPE + attention over
//                        [mk | current] frames + history write (151-161)
//   kb_kv_kernel         keyboard K/V norm + RoPE (171-175)
//   kb_attn_kernel       keyboard attention over [kk | current] (173-184)
#include <cuda_fp8.h>
#include <math.h>

#include "../../include/fastworld_b200.h"
#include "fw_elem.h"
#include "fw_ptx.cuh"

namespace fw {

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

__device__ __forceinline__ void load4(const float* p, float (&v)[4]) {
  float4 u = *reinterpret_cast<const float4*>(p);
  v[0] = u.x; v[1] = u.y; v[2] = u.z; v[3] = u.w;
}
__device__ __forceinline__ void load4(const __nv_bfloat16* p, float (&v)[4]) {
  uint2 u = *reinterpret_cast<const uint2*>(p);
  float2 a = unpack_bf16(u.x), b = unpack_bf16(u.y);
  v[0] = a.x; v[1] = a.y; v[2] = b.x; v[3] = b.y;
}
__device__ __forceinline__ void store4(__nv_bfloat16* p, const float (&v)[4]) {
  *reinterpret_cast<uint2*>(p) = make_uint2(pack_bf16(v[0], v[1]), pack_bf16(v[2], v[3]));
}

// ------------------------------------------------------------------ LayerNorm
// out = LN(x) [* w + b] [* (1 + scale) + shift], one warp per row, D = 128 * NG.
// Four floats -> four e4m3 bytes (memory order) after multiplying by `inv`, saturating.
__device__ __forceinline__ uint32_t pack4_e4m3(float a, float b, float c, float d, float inv) {
  const uint32_t lo = __nv_cvt_float2_to_fp8x2(make_float2(a * inv, b * inv), __NV_SATFINITE, __NV_E4M3);
  const uint32_t hi = __nv_cvt_float2_to_fp8x2(make_float2(c * inv, d * inv), __NV_SATFINITE, __NV_E4M3);
  return lo | (hi << 16);
}

template <typename Tin, int NG>
// At most 85 registers (three blocks per SM): the 2640 rows of a chunk then run in one wave of
// warps (at 127 registers only two blocks fit and 34 of the 330 blocks formed a second wave).
__global__ void __launch_bounds__(256, 3) ln_kernel(const Tin* __restrict__ x, int ldx, int M, float eps,
                                                 const float* __restrict__ shift, const float* __restrict__ scale,
                                                 const __nv_bfloat16* __restrict__ w,
                                                 const __nv_bfloat16* __restrict__ b, __nv_bfloat16* __restrict__ out,
                                                 int ldo, uint8_t* __restrict__ out8, float* __restrict__ sa) {
  pdl_trigger();
  pdl_wait();
  const int row = blockIdx.x * 8 + (threadIdx.x >> 5), lane = threadIdx.x & 31;
  const bool live = row < M;
  constexpr int D = 128 * NG;
  float v[NG][4];
  if (live) {   // the row's loads go out first
#pragma unroll
    for (int g = 0; g < NG; ++g) load4(x + (size_t)row * ldx + g * 128 + lane * 4, v[g]);
  }
  // The per-column vectors (1 + scale and shift, or w and b) are staged in shared memory by the
  // whole block while the row loads are in flight, so the second half of the kernel reads them
  // from shared memory instead of making a second round trip to L2 per warp.  With both an
  // affine and a modulation (no caller of this engine) they are read from global memory.
  const bool staged = (scale != nullptr) != (w != nullptr);
  __shared__ float4 s_a[32 * NG], s_b[32 * NG];
  if (staged) {
    for (int i = threadIdx.x; i < 32 * NG; i += blockDim.x) {
      float a4[4], b4[4];
      if (scale) {
        load4(scale + 4 * i, a4);
        load4(shift + 4 * i, b4);
#pragma unroll
        for (int k = 0; k < 4; ++k) a4[k] = 1.f + a4[k];
      } else {
        load4(w + 4 * i, a4);
        load4(b + 4 * i, b4);
      }
      s_a[i] = make_float4(a4[0], a4[1], a4[2], a4[3]);
      s_b[i] = make_float4(b4[0], b4[1], b4[2], b4[3]);
    }
    __syncthreads();
  }
  if (!live) return;
  float s = 0.f;
#pragma unroll
  for (int g = 0; g < NG; ++g) s += v[g][0] + v[g][1] + v[g][2] + v[g][3];
  const float mean = warp_sum(s) * (1.f / D);
  float q = 0.f;
#pragma unroll
  for (int g = 0; g < NG; ++g)
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float d = v[g][i] - mean;
      q += d * d;
    }
  const float rstd = rsqrtf(warp_sum(q) * (1.f / D) + eps);
  float amax = 0.f;
#pragma unroll
  for (int g = 0; g < NG; ++g) {
    const int c = g * 128 + lane * 4;
    float* y = v[g];
#pragma unroll
    for (int i = 0; i < 4; ++i) y[i] = (y[i] - mean) * rstd;
    if (staged) {   // y * (1 + scale) + shift, or y * w + b
      const float4 A = s_a[g * 32 + lane], B = s_b[g * 32 + lane];
      y[0] = y[0] * A.x + B.x;
      y[1] = y[1] * A.y + B.y;
      y[2] = y[2] * A.z + B.z;
      y[3] = y[3] * A.w + B.w;
    } else if (w) {
      float wv[4], bv[4];
      load4(w + c, wv);
      load4(b + c, bv);
#pragma unroll
      for (int i = 0; i < 4; ++i) y[i] = y[i] * wv[i] + bv[i];
    }
    if (!staged && scale) {
      float sc[4], sh[4];
      load4(scale + c, sc);
      load4(shift + c, sh);
#pragma unroll
      for (int i = 0; i < 4; ++i) y[i] = y[i] * (1.f + sc[i]) + sh[i];
    }
    if (out8) {
#pragma unroll
      for (int i = 0; i < 4; ++i) amax = fmaxf(amax, fabsf(y[i]));
    } else {
      store4(out + (size_t)row * ldo + c, v[g]);
    }
  }
  if (out8) {   // e4m3 output with a per-row scale absmax / 448
    amax = warp_max(amax);
    const float sc = amax > 0.f ? amax * (1.f / 448.f) : 1.f;
    const float inv = 1.f / sc;
#pragma unroll
    for (int g = 0; g < NG; ++g)
      *reinterpret_cast<uint32_t*>(out8 + (size_t)row * ldo + g * 128 + lane * 4) =
          pack4_e4m3(v[g][0], v[g][1], v[g][2], v[g][3], inv);
    if (lane == 0) sa[row] = sc;
  }
}

// Eight consecutive elements into registers (16-byte loads).
__device__ __forceinline__ void load8(const float* p, float (&v)[8]) {
  const float4 a = *reinterpret_cast<const float4*>(p), b = *reinterpret_cast<const float4*>(p + 4);
  v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w; v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
}
__device__ __forceinline__ void load8(const __nv_bfloat16* p, float (&v)[8]) {
  const uint4 u = *reinterpret_cast<const uint4*>(p);
  const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 f = unpack_bf16(w[i]);
    v[2 * i] = f.x;
    v[2 * i + 1] = f.y;
  }
}

// LayerNorm of wide rows (D = 1024 * NG): a row is shared by four warps of D / 4 columns each,
// so that no lane holds more than 40 values (one warp per row, as ln_kernel does, spills for
// D = 5120); the four warps' partial sums meet in shared memory.  Lane l of a warp reads, in each
// 256-column group of its part, the 16-byte chunks at columns l * 4 and 128 + l * 4 (two fully
// coalesced 512-byte requests per warp) and writes its bf16 results at the same columns.  Same
// arithmetic as ln_kernel.
template <typename Tin, int NG>
__global__ void __launch_bounds__(256, 3) ln_wide_kernel(const Tin* __restrict__ x, int ldx, int M, float eps,
                                                      const float* __restrict__ shift, const float* __restrict__ scale,
                                                      const __nv_bfloat16* __restrict__ w,
                                                      const __nv_bfloat16* __restrict__ b,
                                                      __nv_bfloat16* __restrict__ out, int ldo) {
  pdl_trigger();
  pdl_wait();
  constexpr int WPR = 4, ROWS = 8 / WPR, D = 1024 * NG;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int row = blockIdx.x * ROWS + warp / WPR, part = warp % WPR;
  const bool live = row < M;
  const int base = part * 256 * NG + lane * 4;   // + g * 256 + h * 128
  float v[NG][2][4];
  if (live) {
#pragma unroll
    for (int g = 0; g < NG; ++g)
#pragma unroll
      for (int h = 0; h < 2; ++h) load4(x + (size_t)row * ldx + base + g * 256 + h * 128, v[g][h]);
  }
  // per-column vectors staged in shared memory while the row loads are in flight
  const bool staged = (scale != nullptr) != (w != nullptr);
  __shared__ float4 s_a[D / 4], s_b[D / 4];
  __shared__ float s_red[2][8];
  if (staged) {
    for (int i = threadIdx.x; i < D / 4; i += blockDim.x) {
      float a4[4], b4[4];
      if (scale) {
        load4(scale + 4 * i, a4);
        load4(shift + 4 * i, b4);
#pragma unroll
        for (int k = 0; k < 4; ++k) a4[k] = 1.f + a4[k];
      } else {
        load4(w + 4 * i, a4);
        load4(b + 4 * i, b4);
      }
      s_a[i] = make_float4(a4[0], a4[1], a4[2], a4[3]);
      s_b[i] = make_float4(b4[0], b4[1], b4[2], b4[3]);
    }
  }
  auto row_sum = [&](float t, int k) {   // every thread of the block calls this
    t = warp_sum(t);
    if (lane == 0) s_red[k][warp] = t;
    __syncthreads();
    float r = 0.f;
#pragma unroll
    for (int p = 0; p < WPR; ++p) r += s_red[k][(warp / WPR) * WPR + p];
    return r;
  };
  float s = 0.f;
  if (live) {
#pragma unroll
    for (int g = 0; g < NG; ++g)
#pragma unroll
      for (int i = 0; i < 8; ++i) s += v[g][i >> 2][i & 3];
  }
  const float mean = row_sum(s, 0) * (1.f / D);
  float q = 0.f;
  if (live) {
#pragma unroll
    for (int g = 0; g < NG; ++g)
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const float d = v[g][i >> 2][i & 3] - mean;
        q += d * d;
      }
  }
  const float rstd = rsqrtf(row_sum(q, 1) * (1.f / D) + eps);
  if (!live) return;
#pragma unroll
  for (int g = 0; g < NG; ++g)
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const int c = base + g * 256 + h * 128;
      float(&y)[4] = v[g][h];
#pragma unroll
      for (int i = 0; i < 4; ++i) y[i] = (y[i] - mean) * rstd;
      if (staged) {   // y * (1 + scale) + shift, or y * w + b
        const float4 A = s_a[c / 4], B = s_b[c / 4];
        y[0] = y[0] * A.x + B.x;
        y[1] = y[1] * A.y + B.y;
        y[2] = y[2] * A.z + B.z;
        y[3] = y[3] * A.w + B.w;
      } else {
        if (w) {
          float wv[4], bv[4];
          load4(w + c, wv);
          load4(b + c, bv);
#pragma unroll
          for (int i = 0; i < 4; ++i) y[i] = y[i] * wv[i] + bv[i];
        }
        if (scale) {
          float sc[4], sh[4];
          load4(scale + c, sc);
          load4(shift + c, sh);
#pragma unroll
          for (int i = 0; i < 4; ++i) y[i] = y[i] * (1.f + sc[i]) + sh[i];
        }
      }
      store4(out + (size_t)row * ldo + c, y);
    }
}

template <typename Tin>
static int ln_dispatch(const Tin* x, int ldx, int M, int D, float eps, const float* shift, const float* scale,
                       const __nv_bfloat16* w, const __nv_bfloat16* b, __nv_bfloat16* out, int ldo, cudaStream_t s,
                       uint8_t* out8 = nullptr, float* sa = nullptr) {
  if (D % 128 || ldx % 4 || ldo % 4 || (out8 && !sa)) return FW_ESHAPE;
  const dim3 grid((M + 7) / 8), block(256);
  if (!out8 && D % 1024 == 0 && D > 1536) {   // wide rows: four warps per row
    switch (D / 1024) {
#define FW_LNW_CASE(n)                                                                                   \
  case n:                                                                                                \
    launch_k(ln_wide_kernel<Tin, n>, dim3((M + 1) / 2), block, 0, s, x, ldx, M, eps, shift, scale, w, b, out, \
             ldo);                                                                                       \
    return cudaGetLastError() == cudaSuccess ? 0 : FW_ECUDA;
      FW_LNW_CASE(2) FW_LNW_CASE(3) FW_LNW_CASE(4) FW_LNW_CASE(5)
#undef FW_LNW_CASE
      default: break;
    }
  }
  switch (D / 128) {
#define FW_LN_CASE(n) \
  case n: launch_k(ln_kernel<Tin, n>, grid, block, 0, s, x, ldx, M, eps, shift, scale, w, b, out, ldo, out8, sa); break;
    FW_LN_CASE(1) FW_LN_CASE(2) FW_LN_CASE(3) FW_LN_CASE(4) FW_LN_CASE(5) FW_LN_CASE(6) FW_LN_CASE(7)
    FW_LN_CASE(8) FW_LN_CASE(9) FW_LN_CASE(10) FW_LN_CASE(11) FW_LN_CASE(12) FW_LN_CASE(16) FW_LN_CASE(40)
#undef FW_LN_CASE
    default: return FW_ESHAPE;
  }
  return cudaGetLastError() == cudaSuccess ? 0 : FW_ECUDA;
}

int ln_f32(const float* x, int ldx, int M, int D, float eps, const float* shift, const float* scale,
           const __nv_bfloat16* w, const __nv_bfloat16* b, __nv_bfloat16* out, int ldo, cudaStream_t s) {
  return ln_dispatch<float>(x, ldx, M, D, eps, shift, scale, w, b, out, ldo, s);
}
int ln_bf16(const __nv_bfloat16* x, int ldx, int M, int D, float eps, const float* shift, const float* scale,
            const __nv_bfloat16* w, const __nv_bfloat16* b, __nv_bfloat16* out, int ldo, cudaStream_t s) {
  return ln_dispatch<__nv_bfloat16>(x, ldx, M, D, eps, shift, scale, w, b, out, ldo, s);
}
int ln_f32_q8(const float* x, int ldx, int M, int D, float eps, const float* shift, const float* scale,
              const __nv_bfloat16* w, const __nv_bfloat16* b, uint8_t* out8, float* sa, int ldo, cudaStream_t s) {
  return ln_dispatch<float>(x, ldx, M, D, eps, shift, scale, w, b, nullptr, ldo, s, out8, sa);
}
int ln_bf16_q8(const __nv_bfloat16* x, int ldx, int M, int D, float eps, const float* shift, const float* scale,
               const __nv_bfloat16* w, const __nv_bfloat16* b, uint8_t* out8, float* sa, int ldo, cudaStream_t s) {
  return ln_dispatch<__nv_bfloat16>(x, ldx, M, D, eps, shift, scale, w, b, nullptr, ldo, s, out8, sa);
}

// ------------------------------------------------------------------ e4m3 row quantisation
// q[row, :] = e4m3(x[row, :] / scale[row]), scale = absmax(x[row, :]) / 448 (1 for an all-zero row).
// Per-token activation scales for the e4m3 GEMMs, and per-output-channel weight scales when
// applied to a weight [N, K].  One warp per row, two passes (the second hits L1/L2).
__global__ void __launch_bounds__(256) quant_rows_kernel(const __nv_bfloat16* __restrict__ x, int ldx, int M, int K,
                                                         uint8_t* __restrict__ q, int ldq, float* __restrict__ scale) {
  pdl_trigger();
  pdl_wait();
  const int row = blockIdx.x * 8 + (threadIdx.x >> 5), lane = threadIdx.x & 31;
  if (row >= M) return;
  const __nv_bfloat16* xr = x + (size_t)row * ldx;
  // both passes issue eight 16-byte loads per lane before using them (a row of the FFN hidden
  // layer is 35 such steps; one load at a time made the kernel latency-bound)
  constexpr int U = 8;
  float amax = 0.f;
  for (int c0 = lane * 8; c0 < K; c0 += 256 * U) {
    uint4 u[U];
#pragma unroll
    for (int i = 0; i < U; ++i)
      u[i] = c0 + i * 256 < K ? *reinterpret_cast<const uint4*>(xr + c0 + i * 256) : make_uint4(0, 0, 0, 0);
#pragma unroll
    for (int i = 0; i < U; ++i) {
      const uint32_t w4[4] = {u[i].x, u[i].y, u[i].z, u[i].w};
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const float2 f = unpack_bf16(w4[k]);
        amax = fmaxf(amax, fmaxf(fabsf(f.x), fabsf(f.y)));
      }
    }
  }
  amax = warp_max(amax);
  const float sc = amax > 0.f ? amax * (1.f / 448.f) : 1.f;
  const float inv = 1.f / sc;
  for (int c0 = lane * 8; c0 < K; c0 += 256 * U) {
    uint4 u[U];
#pragma unroll
    for (int i = 0; i < U; ++i)
      u[i] = c0 + i * 256 < K ? *reinterpret_cast<const uint4*>(xr + c0 + i * 256) : make_uint4(0, 0, 0, 0);
#pragma unroll
    for (int i = 0; i < U; ++i) {
      const int c = c0 + i * 256;
      if (c < K) {
        const float2 a = unpack_bf16(u[i].x), b = unpack_bf16(u[i].y), cc = unpack_bf16(u[i].z), d = unpack_bf16(u[i].w);
        *reinterpret_cast<uint2*>(q + (size_t)row * ldq + c) =
            make_uint2(pack4_e4m3(a.x, a.y, b.x, b.y, inv), pack4_e4m3(cc.x, cc.y, d.x, d.y, inv));
      }
    }
  }
  if (lane == 0) scale[row] = sc;
}
int quant_rows(const __nv_bfloat16* x, int ldx, int M, int K, uint8_t* q, int ldq, float* scale, cudaStream_t s) {
  if (K % 8 || ldx % 8 || ldq % 16) return FW_ESHAPE;
  launch_k(quant_rows_kernel, (M + 7) / 8, 256, 0, s, x, ldx, M, K, q, ldq, scale);
  return cudaGetLastError() == cudaSuccess ? 0 : FW_ECUDA;
}

// ------------------------------------------------------------------ RMSNorm (+ RoPE)
// out = RMSNorm(x) * w over D = 128 * NG, then (optionally) each (even, odd) pair of every
// head is rotated by rope[row, pair % (hd / 2)] = (cos, sin).  With tensor parallelism the
// row is a shard of the normalised width: `ss` then holds the all-reduced sum of squares of
// the full row (ss[row * 2 + tensor]) and inv_d is 1 / full width.
struct RmsPair {
  const __nv_bfloat16* x[2];
  const __nv_bfloat16* w[2];
  __nv_bfloat16* out[2];
  const float* ss = nullptr;
  float inv_d = 0.f;
  // grouped (w_grp set): blockIdx.y = group g normalises x[0] + g * grp_stride into
  // out[0] + g * grp_stride with weight w_grp[g]
  const __nv_bfloat16* const* w_grp = nullptr;
  long long grp_stride = 0;
};

template <int NG>
__global__ void __launch_bounds__(256) rms_rope_kernel(RmsPair pr, int ldx, int M, float eps,
                                                       const float2* __restrict__ rope, int hd, int ldo) {
  pdl_trigger();
  pdl_wait();
  const int row = blockIdx.x * 8 + (threadIdx.x >> 5), lane = threadIdx.x & 31;
  if (row >= M) return;
  // constant indices into the parameter struct (indexing it by blockIdx.y would copy it to
  // local memory in every thread)
  const bool y1 = blockIdx.y == 1;
  const size_t goff = pr.w_grp ? (size_t)blockIdx.y * (size_t)pr.grp_stride : 0;
  const __nv_bfloat16* __restrict__ x = pr.w_grp ? pr.x[0] + goff : (y1 ? pr.x[1] : pr.x[0]);
  const __nv_bfloat16* __restrict__ w = pr.w_grp ? pr.w_grp[blockIdx.y] : (y1 ? pr.w[1] : pr.w[0]);
  __nv_bfloat16* __restrict__ out = pr.w_grp ? pr.out[0] + goff : (y1 ? pr.out[1] : pr.out[0]);
  constexpr int D = 128 * NG;
  float v[NG][4];
  float q = 0.f;
#pragma unroll
  for (int g = 0; g < NG; ++g) {
    load4(x + (size_t)row * ldx + g * 128 + lane * 4, v[g]);
#pragma unroll
    for (int i = 0; i < 4; ++i) q += v[g][i] * v[g][i];
  }
  const float tot = pr.ss ? __ldg(pr.ss + (size_t)row * 2 + blockIdx.y) : warp_sum(q);
  const float r = rsqrtf(tot * (pr.ss ? pr.inv_d : 1.f / D) + eps);
  const int half = hd >> 1;
#pragma unroll
  for (int g = 0; g < NG; ++g) {
    const int c = g * 128 + lane * 4;
    float wv[4], y[4];
    load4(w + c, wv);
#pragma unroll
    for (int i = 0; i < 4; ++i) y[i] = v[g][i] * r * wv[i];
    if (rope) {
#pragma unroll
      for (int p = 0; p < 2; ++p) {
        const int pair = ((c % hd) >> 1) + p;
        const float2 cs = __ldg(rope + (size_t)row * half + pair);
        const float a = y[2 * p], bb = y[2 * p + 1];
        y[2 * p] = a * cs.x - bb * cs.y;
        y[2 * p + 1] = a * cs.y + bb * cs.x;
      }
    }
    store4(out + (size_t)row * ldo + c, y);
  }
}

// The same with eight consecutive elements per lane (D = 256 * NG8): one 16-byte load and store
// per group; the lane's four RoPE pairs are consecutive table entries (two 16-byte loads).
template <int NG8>
// At most 85 registers (three blocks per SM): with the RoPE pairs held from the start, a tighter
// cap spilled and measured no faster than this one.
__global__ void __launch_bounds__(256, 3) rms_rope8_kernel(RmsPair pr, int ldx, int M, float eps,
                                                        const float2* __restrict__ rope, int hd, int ldo) {
  pdl_trigger();
  pdl_wait();
  const int row = blockIdx.x * 8 + (threadIdx.x >> 5), lane = threadIdx.x & 31;
  if (row >= M) return;
  // constant indices into the parameter struct (indexing it by blockIdx.y would copy it to
  // local memory in every thread)
  const bool y1 = blockIdx.y == 1;
  const size_t goff = pr.w_grp ? (size_t)blockIdx.y * (size_t)pr.grp_stride : 0;
  const __nv_bfloat16* __restrict__ x = pr.w_grp ? pr.x[0] + goff : (y1 ? pr.x[1] : pr.x[0]);
  const __nv_bfloat16* __restrict__ w = pr.w_grp ? pr.w_grp[blockIdx.y] : (y1 ? pr.w[1] : pr.w[0]);
  __nv_bfloat16* __restrict__ out = pr.w_grp ? pr.out[0] + goff : (y1 ? pr.out[1] : pr.out[0]);
  constexpr int D = 256 * NG8;
  const int half = hd >> 1;
  // When the head dim divides 256 (64, 128), a lane's four RoPE pairs are the same in every
  // 256-column group: they are loaded once, together with the row, instead of once per group
  // after the row's statistics.
  const bool rope_once = rope && 256 % hd == 0;
  float4 cs01 = make_float4(0.f, 0.f, 0.f, 0.f), cs23 = cs01;
  if (rope_once) {
    const float4* rp = reinterpret_cast<const float4*>(rope + (size_t)row * half + (((lane * 8) % hd) >> 1));
    cs01 = __ldg(rp);
    cs23 = __ldg(rp + 1);
  }
  float v[NG8][8];
  float q = 0.f;
#pragma unroll
  for (int g = 0; g < NG8; ++g) {
    load8(x + (size_t)row * ldx + g * 256 + lane * 8, v[g]);
#pragma unroll
    for (int i = 0; i < 8; ++i) q += v[g][i] * v[g][i];
  }
  const float tot = pr.ss ? __ldg(pr.ss + (size_t)row * 2 + blockIdx.y) : warp_sum(q);
  const float r = rsqrtf(tot * (pr.ss ? pr.inv_d : 1.f / D) + eps);
#pragma unroll
  for (int g = 0; g < NG8; ++g) {
    const int c = g * 256 + lane * 8;
    float wv[8], y[8];
    load8(w + c, wv);
#pragma unroll
    for (int i = 0; i < 8; ++i) y[i] = v[g][i] * r * wv[i];
    if (rope) {
      if (!rope_once) {
        const float4* rp = reinterpret_cast<const float4*>(rope + (size_t)row * half + ((c % hd) >> 1));
        cs01 = __ldg(rp);
        cs23 = __ldg(rp + 1);
      }
      const float cs[8] = {cs01.x, cs01.y, cs01.z, cs01.w, cs23.x, cs23.y, cs23.z, cs23.w};
#pragma unroll
      for (int p = 0; p < 4; ++p) {
        const float a = y[2 * p], bb = y[2 * p + 1], co = cs[2 * p], si = cs[2 * p + 1];
        y[2 * p] = a * co - bb * si;
        y[2 * p + 1] = a * si + bb * co;
      }
    }
    *reinterpret_cast<uint4*>(out + (size_t)row * ldo + c) =
        make_uint4(pack_bf16(y[0], y[1]), pack_bf16(y[2], y[3]), pack_bf16(y[4], y[5]), pack_bf16(y[6], y[7]));
  }
}

static int rms_rope_launch(const RmsPair& pr, int ny, int ldx, int M, int D, float eps, const float2* rope, int hd,
                           int ldo, cudaStream_t s) {
  if (D % 128 || ldx % 4 || ldo % 4 || (rope && (hd % 4 || D % hd))) return FW_ESHAPE;
  const dim3 grid((M + 7) / 8, ny), block(256);
  if (D % 256 == 0 && ldx % 8 == 0 && ldo % 8 == 0 && (!rope || hd % 8 == 0)) {
    switch (D / 256) {
#define FW_RMS8_CASE(n) \
  case n: launch_k(rms_rope8_kernel<n>, grid, block, 0, s, pr, ldx, M, eps, rope, hd, ldo); \
    return cudaGetLastError() == cudaSuccess ? 0 : FW_ECUDA;
      FW_RMS8_CASE(1) FW_RMS8_CASE(2) FW_RMS8_CASE(3) FW_RMS8_CASE(4) FW_RMS8_CASE(5) FW_RMS8_CASE(6)
      FW_RMS8_CASE(8) FW_RMS8_CASE(10) FW_RMS8_CASE(20)
#undef FW_RMS8_CASE
      default: break;
    }
  }
  switch (D / 128) {
#define FW_RMS_CASE(n) \
  case n: launch_k(rms_rope_kernel<n>, grid, block, 0, s, pr, ldx, M, eps, rope, hd, ldo); break;
    FW_RMS_CASE(1) FW_RMS_CASE(2) FW_RMS_CASE(3) FW_RMS_CASE(4) FW_RMS_CASE(5) FW_RMS_CASE(6) FW_RMS_CASE(8)
    FW_RMS_CASE(10) FW_RMS_CASE(12) FW_RMS_CASE(16) FW_RMS_CASE(20) FW_RMS_CASE(40)
#undef FW_RMS_CASE
    default: return FW_ESHAPE;
  }
  return cudaGetLastError() == cudaSuccess ? 0 : FW_ECUDA;
}

int rms_rope2(const __nv_bfloat16* x, const __nv_bfloat16* w, __nv_bfloat16* out, const __nv_bfloat16* x2,
              const __nv_bfloat16* w2, __nv_bfloat16* out2, int ldx, int M, int D, float eps, const float2* rope, int hd,
              int ldo, cudaStream_t s) {
  RmsPair pr{{x, x2}, {w, w2}, {out, out2}};
  return rms_rope_launch(pr, x2 ? 2 : 1, ldx, M, D, eps, rope, hd, ldo, s);
}

int rms_grp(__nv_bfloat16* x, long long grp_stride, int groups, const __nv_bfloat16* const* w_grp, int ldx, int M,
            int D, float eps, cudaStream_t s) {
  if (!x || !w_grp || groups < 1 || groups > 65535 || grp_stride < 0) return FW_EINVAL;
  RmsPair pr{{x, nullptr}, {nullptr, nullptr}, {x, nullptr}};
  pr.w_grp = w_grp;
  pr.grp_stride = grp_stride;
  return rms_rope_launch(pr, groups, ldx, M, D, eps, nullptr, 128, ldx, s);
}

int rms_rope2_ss(const __nv_bfloat16* x, const __nv_bfloat16* w, __nv_bfloat16* out, const __nv_bfloat16* x2,
                 const __nv_bfloat16* w2, __nv_bfloat16* out2, int ldx, int M, int D, const float* ss, int d_full,
                 float eps, const float2* rope, int hd, int ldo, cudaStream_t s) {
  if (!ss || d_full <= 0) return FW_EINVAL;
  RmsPair pr{{x, x2}, {w, w2}, {out, out2}, ss, 1.f / (float)d_full};
  return rms_rope_launch(pr, x2 ? 2 : 1, ldx, M, D, eps, rope, hd, ldo, s);
}

// Per-row partial sums of squares of one or two bf16 tensors [M, D]: ss[row * 2 + t].  One
// warp per row.
__global__ void __launch_bounds__(256) sumsq_kernel(const __nv_bfloat16* __restrict__ x0,
                                                    const __nv_bfloat16* __restrict__ x1, int ld, int M, int D,
                                                    float* __restrict__ ss) {
  pdl_trigger();
  pdl_wait();
  const int row = blockIdx.x * 8 + (threadIdx.x >> 5), lane = threadIdx.x & 31;
  if (row >= M) return;
  const __nv_bfloat16* __restrict__ x = blockIdx.y ? x1 : x0;
  float q = 0.f;
  for (int c = lane * 8; c < D; c += 256) {
    const uint4 u = *reinterpret_cast<const uint4*>(x + (size_t)row * ld + c);
    const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float2 f = unpack_bf16(w[i]);
      q += f.x * f.x + f.y * f.y;
    }
  }
  q = warp_sum(q);
  if (lane == 0) ss[(size_t)row * 2 + blockIdx.y] = q;
}
int sumsq_rows(const __nv_bfloat16* x0, const __nv_bfloat16* x1, int ld, int M, int D, float* ss, cudaStream_t s) {
  if (D % 8 || ld % 8) return FW_ESHAPE;
  launch_k(sumsq_kernel, dim3((M + 7) / 8, x1 ? 2 : 1), 256, 0, s, x0, x1, ld, M, D, ss);
  return cudaGetLastError() == cudaSuccess ? 0 : FW_ECUDA;
}

// xs[row, :] += gate[(row / rows_per_frame) * gate_stride + :] * (p[row, :] + bias) after the
// all-reduce of a row-parallel linear (gate and bias optional; gate_stride 0 = one gate row for
// all frames); mirror (optional) = bf16 copy of the new xs.  One warp per row, 8 columns per
// lane per step.
__global__ void __launch_bounds__(256) resid_add_kernel(float* __restrict__ xs, int ldx,
                                                        const __nv_bfloat16* __restrict__ p, int ldp,
                                                        const __nv_bfloat16* __restrict__ bias,
                                                        const float* __restrict__ gate, int gate_stride,
                                                        int rows_per_frame, __nv_bfloat16* __restrict__ mirror,
                                                        int M, int D) {
  pdl_trigger();
  pdl_wait();
  const int row = blockIdx.x * 8 + (threadIdx.x >> 5), lane = threadIdx.x & 31;
  if (row >= M) return;
  const float* g = gate ? gate + (size_t)(row / rows_per_frame) * gate_stride : nullptr;
  for (int c = lane * 8; c < D; c += 256) {
    const uint4 u = *reinterpret_cast<const uint4*>(p + (size_t)row * ldp + c);
    const uint32_t pw[4] = {u.x, u.y, u.z, u.w};
    float v[8];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float2 f = unpack_bf16(pw[i]);
      v[2 * i] = f.x;
      v[2 * i + 1] = f.y;
    }
    if (bias) {
      const uint4 b = *reinterpret_cast<const uint4*>(bias + c);
      const uint32_t bw[4] = {b.x, b.y, b.z, b.w};
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float2 f = unpack_bf16(bw[i]);
        v[2 * i] += f.x;
        v[2 * i + 1] += f.y;
      }
    }
    float4* xr = reinterpret_cast<float4*>(xs + (size_t)row * ldx + c);
    float4 a = xr[0], b = xr[1];
    if (g) {
      const float4 g0 = *reinterpret_cast<const float4*>(g + c), g1 = *reinterpret_cast<const float4*>(g + c + 4);
      a.x += g0.x * v[0]; a.y += g0.y * v[1]; a.z += g0.z * v[2]; a.w += g0.w * v[3];
      b.x += g1.x * v[4]; b.y += g1.y * v[5]; b.z += g1.z * v[6]; b.w += g1.w * v[7];
    } else {
      a.x += v[0]; a.y += v[1]; a.z += v[2]; a.w += v[3];
      b.x += v[4]; b.y += v[5]; b.z += v[6]; b.w += v[7];
    }
    xr[0] = a;
    xr[1] = b;
    if (mirror)
      *reinterpret_cast<uint4*>(mirror + (size_t)row * D + c) =
          make_uint4(pack_bf16(a.x, a.y), pack_bf16(a.z, a.w), pack_bf16(b.x, b.y), pack_bf16(b.z, b.w));
  }
}
int resid_add(float* xs, int ldx, const __nv_bfloat16* p, int ldp, const __nv_bfloat16* bias, const float* gate,
              int gate_stride, int rows_per_frame, __nv_bfloat16* mirror, int M, int D, cudaStream_t s) {
  if (D % 8 || ldx % 4 || ldp % 8 || gate_stride % 4 || rows_per_frame <= 0) return FW_ESHAPE;
  launch_k(resid_add_kernel, (M + 7) / 8, 256, 0, s, xs, ldx, p, ldp, bias, gate, gate_stride, rows_per_frame, mirror,
           M, D);
  return cudaGetLastError() == cudaSuccess ? 0 : FW_ECUDA;
}

// ------------------------------------------------------------------ multi-chunk history window
// meta = {min(k, window) * L, L} for steady chunk k = chunk[0] (keys: filled history slots,
// then the current chunk).
__global__ void hist_meta_kernel(const int* __restrict__ chunk, int window, int L, int* __restrict__ meta) {
  pdl_trigger();
  pdl_wait();
  if (threadIdx.x == 0) {
    const int k = max(chunk[0], 0);
    meta[0] = min(k, window) * L;
    meta[1] = L;
  }
}
int hist_meta(const int* chunk, int window, int L, int* meta, cudaStream_t s) {
  if (!chunk || !meta || window < 1) return FW_EINVAL;
  launch_k(hist_meta_kernel, 1, 32, 0, s, chunk, window, L, meta);
  return cudaGetLastError() == cudaSuccess ? 0 : FW_ECUDA;
}

// dst_base + (chunk[0] % window) * slot_bytes <- src (n16 16-byte words): the context forward
// of chunk k writes its K or V into slot k % window of the history ring.
__global__ void __launch_bounds__(256) slot_copy_kernel(uint8_t* __restrict__ dst_base, size_t slot_bytes,
                                                        const int* __restrict__ chunk, int window,
                                                        const uint4* __restrict__ src, size_t n16) {
  pdl_trigger();
  pdl_wait();
  const int slot = max(chunk[0], 0) % window;
  uint4* __restrict__ dst = reinterpret_cast<uint4*>(dst_base + (size_t)slot * slot_bytes);
  const size_t stride = (size_t)gridDim.x * blockDim.x;
  for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n16; i += stride) __stcs(dst + i, __ldcs(src + i));
}
int slot_copy(void* dst_base, size_t slot_bytes, const int* chunk, int window, const void* src, size_t bytes,
              cudaStream_t s) {
  if (!dst_base || !src || !chunk || window < 1) return FW_EINVAL;
  if (((reinterpret_cast<uintptr_t>(dst_base) | reinterpret_cast<uintptr_t>(src)) & 15u) || bytes % 16 ||
      slot_bytes % 16 || bytes > slot_bytes)
    return FW_EALIGN;
  const size_t n16 = bytes / 16;
  size_t want = (n16 + 255) / 256;
  const size_t cap = (size_t)num_sms() * 8;
  const int grid = (int)(want < 1 ? 1 : (want > cap ? cap : want));
  launch_k(slot_copy_kernel, grid, 256, 0, s, reinterpret_cast<uint8_t*>(dst_base), slot_bytes, chunk, window,
           reinterpret_cast<const uint4*>(src), n16);
  return cudaGetLastError() == cudaSuccess ? 0 : FW_ECUDA;
}

int rms_rope(const __nv_bfloat16* x, int ldx, int M, int D, float eps, const __nv_bfloat16* w, const float2* rope,
             int hd, __nv_bfloat16* out, int ldo, cudaStream_t s) {
  return rms_rope2(x, w, out, nullptr, nullptr, nullptr, ldx, M, D, eps, rope, hd, ldo, s);
}

// ------------------------------------------------------------------ RoPE tables
// table[token, i] = (cos, sin)(pos * theta^(-2 j / dim_part)) with (pos, j, dim_part) the
// t / h / w position, the index within its part and the part's real width; angles in fp64
// as in Wan's rope_params.  act_cos/act_sin[f, d] for the action module (pair d / 2).
__global__ void rope_table_kernel(const int* __restrict__ chunk, int F, int th, int tw, int hd, double theta,
                                  float2* __restrict__ table, int act_hd, float* __restrict__ act_cos,
                                  float* __restrict__ act_sin) {
  pdl_trigger();
  pdl_wait();
  const int half = hd / 2;
  const int nt = half - 2 * (half / 3), nh = half / 3;
  const int s0 = __ldg(chunk + 1);   // first absolute latent frame of the chunk
  const int L = F * th * tw;
  const int idx = blockIdx.x * blockDim.x + threadIdx.x;
  if (idx < L * half) {
    const int tok = idx / half, i = idx % half;
    const int f = tok / (th * tw), h = (tok / tw) % th, w = tok % tw;
    int pos, j, part;
    if (i < nt) { pos = s0 + f; j = i; part = 2 * nt; }
    else if (i < nt + nh) { pos = h; j = i - nt; part = 2 * nh; }
    else { pos = w; j = i - nt - nh; part = 2 * nh; }
    const double ang = (double)pos * (1.0 / pow(theta, (double)(2 * j) / (double)part));
    double sn, cs;
    sincos(ang, &sn, &cs);
    table[idx] = make_float2((float)cs, (float)sn);
  }
  if (act_cos && idx < F * act_hd) {
    const int f = idx / act_hd, d = idx % act_hd, j = d >> 1;
    const double ang = (double)(s0 + f) * (1.0 / pow(theta, (double)(2 * j) / (double)act_hd));
    double sn, cs;
    sincos(ang, &sn, &cs);
    act_cos[idx] = (float)cs;
    act_sin[idx] = (float)sn;
  }
}

int rope_tables(const int* chunk, int F, int th, int tw, int hd, double theta, float2* table, int act_hd,
                float* act_cos, float* act_sin, cudaStream_t s) {
  const int n = F * th * tw * (hd / 2);
  const int m = n > F * act_hd ? n : F * act_hd;
  launch_k(rope_table_kernel, (m + 255) / 256, 256, 0, s, chunk, F, th, tw, hd, theta, table, act_hd, act_cos, act_sin);
  return cudaGetLastError() == cudaSuccess ? 0 : FW_ECUDA;
}

__device__ __forceinline__ void unpack8(const uint4& u, float (&v)[8]) {
  const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 f = unpack_bf16(w[i]);
    v[2 * i] = f.x;
    v[2 * i + 1] = f.y;
  }
}

// ------------------------------------------------------------------ small-M linear
// out[m, n] = act_out(sum_k act_in(x[m, k]) W[n, k] + b[n]), one warp per output column n.
// Rows are processed four at a time: each weight element is loaded once per four rows and the
// four dot products are independent, so their loads and reductions overlap (M is small here:
// 1 for the time embedding, 3 frames or 21 keyboard rows for the action module).
__device__ __forceinline__ float act_apply(float v, int act) {
  if (act == ACT_SILU) return v / (1.f + __expf(-v));
  if (act == ACT_GELU_ERF) return 0.5f * v * (1.f + erff(v * 0.7071067811865476f));
  return v;
}
__device__ __forceinline__ void smallm_store(float acc, float bn, int act_out, int m, int n, int lane,
                                             float* __restrict__ outf, __nv_bfloat16* __restrict__ outb, int ldo) {
  acc = act_apply(warp_sum(acc) + bn, act_out);
  if (lane == 0) {
    if (outf) outf[(size_t)m * ldo + n] = acc;
    if (outb) outb[(size_t)m * ldo + n] = __float2bfloat16(acc);
  }
}

template <typename Tx>
__global__ void __launch_bounds__(256) smallm_linear_kernel(const Tx* __restrict__ x, int ldx, int M,
                                                            const __nv_bfloat16* __restrict__ W, int ldw,
                                                            const __nv_bfloat16* __restrict__ bias, int N, int K,
                                                            int act_in, int act_out, float* __restrict__ outf,
                                                            __nv_bfloat16* __restrict__ outb, int ldo, SmallmGrp g) {
  pdl_trigger();
  pdl_wait();
  const int n = blockIdx.x * 8 + (threadIdx.x >> 5), lane = threadIdx.x & 31;
  if (n >= N) return;
  if (g.w) {   // grouped launch
    W = g.w[blockIdx.y];
    bias = g.bias ? g.bias[blockIdx.y] : nullptr;
    x += (size_t)blockIdx.y * (size_t)g.x_stride;
    if (outf) outf += (size_t)blockIdx.y * (size_t)g.out_stride;
    if (outb) outb += (size_t)blockIdx.y * (size_t)g.out_stride;
  }
  const __nv_bfloat16* wr = W + (size_t)n * ldw;
  const float bn = bias ? __bfloat162float(bias[n]) : 0.f;
  for (int m0 = 0; m0 < M; m0 += 4) {
    float acc[4] = {0.f, 0.f, 0.f, 0.f};
    for (int k = lane; k < K; k += 32) {
      const float wv = __bfloat162float(wr[k]);
#pragma unroll
      for (int r = 0; r < 4; ++r)
        if (m0 + r < M) acc[r] += act_apply((float)x[(size_t)(m0 + r) * ldx + k], act_in) * wv;
    }
#pragma unroll
    for (int r = 0; r < 4; ++r)
      if (m0 + r < M) smallm_store(acc[r], bn, act_out, m0 + r, n, lane, outf, outb, ldo);
  }
}

// The same with 16-byte loads: each lane takes 8 consecutive k (one uint4 of weights, 8 inputs
// per row) per step, so a warp reads 512 contiguous weight bytes per instruction; a lane keeps
// four such weight loads in flight.  K % 8 == 0 and 16-byte aligned rows of W and x.
template <typename Tx, int RB>   // RB rows per pass: 1 (M = 1, high occupancy) or 4
__global__ void __launch_bounds__(256, RB == 1 ? 4 : 2) smallm_linear8_kernel(const Tx* __restrict__ x, int ldx, int M,
                                                             const __nv_bfloat16* __restrict__ W, int ldw,
                                                             const __nv_bfloat16* __restrict__ bias, int N, int K,
                                                             int act_in, int act_out, float* __restrict__ outf,
                                                             __nv_bfloat16* __restrict__ outb, int ldo, SmallmGrp g) {
  pdl_trigger();
  pdl_wait();
  const int n = blockIdx.x * 8 + (threadIdx.x >> 5), lane = threadIdx.x & 31;
  if (n >= N) return;
  if (g.w) {   // grouped launch
    W = g.w[blockIdx.y];
    bias = g.bias ? g.bias[blockIdx.y] : nullptr;
    x += (size_t)blockIdx.y * (size_t)g.x_stride;
    if (outf) outf += (size_t)blockIdx.y * (size_t)g.out_stride;
    if (outb) outb += (size_t)blockIdx.y * (size_t)g.out_stride;
  }
  const uint4* wr = reinterpret_cast<const uint4*>(W + (size_t)n * ldw);
  const float bn = bias ? __bfloat162float(bias[n]) : 0.f;
  const int K8 = K >> 3;
  for (int m0 = 0; m0 < M; m0 += RB) {
    float acc[RB];
#pragma unroll
    for (int r = 0; r < RB; ++r) acc[r] = 0.f;
    for (int kb = lane; kb < K8; kb += 128) {   // four weight vectors in flight per lane
      uint4 wq[4];
#pragma unroll
      for (int u = 0; u < 4; ++u) wq[u] = kb + 32 * u < K8 ? __ldg(wr + kb + 32 * u) : make_uint4(0, 0, 0, 0);
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const int k8 = kb + 32 * u;
        float wv[8];
        unpack8(wq[u], wv);
#pragma unroll
        for (int r = 0; r < RB; ++r) {
          if (k8 < K8 && m0 + r < M) {
            float xv[8];
            load8(x + (size_t)(m0 + r) * ldx + k8 * 8, xv);
#pragma unroll
            for (int i = 0; i < 8; ++i) acc[r] += act_apply(xv[i], act_in) * wv[i];
          }
        }
      }
    }
#pragma unroll
    for (int r = 0; r < RB; ++r)
      if (m0 + r < M) smallm_store(acc[r], bn, act_out, m0 + r, n, lane, outf, outb, ldo);
  }
}

template <typename Tx>
static int smallm_dispatch(const Tx* x, int ldx, int M, const __nv_bfloat16* W, int ldw, const __nv_bfloat16* b,
                           int N, int K, int act_in, int act_out, float* outf, __nv_bfloat16* outb, int ldo,
                           cudaStream_t s, const SmallmGrp* grp) {
  auto al16 = [](const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; };
  const SmallmGrp g = grp ? *grp : SmallmGrp{};
  if (g.w && (g.groups < 1 || g.groups > 65535 || g.x_stride < 0 || g.out_stride < 0)) return FW_EINVAL;
  const bool vec = K % 8 == 0 && ldw % 8 == 0 && ldx % 8 == 0 && al16(x) && (g.w ? g.aligned : al16(W)) &&
                   (g.x_stride % 8 == 0);
  const dim3 grid((N + 7) / 8, g.w ? g.groups : 1);
  if (vec && M == 1)
    launch_k(smallm_linear8_kernel<Tx, 1>, grid, 256, 0, s, x, ldx, M, W, ldw, b, N, K, act_in, act_out, outf, outb,
             ldo, g);
  else if (vec)
    launch_k(smallm_linear8_kernel<Tx, 4>, grid, 256, 0, s, x, ldx, M, W, ldw, b, N, K, act_in, act_out, outf, outb,
             ldo, g);
  else
    launch_k(smallm_linear_kernel<Tx>, grid, 256, 0, s, x, ldx, M, W, ldw, b, N, K, act_in, act_out, outf, outb,
             ldo, g);
  return cudaGetLastError() == cudaSuccess ? 0 : FW_ECUDA;
}

int smallm_linear_f32(const float* x, int ldx, int M, const __nv_bfloat16* W, int ldw, const __nv_bfloat16* b, int N,
                      int K, int act_in, int act_out, float* outf, __nv_bfloat16* outb, int ldo, cudaStream_t s,
                      const SmallmGrp* grp) {
  return smallm_dispatch<float>(x, ldx, M, W, ldw, b, N, K, act_in, act_out, outf, outb, ldo, s, grp);
}
int smallm_linear_bf16(const __nv_bfloat16* x, int ldx, int M, const __nv_bfloat16* W, int ldw,
                       const __nv_bfloat16* b, int N, int K, int act_in, int act_out, float* outf,
                       __nv_bfloat16* outb, int ldo, cudaStream_t s, const SmallmGrp* grp) {
  return smallm_dispatch<__nv_bfloat16>(x, ldx, M, W, ldw, b, N, K, act_in, act_out, outf, outb, ldo, s, grp);
}

// ------------------------------------------------------------------ time embedding helpers
// Wan sinusoidal_embedding_1d of one timestep: [cos(t w_i), sin(t w_i)], w_i = 10000^(-i/half).
__global__ void sinusoid_kernel(double t, int dim, float* out) {
  pdl_trigger();
  pdl_wait();
  const int half = dim / 2, i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i < half) {
    const double a = t * pow(10000.0, -(double)i / (double)half);
    double sn, cs;
    sincos(a, &sn, &cs);
    out[i] = (float)cs;
    out[i + half] = (float)sn;
  }
}
int sinusoid(double t, int dim, float* out, cudaStream_t s) {
  launch_k(sinusoid_kernel, (dim / 2 + 127) / 128, 128, 0, s, t, dim, out);
  return cudaGetLastError() == cudaSuccess ? 0 : FW_ECUDA;
}

// ee[l, j, :] = mods[l, j, :] + e0[j, :] (block adaLN tables, static.py:204);
// head[j, :] = hmod[j, :] + e (head modulation).
__global__ void modulation_kernel(const __nv_bfloat16* __restrict__ mods, const float* __restrict__ e0, int layers,
                                  int D, float* __restrict__ ee, const __nv_bfloat16* __restrict__ hmod,
                                  const float* __restrict__ e, float* __restrict__ head) {
  pdl_trigger();
  pdl_wait();
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  const int n = layers * 6 * D;
  if (i < n) ee[i] = __bfloat162float(mods[i]) + e0[i % (6 * D)];
  if (i < 2 * D) head[i] = __bfloat162float(hmod[i]) + e[i % D];
}
int modulation(const __nv_bfloat16* mods, const float* e0, int layers, int D, float* ee, const __nv_bfloat16* hmod,
               const float* e, float* head, cudaStream_t s) {
  const int n = layers * 6 * D > 2 * D ? layers * 6 * D : 2 * D;
  launch_k(modulation_kernel, (n + 255) / 256, 256, 0, s, mods, e0, layers, D, ee, hmod, e, head);
  return cudaGetLastError() == cudaSuccess ? 0 : FW_ECUDA;
}

// ------------------------------------------------------------------ patchify
// A[token, c * 4 + i * 2 + j] = cat(x, cc)[c, f, 2 h + i, 2 w + j]  (Conv3d weight order).
__global__ void patchify_kernel(const __nv_bfloat16* __restrict__ x, int C1, const __nv_bfloat16* __restrict__ cc,
                                int C2, int F, int H, int W, __nv_bfloat16* __restrict__ A) {
  pdl_trigger();
  pdl_wait();
  const int th = H / 2, tw = W / 2, C = C1 + C2, Kp = C * 4;
  const int L = F * th * tw;
  const int idx = blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= L * Kp) return;
  const int tok = idx / Kp, k = idx % Kp;
  const int c = k >> 2, i = (k >> 1) & 1, j = k & 1;
  const int f = tok / (th * tw), h = (tok / tw) % th, w = tok % tw;
  const size_t off = (((size_t)f * H) + 2 * h + i) * W + 2 * w + j;
  A[idx] = c < C1 ? x[(size_t)c * F * H * W + off] : cc[(size_t)(c - C1) * F * H * W + off];
}
int patchify(const __nv_bfloat16* x, int C1, const __nv_bfloat16* cc, int C2, int F, int H, int W, __nv_bfloat16* A,
             cudaStream_t s) {
  const int n = F * (H / 2) * (W / 2) * (C1 + C2) * 4;
  launch_k(patchify_kernel, (n + 255) / 256, 256, 0, s, x, C1, cc, C2, F, H, W, A);
  return cudaGetLastError() == cudaSuccess ? 0 : FW_ECUDA;
}

// ------------------------------------------------------------------ unpatchify + scheduler
// flow[c, f, h, w] = head[token(f, h/2, w/2), ((h%2) * 2 + (w%2)) * C + c];
// den = bf16(x - sigma * flow); out = den (optional);
// xnext = bf16((1 - sigma_n) * den + sigma_n * noise[f, c, h, w]) (optional).
__global__ void scheduler_kernel(const float* __restrict__ head, const __nv_bfloat16* __restrict__ x, float sigma,
                                 __nv_bfloat16* __restrict__ den, __nv_bfloat16* __restrict__ out_copy,
                                 const __nv_bfloat16* __restrict__ noise, float sigma_n,
                                 __nv_bfloat16* __restrict__ xnext, int C, int F, int H, int W) {
  pdl_trigger();
  pdl_wait();
  const int idx = blockIdx.x * blockDim.x + threadIdx.x;
  const int n = C * F * H * W;
  if (idx >= n) return;
  const int w = idx % W, h = (idx / W) % H, f = (idx / (W * H)) % F, c = idx / (W * H * F);
  const int tw = W / 2, th = H / 2;
  const int tok = (f * th + h / 2) * tw + w / 2;
  const int feat = ((h & 1) * 2 + (w & 1)) * C + c;
  const float flow = head[(size_t)tok * (4 * C) + feat];
  const __nv_bfloat16 d = __float2bfloat16(__bfloat162float(x[idx]) - sigma * flow);
  if (den) den[idx] = d;
  if (out_copy) out_copy[idx] = d;
  if (noise) {
    const float nz = __bfloat162float(noise[(((size_t)f * C + c) * H + h) * W + w]);
    xnext[idx] = __float2bfloat16((1.f - sigma_n) * __bfloat162float(d) + sigma_n * nz);
  }
}
int scheduler(const float* head, const __nv_bfloat16* x, float sigma, __nv_bfloat16* den, __nv_bfloat16* out_copy,
              const __nv_bfloat16* noise, float sigma_n, __nv_bfloat16* xnext, int C, int F, int H, int W,
              cudaStream_t s) {
  const int n = C * F * H * W;
  launch_k(scheduler_kernel, (n + 255) / 256, 256, 0, s, head, x, sigma, den, out_copy, noise, sigma_n, xnext, C, F, H, W);
  return cudaGetLastError() == cudaSuccess ? 0 : FW_ECUDA;
}

// ------------------------------------------------------------------ action module
// Per-head RMSNorm (64 dims, one pair per lane) + interleaved-pair RoPE.
__device__ __forceinline__ float2 norm_rope64(float2 v, float wa, float wb, float c, float s, float eps) {
  const float r = rsqrtf(warp_sum(v.x * v.x + v.y * v.y) * (1.f / 64.f) + eps);
  const float a = v.x * r * wa, b = v.y * r * wb;
  return make_float2(a * c - b * s, b * c + a * s);
}
__device__ __forceinline__ float2 ld2(const __nv_bfloat16* p) {
  return unpack_bf16(*reinterpret_cast<const uint32_t*>(p));
}
__device__ __forceinline__ void st2(__nv_bfloat16* p, float2 v) {
  *reinterpret_cast<uint32_t*>(p) = pack_bf16(v.x, v.y);
}
__device__ __forceinline__ float2 bround(float2 v) { return unpack_bf16(pack_bf16(v.x, v.y)); }

// 8 lanes per (row, head), 8 consecutive head dims per lane (4 interleaved RoPE pairs); the
// lane group's reductions use 3 xor-shuffle steps.
__device__ __forceinline__ float group8_sum(float v) {
  v += __shfl_xor_sync(0xffffffffu, v, 4);
  v += __shfl_xor_sync(0xffffffffu, v, 2);
  v += __shfl_xor_sync(0xffffffffu, v, 1);
  return v;
}
__device__ __forceinline__ uint4 pack8(const float (&v)[8]) {
  return make_uint4(pack_bf16(v[0], v[1]), pack_bf16(v[2], v[3]), pack_bf16(v[4], v[5]), pack_bf16(v[6], v[7]));
}
// RMSNorm over the head's 64 dims (weights w[8] of this lane's dims) + interleaved-pair RoPE
// with cos / sin of pair (d + 2i) taken at cs / sn[2i]; the result rounded to bf16 (the
// reference keeps q and k in bf16).
__device__ __forceinline__ void norm_rope8(float (&v)[8], const float (&w)[8], const float* cs, const float* sn,
                                           float eps) {
  float q = 0.f;
#pragma unroll
  for (int i = 0; i < 8; ++i) q += v[i] * v[i];
  const float r = rsqrtf(group8_sum(q) * (1.f / 64.f) + eps);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float a = v[2 * i] * r * w[2 * i], b = v[2 * i + 1] * r * w[2 * i + 1];
    const float c = cs[2 * i], sv = sn[2 * i];
    v[2 * i] = a * c - b * sv;
    v[2 * i + 1] = b * c + a * sv;
  }
#pragma unroll
  for (int i = 0; i < 8; ++i) v[i] = __bfloat162float(__float2bfloat16_rn(v[i]));
}
__device__ __forceinline__ float dot8(const float (&a)[8], const float (&b)[8]) {
  float s = 0.f;
#pragma unroll
  for (int i = 0; i < 8; ++i) s += a[i] * b[i];
  return s;
}

// Mouse branch: 8 lanes per (spatial position s, head h), four per warp.  qkv [L, 3A] rows
// f * S + s; history mk/mv [S, F, AH, 64]; out [L, A].  Keys: [history (unless first) |
// current frames].
template <int F>
__global__ void __launch_bounds__(256) mouse_attn_kernel(const __nv_bfloat16* __restrict__ qkv,
                                                         const __nv_bfloat16* __restrict__ wq,
                                                         const __nv_bfloat16* __restrict__ wk,
                                                         const float* __restrict__ acos_,
                                                         const float* __restrict__ asin_, __nv_bfloat16* mk,
                                                         __nv_bfloat16* mv, int first, int write,
                                                         __nv_bfloat16* __restrict__ out, int S, int AH, float eps) {
  pdl_trigger();
  pdl_wait();
  const int lane = threadIdx.x & 31;
  const int slot = (blockIdx.x * 8 + (threadIdx.x >> 5)) * 4 + (lane >> 3);
  const bool live = slot < S * AH;   // dead groups still take part in the warp shuffles
  const int sl = live ? slot : 0;
  const int s = sl / AH, h = sl % AH, A = AH * 64, d = (lane & 7) * 8;
  float wqv[8], wkv[8];
  unpack8(*reinterpret_cast<const uint4*>(wq + d), wqv);
  unpack8(*reinterpret_cast<const uint4*>(wk + d), wkv);
  float q[F][8], kc[F][8];
  uint4 vc[F], kh[F], vh[F];
#pragma unroll
  for (int f = 0; f < F; ++f) {
    const __nv_bfloat16* r = qkv + (size_t)(f * S + s) * 3 * A + h * 64 + d;
    unpack8(*reinterpret_cast<const uint4*>(r), q[f]);
    unpack8(*reinterpret_cast<const uint4*>(r + A), kc[f]);
    vc[f] = *reinterpret_cast<const uint4*>(r + 2 * A);
    norm_rope8(q[f], wqv, acos_ + f * 64 + d, asin_ + f * 64 + d, eps);
    norm_rope8(kc[f], wkv, acos_ + f * 64 + d, asin_ + f * 64 + d, eps);
    const size_t ho = (((size_t)s * F + f) * AH + h) * 64 + d;
    kh[f] = first ? make_uint4(0, 0, 0, 0) : *reinterpret_cast<const uint4*>(mk + ho);
    vh[f] = first ? make_uint4(0, 0, 0, 0) : *reinterpret_cast<const uint4*>(mv + ho);
  }
  const float scale = 0.125f;   // 1 / sqrt(64)
#pragma unroll
  for (int f = 0; f < F; ++f) {
    float sc[2 * F];
    float mx = -INFINITY;
#pragma unroll
    for (int j = 0; j < F; ++j) {
      float khf[8];
      unpack8(kh[j], khf);
      const float a = group8_sum(dot8(q[f], khf)) * scale, b = group8_sum(dot8(q[f], kc[j])) * scale;
      sc[j] = first ? -INFINITY : a;
      sc[F + j] = b;
      mx = fmaxf(mx, fmaxf(sc[j], sc[F + j]));
    }
    float den = 0.f, o[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
#pragma unroll
    for (int j = 0; j < F; ++j) {
      const float ph = __expf(sc[j] - mx), pc = __expf(sc[F + j] - mx);
      float a[8], b[8];
      unpack8(vh[j], a);
      unpack8(vc[j], b);
      den += ph + pc;
#pragma unroll
      for (int i = 0; i < 8; ++i) o[i] += ph * a[i] + pc * b[i];
    }
    const float inv = 1.f / den;
#pragma unroll
    for (int i = 0; i < 8; ++i) o[i] *= inv;
    if (live) *reinterpret_cast<uint4*>(out + (size_t)(f * S + s) * A + h * 64 + d) = pack8(o);
  }
  if (write && live) {
#pragma unroll
    for (int f = 0; f < F; ++f) {
      const size_t ho = (((size_t)s * F + f) * AH + h) * 64 + d;
      *reinterpret_cast<uint4*>(mk + ho) = pack8(kc[f]);
      *reinterpret_cast<uint4*>(mv + ho) = vc[f];
    }
  }
}

int mouse_attn(const __nv_bfloat16* qkv, const __nv_bfloat16* wq, const __nv_bfloat16* wk, const float* acos_,
               const float* asin_, __nv_bfloat16* mk, __nv_bfloat16* mv, int first, int write, __nv_bfloat16* out,
               int S, int F, int AH, float eps, cudaStream_t s) {
  if (F != 3) return FW_ESHAPE;
  launch_k(mouse_attn_kernel<3>, (S * AH + 31) / 32, 256, 0, s, qkv, wq, wk, acos_, asin_, mk, mv, first, write, out, S,
           AH, eps);
  return cudaGetLastError() == cudaSuccess ? 0 : FW_ECUDA;
}

// Keyboard K/V of one block: kv [F, 2A] fp32 -> K = RoPE(RMSNorm(k) * wk) and V, bf16 [F, A].
// blockIdx.y = group (action layer) when wk_grp is set: kv, kout and vout advance by one layer.
__global__ void kb_kv_kernel(const float* __restrict__ kv, const __nv_bfloat16* __restrict__ wk,
                             const __nv_bfloat16* const* __restrict__ wk_grp, const float* __restrict__ acos_,
                             const float* __restrict__ asin_, __nv_bfloat16* __restrict__ kout,
                             __nv_bfloat16* __restrict__ vout, int F, int AH, float eps) {
  pdl_trigger();
  pdl_wait();
  const int wid = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5), lane = threadIdx.x & 31;
  if (wid >= F * AH) return;
  const int f = wid / AH, h = wid % AH, A = AH * 64, d = 2 * lane;
  if (wk_grp) {
    wk = wk_grp[blockIdx.y];
    kv += (size_t)blockIdx.y * F * 2 * A;
    kout += (size_t)blockIdx.y * F * A;
    vout += (size_t)blockIdx.y * F * A;
  }
  const float2 w = ld2(wk + d);
  const float* r = kv + (size_t)f * 2 * A + h * 64 + d;
  const float2 k = norm_rope64(make_float2(r[0], r[1]), w.x, w.y, acos_[f * 64 + d], asin_[f * 64 + d], eps);
  st2(kout + (size_t)f * A + h * 64 + d, k);
  st2(vout + (size_t)f * A + h * 64 + d, make_float2(r[A], r[A + 1]));
}
int kb_kv(const float* kv, const __nv_bfloat16* wk, const float* acos_, const float* asin_, __nv_bfloat16* kout,
          __nv_bfloat16* vout, int F, int AH, float eps, cudaStream_t s) {
  launch_k(kb_kv_kernel, (F * AH + 3) / 4, 128, 0, s, kv, wk, (const __nv_bfloat16* const*)nullptr, acos_, asin_,
           kout, vout, F, AH, eps);
  return cudaGetLastError() == cudaSuccess ? 0 : FW_ECUDA;
}
int kb_kv_grp(const float* kv, const __nv_bfloat16* const* wk_grp, int groups, const float* acos_,
              const float* asin_, __nv_bfloat16* kout, __nv_bfloat16* vout, int F, int AH, float eps, cudaStream_t s) {
  if (!wk_grp || groups < 1 || groups > 65535) return FW_EINVAL;
  launch_k(kb_kv_kernel, dim3((F * AH + 3) / 4, groups), 128, 0, s, kv, (const __nv_bfloat16*)nullptr, wk_grp,
           acos_, asin_, kout, vout, F, AH, eps);
  return cudaGetLastError() == cudaSuccess ? 0 : FW_ECUDA;
}

// Keyboard attention: 8 lanes per (token row, head), four per warp; q = RoPE(RMSNorm(mq));
// keys [kh (unless first) | kc] and values of the row's frame-independent keyboard tokens.
template <int F>
__global__ void __launch_bounds__(256) kb_attn_kernel(const __nv_bfloat16* __restrict__ mq,
                                                      const __nv_bfloat16* __restrict__ wq,
                                                      const float* __restrict__ acos_,
                                                      const float* __restrict__ asin_,
                                                      const __nv_bfloat16* __restrict__ kh,
                                                      const __nv_bfloat16* __restrict__ vh,
                                                      const __nv_bfloat16* __restrict__ kc,
                                                      const __nv_bfloat16* __restrict__ vc, int first,
                                                      __nv_bfloat16* __restrict__ out, int L, int S, int AH, float eps) {
  pdl_trigger();
  pdl_wait();
  const int lane = threadIdx.x & 31;
  const int slot = (blockIdx.x * 8 + (threadIdx.x >> 5)) * 4 + (lane >> 3);
  const bool live = slot < L * AH;
  const int sl = live ? slot : 0;
  const int row = sl / AH, h = sl % AH, f = row / S, A = AH * 64, d = (lane & 7) * 8;
  float w[8], q[8];
  unpack8(*reinterpret_cast<const uint4*>(wq + d), w);
  unpack8(*reinterpret_cast<const uint4*>(mq + (size_t)row * A + h * 64 + d), q);
  norm_rope8(q, w, acos_ + f * 64 + d, asin_ + f * 64 + d, eps);
  float sc[2 * F];
  float mx = -INFINITY;
#pragma unroll
  for (int j = 0; j < F; ++j) {
    float a[8], b[8];
    unpack8(*reinterpret_cast<const uint4*>(kh + (size_t)j * A + h * 64 + d), a);
    unpack8(*reinterpret_cast<const uint4*>(kc + (size_t)j * A + h * 64 + d), b);
    const float sa = group8_sum(dot8(q, a)) * 0.125f, sb = group8_sum(dot8(q, b)) * 0.125f;
    sc[j] = first ? -INFINITY : sa;
    sc[F + j] = sb;
    mx = fmaxf(mx, fmaxf(sc[j], sc[F + j]));
  }
  float den = 0.f, o[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
#pragma unroll
  for (int j = 0; j < F; ++j) {
    const float ph = __expf(sc[j] - mx), pc = __expf(sc[F + j] - mx);
    float a[8], b[8];
    unpack8(*reinterpret_cast<const uint4*>(vh + (size_t)j * A + h * 64 + d), a);
    unpack8(*reinterpret_cast<const uint4*>(vc + (size_t)j * A + h * 64 + d), b);
    den += ph + pc;
#pragma unroll
    for (int i = 0; i < 8; ++i) o[i] += ph * a[i] + pc * b[i];
  }
  const float inv = 1.f / den;
#pragma unroll
  for (int i = 0; i < 8; ++i) o[i] *= inv;
  if (live) *reinterpret_cast<uint4*>(out + (size_t)row * A + h * 64 + d) = pack8(o);
}

int kb_attn(const __nv_bfloat16* mq, const __nv_bfloat16* wq, const float* acos_, const float* asin_,
            const __nv_bfloat16* kh, const __nv_bfloat16* vh, const __nv_bfloat16* kc, const __nv_bfloat16* vc,
            int first, __nv_bfloat16* out, int L, int S, int F, int AH, float eps, cudaStream_t s) {
  if (F != 3) return FW_ESHAPE;
  launch_k(kb_attn_kernel<3>, (L * AH + 31) / 32, 256, 0, s, mq, wq, acos_, asin_, kh, vh, kc, vc, first, out, L, S,
           AH, eps);
  return cudaGetLastError() == cudaSuccess ? 0 : FW_ECUDA;
}

// ------------------------------------------------------------------ copies
// Vectorised copy: 16-byte body (both pointers 16-byte aligned), byte tail.
__global__ void __launch_bounds__(256) copy_kernel(uint4* __restrict__ dst, const uint4* __restrict__ src, size_t n16,
                                                   uint8_t* __restrict__ dtail, const uint8_t* __restrict__ stail,
                                                   int ntail) {
  pdl_trigger();
  pdl_wait();
  const size_t stride = (size_t)gridDim.x * blockDim.x;
  size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
  for (; i + 3 * stride < n16; i += 4 * stride) {
    const uint4 a = __ldcs(src + i), b = __ldcs(src + i + stride), c = __ldcs(src + i + 2 * stride),
                d = __ldcs(src + i + 3 * stride);
    __stcs(dst + i, a);
    __stcs(dst + i + stride, b);
    __stcs(dst + i + 2 * stride, c);
    __stcs(dst + i + 3 * stride, d);
  }
  for (; i < n16; i += stride) __stcs(dst + i, __ldcs(src + i));
  const int t = blockIdx.x * blockDim.x + threadIdx.x;
  if (t < ntail) dtail[t] = stail[t];
}
int copy_bytes(void* dst, const void* src, size_t bytes, cudaStream_t s) {
  if (!dst || !src) return FW_EINVAL;
  if ((reinterpret_cast<uintptr_t>(dst) | reinterpret_cast<uintptr_t>(src)) & 15u) return FW_EALIGN;
  if (bytes == 0) return 0;
  const size_t n16 = bytes / 16;
  const int ntail = (int)(bytes % 16);
  size_t want = (n16 + 255) / 256;
  const size_t cap = (size_t)num_sms() * 8;
  const int grid = (int)(want < 1 ? 1 : (want > cap ? cap : want));
  launch_k(copy_kernel, grid, 256, 0, s, reinterpret_cast<uint4*>(dst), reinterpret_cast<const uint4*>(src), n16,
                                   reinterpret_cast<uint8_t*>(dst) + n16 * 16,
                                   reinterpret_cast<const uint8_t*>(src) + n16 * 16, ntail);
  return cudaGetLastError() == cudaSuccess ? 0 : FW_ECUDA;
}

}  // namespace fw
