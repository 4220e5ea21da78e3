// Chunk preparation on the device (the reference's host-side StaticMG._prep,
// fastworld/models/mg2/static.py:76-127), one launch, no host-to-device copy:
//
//   * chunk info {k, frames * k, 0, 0} (read by the RoPE tables, the history ring and the
//     action module's RoPE rows);
//   * the action module's windows: keyboard kc [KC, 4] and grouped mouse gm [F, PAD, 2].
//     Window position i reads pixel frame q = ratio * F * k + i - PAD, which belongs to chunk 0
//     when q < 0 (the padding repeats the first action) and otherwise to the chunk that owns
//     pixel frame q (chunk 0 owns 1 + ratio * (F - 1) frames, later chunks ratio * F each);
//     frame f of the chunk reads the PAD mouse entries starting at ratio * f.  The host passes
//     the actions of chunks j_lo .. j_lo + n_act - 1 (the only ones the window reads) by value;
//   * the image condition slice cc = cond[:, F * k : F * (k + 1)];
//   * the initial latent x_in and the per-step renoising noise, N(0, 1) in bf16, from a
//     counter-based generator keyed by the path seed: Philox-4x32-10 (Salmon, Moraes, Dror and
//     Shaw, "Parallel random numbers: as easy as 1, 2, 3", SC 2011) with key = the 64-bit seed
//     and counter = {group, tensor, 0, 0}, where tensor 0 is x_in, tensor t the noise of step
//     t - 1 and group g covers elements 4g .. 4g + 3 of that tensor; its four words become four
//     normals by the Box-Muller transform (u = (word + 0.5) / 2^32).  Every element depends
//     only on (seed, tensor, element index), so the noise is the same in any launch shape.
//     This stream differs from torch's (the reference draws with torch.randn); the session
//     keeps the torch path for bit-compatibility with the reference.
#include "../../include/fastworld_b200.h"
#include "fw_elem.h"
#include "fw_internal.h"
#include "fw_ptx.cuh"

namespace fw {

namespace {

struct Philox4 {
  uint32_t v[4];
};

__host__ __device__ __forceinline__ void mulhilo(uint32_t a, uint32_t b, uint32_t& hi, uint32_t& lo) {
  const uint64_t p = (uint64_t)a * (uint64_t)b;
  hi = (uint32_t)(p >> 32);
  lo = (uint32_t)p;
}

// Philox-4x32 with 10 rounds (multipliers and Weyl key increments of the published algorithm).
__host__ __device__ __forceinline__ Philox4 philox4x32_10(uint32_t c0, uint32_t c1, uint32_t c2, uint32_t c3,
                                                         uint32_t k0, uint32_t k1) {
  constexpr uint32_t M0 = 0xD2511F53u, M1 = 0xCD9E8D57u, W0 = 0x9E3779B9u, W1 = 0xBB67AE85u;
#pragma unroll
  for (int r = 0; r < 10; ++r) {
    uint32_t hi0, lo0, hi1, lo1;
    mulhilo(M0, c0, hi0, lo0);
    mulhilo(M1, c2, hi1, lo1);
    const uint32_t n0 = hi1 ^ c1 ^ k0, n2 = hi0 ^ c3 ^ k1;
    c0 = n0;
    c1 = lo1;
    c2 = n2;
    c3 = lo0;
    k0 += W0;
    k1 += W1;
  }
  return Philox4{{c0, c1, c2, c3}};
}

struct PrepArgs {
  // chunk
  int k, F, ratio, pad, kc_len, kb_dim, ms_dim;
  // actions of chunks j_lo .. j_lo + n_act - 1: keyboard then mouse values
  int j_lo, n_act;
  float act[FW_PREP_MAX_ACT][8];
  int* chunk;
  __nv_bfloat16* kc;   // [kc_len, kb_dim]
  __nv_bfloat16* gm;   // [F, pad, ms_dim]
  // image condition slice
  const __nv_bfloat16* cond;   // [cond_ch, cond_frames, H, W]
  __nv_bfloat16* cc;           // [cond_ch, F, H, W]
  int cond_ch, cond_frames, hw;
  // noise
  uint32_t seed_lo, seed_hi;
  __nv_bfloat16* dst[FW_MAX_STEPS];   // tensor t -> its buffer
  int n_noise, noise_elems;           // tensors drawn (0 = none), elements per tensor (multiple of 4)
  int noise_blocks, cc_blocks;        // grid split: [noise | cc | windows]
  int* status;
};

constexpr int kPrepThreads = 256;

__device__ __forceinline__ int chunk_of_pixel_frame(int q, int F, int ratio) {
  const int first = 1 + ratio * (F - 1);
  return q < first ? 0 : 1 + (q - first) / (ratio * F);
}

__global__ void __launch_bounds__(kPrepThreads) prep_kernel(const PrepArgs a) {
  pdl_trigger();
  pdl_wait();
  const int b = blockIdx.x;
  if (b < a.noise_blocks) {
    // ---- noise: one Philox call per thread and group of four elements
    const int groups = a.noise_elems / 4;
    const int per_t = (groups + kPrepThreads - 1) / kPrepThreads;   // blocks per tensor
    const int t = b / per_t, g = (b % per_t) * kPrepThreads + threadIdx.x;
    if (t >= a.n_noise || g >= groups) return;
    const Philox4 r = philox4x32_10((uint32_t)g, (uint32_t)t, 0u, 0u, a.seed_lo, a.seed_hi);
    float n[4];
#pragma unroll
    for (int p = 0; p < 2; ++p) {
      const float u1 = ((float)r.v[2 * p] + 0.5f) * 2.3283064365386963e-10f;   // (0, 1)
      const float u2 = ((float)r.v[2 * p + 1] + 0.5f) * 2.3283064365386963e-10f;
      const float rad = sqrtf(-2.f * logf(u1));
      float sn, cs;
      sincospif(2.f * u2, &sn, &cs);
      n[2 * p] = rad * cs;
      n[2 * p + 1] = rad * sn;
    }
    *reinterpret_cast<uint2*>(a.dst[t] + (size_t)g * 4) = make_uint2(pack_bf16(n[0], n[1]), pack_bf16(n[2], n[3]));
    return;
  }
  if (b < a.noise_blocks + a.cc_blocks) {
    // ---- condition slice: cond_ch runs of F * H * W bf16, 16 bytes per thread
    const int per_c = a.F * a.hw / 8;   // uint4 per channel
    const int i = (b - a.noise_blocks) * kPrepThreads + threadIdx.x;
    if (i >= a.cond_ch * per_c) return;
    const int c = i / per_c, o = i % per_c;
    const uint4* src = reinterpret_cast<const uint4*>(a.cond + ((size_t)c * a.cond_frames + (size_t)a.F * a.k) * a.hw);
    reinterpret_cast<uint4*>(a.cc + (size_t)c * a.F * a.hw)[o] = src[o];
    return;
  }
  // ---- chunk info and action windows (one block)
  if (threadIdx.x == 0) {
    a.chunk[0] = a.k;
    a.chunk[1] = a.F * a.k;
    a.chunk[2] = 0;
    a.chunk[3] = 0;
  }
  const int start = a.ratio * a.F * a.k;
  for (int i = threadIdx.x; i < a.kc_len; i += kPrepThreads) {
    const int q = start + i - a.pad;
    const int j = q < 0 ? 0 : chunk_of_pixel_frame(q, a.F, a.ratio);
    const int slot = j - a.j_lo;
    const bool have = slot >= 0 && slot < a.n_act;
    if (!have) record_status(a.status, DEV_PREP_ACTIONS);
    for (int d = 0; d < a.kb_dim; ++d)
      a.kc[(size_t)i * a.kb_dim + d] = __float2bfloat16_rn(have ? a.act[slot][d] : 0.f);
    // mouse window: frame f reads window positions ratio * f .. ratio * f + pad - 1
    for (int f = 0; f < a.F; ++f) {
      const int p = i - a.ratio * f;
      if (p < 0 || p >= a.pad) continue;
      for (int d = 0; d < a.ms_dim; ++d)
        a.gm[((size_t)f * a.pad + p) * a.ms_dim + d] = __float2bfloat16_rn(have ? a.act[slot][a.kb_dim + d] : 0.f);
    }
  }
}

}  // namespace

}  // namespace fw

extern "C" int fw_philox4x32_10(const unsigned* counter4, const unsigned* key2, unsigned* out4) {
  if (!counter4 || !key2 || !out4) return FW_EINVAL;
  const fw::Philox4 r = fw::philox4x32_10(counter4[0], counter4[1], counter4[2], counter4[3], key2[0], key2[1]);
  for (int i = 0; i < 4; ++i) out4[i] = r.v[i];
  return FW_OK;
}

namespace fw {

int prep_launch(const fw_config& c, const fw_prep_args& p, int* chunk, __nv_bfloat16* kc, __nv_bfloat16* gm,
                __nv_bfloat16* cc, __nv_bfloat16* const* noise_dst, int n_noise, int* status, cudaStream_t s) {
  const int F = c.frames, hw = c.lat_h * c.lat_w;
  if (p.chunk < 0 || p.n_act < 1 || p.n_act > FW_PREP_MAX_ACT || p.j_lo < 0 || p.j_lo > p.chunk) return FW_EINVAL;
  if (c.keyboard_dim + c.mouse_dim > 8) return FW_ESHAPE;
  if (!p.cond || p.cond_frames < F * (p.chunk + 1) || (reinterpret_cast<uintptr_t>(p.cond) & 15u)) return FW_EINVAL;
  if (hw % 8) return FW_ESHAPE;   // 16-byte runs of the condition slice
  PrepArgs a = {};
  a.k = p.chunk;
  a.F = F;
  a.ratio = c.time_ratio;
  a.pad = c.time_ratio * c.window;
  a.kc_len = F * c.time_ratio + a.pad - 3;
  a.kb_dim = c.keyboard_dim;
  a.ms_dim = c.mouse_dim;
  a.j_lo = p.j_lo;
  a.n_act = p.n_act;
  for (int j = 0; j < p.n_act; ++j)
    for (int d = 0; d < 8; ++d) a.act[j][d] = d < c.keyboard_dim + c.mouse_dim ? p.actions[j * 8 + d] : 0.f;
  a.chunk = chunk;
  a.kc = kc;
  a.gm = gm;
  a.cond = reinterpret_cast<const __nv_bfloat16*>(p.cond);
  a.cc = cc;
  a.cond_ch = c.cond_ch;
  a.cond_frames = p.cond_frames;
  a.hw = hw;
  a.seed_lo = (uint32_t)(p.seed & 0xffffffffull);
  a.seed_hi = (uint32_t)(p.seed >> 32);
  a.n_noise = p.draw_noise ? n_noise : 0;
  a.noise_elems = c.lat_ch * F * hw;
  if (a.noise_elems % 4 || n_noise > FW_MAX_STEPS) return FW_ESHAPE;
  for (int t = 0; t < n_noise; ++t) a.dst[t] = noise_dst[t];
  const int per_t = (a.noise_elems / 4 + kPrepThreads - 1) / kPrepThreads;
  a.noise_blocks = a.n_noise * per_t;
  a.cc_blocks = (c.cond_ch * F * hw / 8 + kPrepThreads - 1) / kPrepThreads;
  a.status = status;
  launch_k(prep_kernel, a.noise_blocks + a.cc_blocks + 1, kPrepThreads, 0, s, a);
  return cudaGetLastError() == cudaSuccess ? 0 : FW_ECUDA;
}

}  // namespace fw
