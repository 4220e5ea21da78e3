// The LingBot-World-v2 causal chunk runtime (the reference's StaticLingbot,
// fastworld/models/lingbot_v2/static.py:49-320) on the library's sm_100a kernels.
//
// One chunk = the camera branch (static.py:188-207, hoisted: once per chunk), 4 denoising
// forwards with x0 = x - sigma * flow in fp64 and renoising (266-277), a forward at t = 0 over
// x0 that refreshes the chunk's keys (278-279), and the end-of-chunk roll of the KV window (280-281,
// 257-264).  A forward (209-255) writes its RoPE'd keys and values into the per-layer KV buffer at
// the plan's write offset, then attends to the buffer's first key_len frames; the self-attention
// residual update is followed by the camera affine xs = (1 + scale) * xs + shift; cross-attention
// reads the prompt's K/V (fw_lb_set_prompt, 128-137).
//
// The chunk's plan (write offset, key length, roll) and chunk index live in device memory
// (tensors "plan", "chunk"), so one captured graph serves every chunk; the roll is a sequence
// of non-overlapping piece copies, as the eager runtime's (static.py:257-264), whose count the
// plan sets on the device.
//
// GEMMs, attention, LayerNorm, RMSNorm + RoPE, the time embedding, patchify and the RoPE table
// are the kernels the MG2 engine uses; this file adds the elementwise pieces (fp32 patchify,
// SiLU, add, camera affine, KV write and roll, the fp32 / fp64 scheduler) and the launch plan.
#include <cmath>
#include <cstring>
#include <string>
#include <vector>

#include "../../include/fastworld_b200.h"
#include "fw_elem.h"
#include "fw_internal.h"
#include "fw_ptx.cuh"

namespace fw {
namespace lb {

// A[token, c * 4 + i * 2 + j] = bf16(cat(x, y)[c, f, 2 h + i, 2 w + j]) from fp32 x and y.
__global__ void patchify_f32_kernel(const float* __restrict__ x, int C1, const float* __restrict__ y, int C2, int F,
                                    int H, int W, __nv_bfloat16* __restrict__ A) {
  pdl_trigger();
  pdl_wait();
  const int th = H / 2, tw = W / 2, Kp = (C1 + C2) * 4;
  const int L = F * th * tw;
  const int idx = blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= L * Kp) return;
  const int tok = idx / Kp, k = idx % Kp;
  const int c = k >> 2, i = (k >> 1) & 1, j = k & 1;
  const int f = tok / (th * tw), h = (tok / tw) % th, w = tok % tw;
  const size_t off = (((size_t)f * H) + 2 * h + i) * W + 2 * w + j;
  A[idx] = __float2bfloat16(c < C1 ? x[(size_t)c * F * H * W + off] : y[(size_t)(c - C1) * F * H * W + off]);
}

// x = silu(x) in place (bf16, as the eager bf16 module computes it: the activation of a bf16
// tensor, rounded to bf16).
__global__ void silu_kernel(__nv_bfloat16* __restrict__ x, size_t n) {
  pdl_trigger();
  pdl_wait();
  const size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i * 8 >= n) return;
  uint4 u = reinterpret_cast<uint4*>(x)[i];
  uint32_t* w = reinterpret_cast<uint32_t*>(&u);
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    const float2 v = unpack_bf16(w[k]);
    w[k] = pack_bf16(v.x / (1.f + __expf(-v.x)), v.y / (1.f + __expf(-v.y)));
  }
  reinterpret_cast<uint4*>(x)[i] = u;
}

// out = bf16(a + b).
__global__ void add_kernel(const __nv_bfloat16* __restrict__ a, const __nv_bfloat16* __restrict__ b,
                           __nv_bfloat16* __restrict__ out, size_t n) {
  pdl_trigger();
  pdl_wait();
  const size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i * 8 >= n) return;
  const uint4 ua = reinterpret_cast<const uint4*>(a)[i], ub = reinterpret_cast<const uint4*>(b)[i];
  const uint32_t* wa = reinterpret_cast<const uint32_t*>(&ua);
  const uint32_t* wb = reinterpret_cast<const uint32_t*>(&ub);
  uint4 uo;
  uint32_t* wo = reinterpret_cast<uint32_t*>(&uo);
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    const float2 va = unpack_bf16(wa[k]), vb = unpack_bf16(wb[k]);
    wo[k] = pack_bf16(va.x + vb.x, va.y + vb.y);
  }
  reinterpret_cast<uint4*>(out)[i] = uo;
}

// xs = bf16(1 + scale) * xs + shift (fp32 residual; the camera scale and shift bf16 [L, D]; the
// eager module forms 1 + scale as a bf16 tensor, static.py:207).
__global__ void cam_affine_kernel(float* __restrict__ xs, const __nv_bfloat16* __restrict__ sc,
                                  const __nv_bfloat16* __restrict__ sh, size_t n) {
  pdl_trigger();
  pdl_wait();
  const size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i * 4 >= n) return;
  float4 x = reinterpret_cast<float4*>(xs)[i];
  const uint2 a = reinterpret_cast<const uint2*>(sc)[i], b = reinterpret_cast<const uint2*>(sh)[i];
  float2 a0 = unpack_bf16(a.x), a1 = unpack_bf16(a.y);
  const float2 b0 = unpack_bf16(b.x), b1 = unpack_bf16(b.y);
  a0 = unpack_bf16(pack_bf16(1.f + a0.x, 1.f + a0.y));
  a1 = unpack_bf16(pack_bf16(1.f + a1.x, 1.f + a1.y));
  x.x = a0.x * x.x + b0.x;
  x.y = a0.y * x.y + b0.y;
  x.z = a1.x * x.z + b1.x;
  x.w = a1.y * x.w + b1.y;
  reinterpret_cast<float4*>(xs)[i] = x;
}

// K[woff : woff + L] = k, V[woff : woff + L] = v (rows of D bf16; woff = plan[0] rows, read on
// the device; rows past the buffer are not written).
__global__ void kv_write_kernel(__nv_bfloat16* __restrict__ K, __nv_bfloat16* __restrict__ V,
                                const __nv_bfloat16* __restrict__ k, const __nv_bfloat16* __restrict__ v,
                                const int* __restrict__ plan, int L, int D, int cap) {
  pdl_trigger();
  pdl_wait();
  const int woff = __ldg(plan);
  const size_t n16 = (size_t)L * D / 8;
  const size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n16 || woff < 0) return;
  const size_t row = i * 8 / D;
  if ((size_t)woff + row >= (size_t)cap) return;
  const size_t o = (size_t)woff * D / 8 + i;
  reinterpret_cast<uint4*>(K)[o] = reinterpret_cast<const uint4*>(k)[i];
  reinterpret_cast<uint4*>(V)[o] = reinterpret_cast<const uint4*>(v)[i];
}

// One piece of the end-of-chunk roll for every layer's K and V (blockIdx.y = buffer):
// rows [src + p sh, src + min((p + 1) sh, n)) move to dst + p sh.  plan[3..6] = src, dst, n, sh
// (rows; n = 0: no roll).  Pieces run in order as separate launches, so a piece never reads
// rows an earlier piece of the same launch writes (sh = src - dst).
struct RollPtrs {
  __nv_bfloat16* buf[2 * 64];
};
__global__ void roll_kernel(const RollPtrs p, const int* __restrict__ plan, int piece, int D, int cap) {
  pdl_trigger();
  pdl_wait();
  const int src = __ldg(plan + 3), dst = __ldg(plan + 4), n = __ldg(plan + 5), sh = __ldg(plan + 6);
  if (n <= 0 || sh <= 0) return;
  const int r0 = piece * sh;
  if (r0 >= n) return;
  const int rows = min(sh, n - r0);
  if (src + r0 + rows > cap || dst + r0 + rows > cap || dst < 0) return;
  __nv_bfloat16* b = p.buf[blockIdx.y];
  const size_t n16 = (size_t)rows * D / 8;
  const uint4* s4 = reinterpret_cast<const uint4*>(b + (size_t)(src + r0) * D);
  uint4* d4 = reinterpret_cast<uint4*>(b + (size_t)(dst + r0) * D);
  for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n16; i += (size_t)gridDim.x * blockDim.x)
    d4[i] = s4[i];
}

// flow[c, f, h, w] = head[token(f, h/2, w/2), ((h%2) * 2 + (w%2)) * C + c];
// x0 = fp32(fp64(x) - sig_x0 * fp64(flow)); xnext = alpha * x0 + sigma * noise (fp32).
__global__ void scheduler_kernel(const float* __restrict__ head, const float* __restrict__ x, double sig_x0,
                                 float* __restrict__ x0, const float* __restrict__ noise, float alpha, float sigma,
                                 float* __restrict__ xnext, int C, int F, int H, int W) {
  pdl_trigger();
  pdl_wait();
  const int idx = blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= C * F * H * W) return;
  const int w = idx % W, h = (idx / W) % H, f = (idx / (W * H)) % F, c = idx / (W * H * F);
  const int tok = (f * (H / 2) + h / 2) * (W / 2) + w / 2;
  const float flow = head[(size_t)tok * (4 * C) + ((h & 1) * 2 + (w & 1)) * C + c];
  const float d = (float)((double)x[idx] - sig_x0 * (double)flow);
  x0[idx] = d;
  if (xnext) xnext[idx] = alpha * d + sigma * noise[idx];
}

inline unsigned blocks(size_t n, int per) { return (unsigned)((n + per - 1) / per); }

struct Gemm {
  CUtensorMap a{}, b{}, c{}, o[3] = {};
  GemmArgs args;
  int bn = 256;
  bool has_c = false;
};
struct Attn {
  CUtensorMap q{}, k0{}, v0{}, k1{}, v1{}, o{};
  AttnArgs args;
};
struct Layer {
  Gemm qkv, o, caq, cao, ff0, ff2, inj1, inj2, scale, shift, cakv;
  Attn self, cross;
};

}  // namespace lb
}  // namespace fw

struct fw_lb {
  fw_lb_config cfg{};
  struct Tensor {
    std::string name;
    int kind, dtype, ndim;
    int64_t shape[5];
    size_t bytes;
    void* ptr = nullptr;
  };
  std::vector<Tensor> tensors;
  std::vector<std::pair<std::string, size_t>> ws;   // workspace slices (name, offset)
  size_t ws_bytes = 0;
  bool finalized = false;
  int L = 0, D = 0, Ft = 0, cap = 0, roll_pieces = 0;
  std::vector<fw::lb::Layer> layers;
  fw::lb::Gemm patch, cam_in, c2ws1, c2ws2, head, te0, te2;
  int* status = nullptr;
};

namespace {

using namespace fw;
using namespace fw::lb;

int find(const fw_lb* h, const std::string& n) {
  for (size_t i = 0; i < h->tensors.size(); ++i)
    if (h->tensors[i].name == n) return (int)i;
  return -1;
}
size_t dsize(int dt) { return dt == FW_F32 || dt == FW_I32 ? 4 : (dt == FW_U8 ? 1 : 2); }
void add(fw_lb* h, const std::string& n, int kind, int dt, std::vector<int64_t> shape) {
  fw_lb::Tensor t;
  t.name = n;
  t.kind = kind;
  t.dtype = dt;
  t.ndim = (int)shape.size();
  size_t e = 1;
  for (int i = 0; i < 5; ++i) t.shape[i] = i < t.ndim ? shape[i] : 0;
  for (int64_t d : shape) e *= (size_t)d;
  t.bytes = e * dsize(dt);
  h->tensors.push_back(t);
}
template <typename T = void>
T* P(fw_lb* h, const std::string& n) {
  const int i = find(h, n);
  return i < 0 ? nullptr : static_cast<T*>(h->tensors[i].ptr);
}
const __nv_bfloat16* W(fw_lb* h, const std::string& n) { return P<const __nv_bfloat16>(h, n); }
void ws_add(fw_lb* h, const std::string& n, size_t bytes) {
  h->ws.push_back({n, h->ws_bytes});
  h->ws_bytes += (bytes + 1023) & ~(size_t)1023;
}
template <typename T = __nv_bfloat16>
T* WS(fw_lb* h, const std::string& n) {
  char* base = static_cast<char*>(P(h, "workspace"));
  for (auto& s : h->ws)
    if (s.first == n) return reinterpret_cast<T*>(base + s.second);
  return nullptr;
}

#define LB_TRY(x)            \
  do {                       \
    const int _rc = (x);     \
    if (_rc) return _rc;     \
  } while (0)

int pick_bn(int N) { return N >= 256 ? 256 : (N >= 128 ? 128 : 64); }

// C[M, N] = A[M, K] B[N, K]^T with epilogue `e` (bf16 outputs by TMA store; a gated residual
// becomes a TMA reduce-add into the fp32 residual).
int make_gemm(Gemm& g, const void* A, int M, int K, const void* B, int N, const GemmEpi& e, int* status) {
  g.bn = pick_bn(N);
  LB_TRY(make_tmap_2d(&g.a, A, 2, M, K, K, 128, 64, true));
  LB_TRY(make_tmap_2d(&g.b, B, 2, N, K, K, g.bn, 64, true));
  g.args.M = M;
  g.args.N = N;
  g.args.K = K;
  g.args.epi = e;
  g.args.status = status;
  g.args.b_static = true;
  if (e.mode == EPI_RESID_F32 && !e.mirror && resid_tma_enabled()) {
    LB_TRY(make_tmap_2d(&g.c, e.resid, 4, M, N, e.ld_resid, 32, 32, true));
    g.args.epi.mode = EPI_RESID_TMA;
    g.has_c = true;
  }
  LB_TRY(make_out_tmaps(g.args, g.o));
  return gemm_check(g.args, g.bn);
}
int run(const Gemm& g, cudaStream_t s) {
  return gemm_bf16_launch(g.a, g.b, g.bn, g.args, s, 0, g.has_c ? &g.c : nullptr, g.o);
}
GemmEpi epi_out(void* out, int ld, const __nv_bfloat16* bias, int mode = EPI_BF16) {
  GemmEpi e;
  e.mode = mode;
  e.out[0] = out;
  e.ld_out = ld;
  e.seg_w = 1 << 30;
  e.bias = bias;
  return e;
}
GemmEpi epi_resid(float* xs, int ld, const __nv_bfloat16* bias, const float* gate) {
  GemmEpi e;
  e.mode = EPI_RESID_F32;
  e.resid = xs;
  e.ld_resid = ld;
  e.bias = bias;
  e.gate = gate;
  return e;
}
int make_attn(Attn& a, const void* q, int Lq, int heads, const void* k0, const void* v0, int cap0, const void* k1,
              const void* v1, int cap1, const int* meta, void* out, int* status) {
  const int cols = heads * 128;
  LB_TRY(make_tmap_2d(&a.q, q, 2, Lq, cols, cols, 128, 64, true));
  LB_TRY(make_tmap_2d(&a.k0, k0, 2, cap0, cols, cols, 128, 64, true));
  LB_TRY(make_tmap_2d(&a.v0, v0, 2, cap0, cols, cols, 128, 64, true));
  LB_TRY(make_tmap_2d(&a.k1, k1, 2, cap1, cols, cols, 128, 64, true));
  LB_TRY(make_tmap_2d(&a.v1, v1, 2, cap1, cols, cols, 128, 64, true));
  LB_TRY(make_tmap_2d(&a.o, out, 2, Lq, cols, cols, 128, 64, true));
  a.args.Lq = Lq;
  a.args.heads = heads;
  a.args.meta = meta;
  a.args.max_keys0 = cap0;
  a.args.max_keys1 = cap1;
  a.args.out = static_cast<__nv_bfloat16*>(out);
  a.args.ld_out = cols;
  a.args.scale_log2 = (float)(1.4426950408889634 / std::sqrt(128.0));
  a.args.status = status;
  return 0;
}
int run(const Attn& a, cudaStream_t s) { return attention_launch(a.q, a.k0, a.v0, a.k1, a.v1, a.args, s, &a.o); }

// The eager runtime's KV bookkeeping (static.py:30-46): the largest number of roll pieces any
// chunk needs (ceil(moved / evicted)).
int max_roll_pieces(int C, int Wn, int S) {
  int local_end = 0, global_end = 0, best = 0;
  for (int c = 0; c < 256; ++c) {
    const int cur_end = (c + 1) * C;
    if (cur_end > global_end && C + local_end > Wn) {
      const int ev = C + local_end - Wn, moved = local_end - ev - S;
      if (moved > 0 && ev > 0) best = std::max(best, (moved + ev - 1) / ev);
      local_end = local_end + cur_end - global_end - ev;
    } else {
      local_end = local_end + cur_end - global_end;
    }
    global_end = cur_end;
  }
  return best;
}

// ------------------------------------------------------------------ launch sequence
int camera(fw_lb* h, cudaStream_t s) {
  const fw_lb_config& c = h->cfg;
  const size_t n = (size_t)h->L * h->D;
  __nv_bfloat16 *emb = WS(h, "cam_emb"), *t = WS(h, "cam_t"), *hh = WS(h, "cam_h");
  LB_TRY(patchify(P<__nv_bfloat16>(h, "pl_in"), c.cam_ch, nullptr, 0, c.chunk, c.lat_h, c.lat_w, WS(h, "camA"), s));
  LB_TRY(run(h->cam_in, s));   // emb = Linear(Plücker patches)
  LB_TRY(run(h->c2ws1, s));    // t = c2ws1(emb)
  launch_k(silu_kernel, blocks(n / 8, 256), 256, 0, s, t, n);
  LB_TRY(run(h->c2ws2, s));    // h = c2ws2(silu(t))
  launch_k(add_kernel, blocks(n / 8, 256), 256, 0, s, emb, hh, emb, n);   // emb += h
  for (int i = 0; i < c.layers; ++i) {
    const Layer& ly = h->layers[i];
    LB_TRY(run(ly.inj1, s));
    launch_k(silu_kernel, blocks(n / 8, 256), 256, 0, s, t, n);
    LB_TRY(run(ly.inj2, s));
    launch_k(add_kernel, blocks(n / 8, 256), 256, 0, s, hh, emb, hh, n);   // h = inj2(...) + emb
    LB_TRY(run(ly.scale, s));
    LB_TRY(run(ly.shift, s));
  }
  return cudaGetLastError() == cudaSuccess ? 0 : FW_ECUDA;
}

// One forward at step `step` (n_steps = the t = 0 key refresh) of latent x (fp32).
int forward(fw_lb* h, int step, const float* x, float* x0, const float* noise, float* xnext, bool head,
            cudaStream_t s) {
  const fw_lb_config& c = h->cfg;
  const int L = h->L, D = h->D;
  const double t = step < c.n_steps ? (double)c.timesteps[step] : 0.0;
  float *tsin = WS<float>(h, "tsin"), *th = WS<float>(h, "th"), *e = WS<float>(h, "e"), *e0 = WS<float>(h, "e0");
  float *ee = WS<float>(h, "ee"), *hmod = WS<float>(h, "hmod"), *xs = WS<float>(h, "xs");
  LB_TRY(sinusoid(t, c.freq_dim, tsin, s));
  LB_TRY(smallm_linear_f32(tsin, c.freq_dim, 1, W(h, "time.0.w"), c.freq_dim, W(h, "time.0.b"), D, c.freq_dim,
                           ACT_NONE, ACT_SILU, th, nullptr, D, s));
  LB_TRY(smallm_linear_f32(th, D, 1, W(h, "time.2.w"), D, W(h, "time.2.b"), D, D, ACT_NONE, ACT_NONE, e, nullptr, D, s));
  LB_TRY(smallm_linear_f32(e, D, 1, W(h, "tproj.w"), D, W(h, "tproj.b"), 6 * D, D, ACT_SILU, ACT_NONE, e0, nullptr,
                           6 * D, s));
  LB_TRY(modulation(W(h, "mods"), e0, c.layers, D, ee, W(h, "head.mod"), e, hmod, s));
  const int Cin = c.lat_ch + c.y_ch;
  launch_k(patchify_f32_kernel, blocks((size_t)L * Cin * 4, 256), 256, 0, s, x, c.lat_ch, P<const float>(h, "y_in"),
           c.y_ch, c.chunk, c.lat_h, c.lat_w, WS(h, "patchA"));
  LB_TRY(run(h->patch, s));
  const float2* rope = WS<float2>(h, "rope");
  __nv_bfloat16 *y = WS(h, "y"), *q = WS(h, "q"), *kc = WS(h, "kcur"), *vc = WS(h, "vcur");
  const int* plan = P<const int>(h, "plan");
  const size_t n = (size_t)L * D;
  for (int i = 0; i < c.layers; ++i) {
    const Layer& ly = h->layers[i];
    const std::string p = "b" + std::to_string(i) + ".";
    const float* e6 = ee + (size_t)i * 6 * D;
    LB_TRY(ln_f32(xs, D, L, D, c.eps, e6, e6 + D, nullptr, nullptr, y, D, s));
    LB_TRY(run(ly.qkv, s));
    LB_TRY(rms_rope2(q, W(h, p + "sa.nq.w"), q, kc, W(h, p + "sa.nk.w"), kc, D, L, D, c.eps, rope, c.head_dim, D, s));
    // keys and values enter the window before the attention reads it (static.py:228-231)
    launch_k(kv_write_kernel, blocks(n / 8, 256), 256, 0, s, P<__nv_bfloat16>(h, "K." + std::to_string(i)),
             P<__nv_bfloat16>(h, "V." + std::to_string(i)), (const __nv_bfloat16*)kc, (const __nv_bfloat16*)vc, plan, L,
             D, h->cap);
    LB_TRY(run(ly.self, s));
    LB_TRY(run(ly.o, s));
    launch_k(cam_affine_kernel, blocks(n / 4, 256), 256, 0, s, xs, (const __nv_bfloat16*)(WS(h, "cam1") + (size_t)i * n),
             (const __nv_bfloat16*)(WS(h, "camb") + (size_t)i * n), n);
    LB_TRY(ln_f32(xs, D, L, D, c.eps, nullptr, nullptr, W(h, p + "n3.w"), W(h, p + "n3.b"), y, D, s));
    LB_TRY(run(ly.caq, s));
    LB_TRY(rms_rope2(q, W(h, p + "ca.nq.w"), q, nullptr, nullptr, nullptr, D, L, D, c.eps, nullptr, c.head_dim, D, s));
    LB_TRY(run(ly.cross, s));
    LB_TRY(run(ly.cao, s));
    LB_TRY(ln_f32(xs, D, L, D, c.eps, e6 + 3 * D, e6 + 4 * D, nullptr, nullptr, y, D, s));
    LB_TRY(run(ly.ff0, s));
    LB_TRY(run(ly.ff2, s));
  }
  if (!head) return cudaGetLastError() == cudaSuccess ? 0 : FW_ECUDA;
  LB_TRY(ln_f32(xs, D, L, D, c.eps, hmod, hmod + D, nullptr, nullptr, y, D, s));
  LB_TRY(run(h->head, s));
  const bool renoise = xnext != nullptr;
  launch_k(scheduler_kernel, blocks((size_t)c.lat_ch * c.chunk * c.lat_h * c.lat_w, 256), 256, 0, s,
           (const float*)WS<float>(h, "headout"), x, step < c.n_steps ? c.sig_x0[step] : 0.0, x0, noise,
           renoise ? c.an_alpha[step] : 0.f, renoise ? c.an_sigma[step] : 0.f, xnext, c.lat_ch, c.chunk, c.lat_h,
           c.lat_w);
  return cudaGetLastError() == cudaSuccess ? 0 : FW_ECUDA;
}

int chunk(fw_lb* h, cudaStream_t s) {
  const fw_lb_config& c = h->cfg;
  LB_TRY(rope_tables(P<const int>(h, "chunk"), c.chunk, c.lat_h / 2, c.lat_w / 2, c.head_dim, 10000.0,
                     WS<float2>(h, "rope"), 0, nullptr, nullptr, s));
  LB_TRY(camera(h, s));
  const float* x = P<const float>(h, "x_in");
  float* bufs[2] = {WS<float>(h, "xa"), WS<float>(h, "xb")};
  float* x0 = WS<float>(h, "x0");
  for (int i = 0; i < c.n_steps; ++i) {
    const bool last = i == c.n_steps - 1;
    float* out = last ? P<float>(h, "out") : x0;
    LB_TRY(forward(h, i, x, out, last ? nullptr : P<const float>(h, "noise." + std::to_string(i)),
                   last ? nullptr : bufs[i & 1], true, s));
    x = bufs[i & 1];
  }
  // the t = 0 forward over the denoised latent refreshes the chunk's keys (static.py:278-279)
  LB_TRY(forward(h, c.n_steps, P<const float>(h, "out"), nullptr, nullptr, nullptr, false, s));
  RollPtrs rp{};
  for (int i = 0; i < c.layers; ++i) {
    rp.buf[2 * i] = P<__nv_bfloat16>(h, "K." + std::to_string(i));
    rp.buf[2 * i + 1] = P<__nv_bfloat16>(h, "V." + std::to_string(i));
  }
  for (int piece = 0; piece < h->roll_pieces; ++piece)
    launch_k(roll_kernel, dim3(64, 2 * c.layers), 256, 0, s, rp, P<const int>(h, "plan"), piece, h->D, h->cap);
  return cudaGetLastError() == cudaSuccess ? 0 : FW_ECUDA;
}

}  // namespace

extern "C" {

int fw_lb_create(const fw_lb_config* cfg, fw_lb** out) {
  if (!cfg || !out) return FW_EINVAL;
  *out = nullptr;
  const fw_lb_config& c = *cfg;
  if (c.dim != c.heads * c.head_dim || c.head_dim != 128 || c.dim % 256 || c.ffn % 256 || c.layers < 1 ||
      c.layers > 64 || c.n_steps < 1 || c.n_steps > 8 || c.lat_h % 2 || c.lat_w % 2 || c.chunk < 1 ||
      c.kv_frames < c.chunk || c.sink_frames < 0 || c.sink_frames >= c.kv_frames || c.text_len < 1 ||
      c.text_dim % 8 || (c.cam_ch * 4) % 8 || c.lat_ch != 16)
    return FW_ESHAPE;
  fw_lb* h = new fw_lb();
  h->cfg = c;
  h->D = c.dim;
  h->Ft = (c.lat_h / 2) * (c.lat_w / 2);
  h->L = c.chunk * h->Ft;
  h->cap = c.kv_frames * h->Ft;
  h->roll_pieces = max_roll_pieces(c.chunk, c.kv_frames, c.sink_frames);
  const int D = c.dim, L = h->L, Cin = c.lat_ch + c.y_ch;
  auto wt = [&](const std::string& n, std::vector<int64_t> s) { add(h, n, FW_KIND_WEIGHT, FW_BF16, s); };
  wt("patch.w", {D, Cin * 4});
  wt("patch.b", {D});
  wt("text.0.w", {D, c.text_dim});
  wt("text.0.b", {D});
  wt("text.2.w", {D, D});
  wt("text.2.b", {D});
  wt("time.0.w", {D, c.freq_dim});
  wt("time.0.b", {D});
  wt("time.2.w", {D, D});
  wt("time.2.b", {D});
  wt("tproj.w", {6 * D, D});
  wt("tproj.b", {6 * D});
  wt("cam.in.w", {D, c.cam_ch * 4});
  wt("cam.in.b", {D});
  wt("cam.h1.w", {D, D});
  wt("cam.h1.b", {D});
  wt("cam.h2.w", {D, D});
  wt("cam.h2.b", {D});
  wt("head.mod", {2, D});
  wt("head.w", {4 * c.lat_ch, D});
  wt("head.b", {4 * c.lat_ch});
  wt("mods", {c.layers, 6, D});
  for (int i = 0; i < c.layers; ++i) {
    const std::string p = "b" + std::to_string(i) + ".";
    wt(p + "sa.qkv.w", {3 * D, D});
    wt(p + "sa.qkv.b", {3 * D});
    wt(p + "sa.o.w", {D, D});
    wt(p + "sa.o.b", {D});
    wt(p + "sa.nq.w", {D});
    wt(p + "sa.nk.w", {D});
    wt(p + "n3.w", {D});
    wt(p + "n3.b", {D});
    wt(p + "ca.q.w", {D, D});
    wt(p + "ca.q.b", {D});
    wt(p + "ca.kv.w", {2 * D, D});
    wt(p + "ca.kv.b", {2 * D});
    wt(p + "ca.o.w", {D, D});
    wt(p + "ca.o.b", {D});
    wt(p + "ca.nq.w", {D});
    wt(p + "ca.nk.w", {D});
    wt(p + "ffn.0.w", {c.ffn, D});
    wt(p + "ffn.0.b", {c.ffn});
    wt(p + "ffn.2.w", {D, c.ffn});
    wt(p + "ffn.2.b", {D});
    for (const char* m : {"inj1", "inj2", "scale", "shift"}) {
      wt(p + "cam." + m + ".w", {D, D});
      wt(p + "cam." + m + ".b", {D});
    }
  }
  for (int i = 0; i < c.layers; ++i) add(h, "K." + std::to_string(i), FW_KIND_STATE, FW_BF16, {h->cap, D});
  for (int i = 0; i < c.layers; ++i) add(h, "V." + std::to_string(i), FW_KIND_STATE, FW_BF16, {h->cap, D});
  const std::vector<int64_t> lat = {c.lat_ch, c.chunk, c.lat_h, c.lat_w};
  add(h, "x_in", FW_KIND_INPUT, FW_F32, lat);
  for (int i = 0; i + 1 < c.n_steps; ++i) add(h, "noise." + std::to_string(i), FW_KIND_INPUT, FW_F32, lat);
  add(h, "y_in", FW_KIND_INPUT, FW_F32, {c.y_ch, c.chunk, c.lat_h, c.lat_w});
  add(h, "pl_in", FW_KIND_INPUT, FW_BF16, {c.cam_ch, c.chunk, c.lat_h, c.lat_w});
  add(h, "ctx_in", FW_KIND_INPUT, FW_BF16, {c.text_len, c.text_dim});
  add(h, "plan", FW_KIND_INPUT, FW_I32, {8});
  add(h, "chunk", FW_KIND_INPUT, FW_I32, {4});
  add(h, "out", FW_KIND_OUTPUT, FW_F32, lat);
  add(h, "status", FW_KIND_STATUS, FW_I32, {4});
  // derived per prompt: every block's cross-attention K / V over the padded text
  add(h, "xk", FW_KIND_DERIVED, FW_BF16, {c.layers, c.text_len, D});
  add(h, "xv", FW_KIND_DERIVED, FW_BF16, {c.layers, c.text_len, D});
  const size_t bf = 2, f4 = 4, latn = (size_t)c.lat_ch * c.chunk * c.lat_h * c.lat_w;
  ws_add(h, "xs", (size_t)L * D * f4);
  for (const char* n : {"y", "q", "kcur", "vcur", "ao", "cam_emb", "cam_t", "cam_h"}) ws_add(h, n, (size_t)L * D * bf);
  ws_add(h, "hb", (size_t)L * c.ffn * bf);
  ws_add(h, "patchA", (size_t)L * Cin * 4 * bf);
  ws_add(h, "camA", (size_t)L * c.cam_ch * 4 * bf);
  ws_add(h, "cam1", (size_t)c.layers * L * D * bf);
  ws_add(h, "camb", (size_t)c.layers * L * D * bf);
  ws_add(h, "headout", (size_t)L * 4 * c.lat_ch * f4);
  for (const char* n : {"xa", "xb", "x0"}) ws_add(h, n, latn * f4);
  ws_add(h, "rope", (size_t)L * 64 * 2 * f4);
  ws_add(h, "tsin", (size_t)c.freq_dim * f4);
  ws_add(h, "th", (size_t)D * f4);
  ws_add(h, "e", (size_t)D * f4);
  ws_add(h, "e0", (size_t)6 * D * f4);
  ws_add(h, "ee", (size_t)c.layers * 6 * D * f4);
  ws_add(h, "hmod", (size_t)2 * D * f4);
  ws_add(h, "ctx_a", (size_t)c.text_len * D * bf);
  ws_add(h, "ctx", (size_t)c.text_len * D * bf);
  ws_add(h, "xmeta", 16);
  add(h, "workspace", FW_KIND_WORKSPACE, FW_U8, {(int64_t)h->ws_bytes});
  *out = h;
  return FW_OK;
}

int fw_lb_tensor_count(const fw_lb* h) { return h ? (int)h->tensors.size() : FW_EINVAL; }

int fw_lb_tensor_info_at(const fw_lb* h, int index, fw_tensor_info* info) {
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

int fw_lb_bind(fw_lb* h, const char* name, void* p, size_t bytes) {
  if (!h || !name || !p || h->finalized) return FW_EINVAL;
  const int i = find(h, name);
  if (i < 0) return FW_EINVAL;
  if (bytes < h->tensors[i].bytes) return FW_ESIZE;
  if (reinterpret_cast<uintptr_t>(p) & 15u) return FW_EALIGN;
  h->tensors[i].ptr = p;
  return FW_OK;
}

int fw_lb_finalize(fw_lb* h) {
  if (!h || h->finalized) return FW_EINVAL;
  for (const auto& t : h->tensors)
    if (!t.ptr) return FW_ENOTBOUND;
  const fw_lb_config& c = h->cfg;
  const int L = h->L, D = h->D, T = c.text_len;
  h->status = P<int>(h, "status");
  int* st = h->status;
  float* xs = WS<float>(h, "xs");
  __nv_bfloat16 *y = WS(h, "y"), *q = WS(h, "q"), *kc = WS(h, "kcur"), *vc = WS(h, "vcur"), *ao = WS(h, "ao");
  __nv_bfloat16 *hb = WS(h, "hb"), *emb = WS(h, "cam_emb"), *ct = WS(h, "cam_t"), *chh = WS(h, "cam_h");
  __nv_bfloat16 *xk = P<__nv_bfloat16>(h, "xk"), *xv = P<__nv_bfloat16>(h, "xv");
  int* xmeta = WS<int>(h, "xmeta");   // {text_len, 0}: the cross-attention's key count
  const int xm[4] = {T, 0, 0, 0};
  if (cudaMemcpy(xmeta, xm, sizeof(xm), cudaMemcpyHostToDevice) != cudaSuccess) return FW_ECUDA;
  LB_TRY(make_gemm(h->patch, WS(h, "patchA"), L, (c.lat_ch + c.y_ch) * 4, W(h, "patch.w"), D,
                   epi_out(xs, D, W(h, "patch.b"), EPI_F32), st));
  LB_TRY(make_gemm(h->cam_in, WS(h, "camA"), L, c.cam_ch * 4, W(h, "cam.in.w"), D, epi_out(emb, D, W(h, "cam.in.b")),
                   st));
  LB_TRY(make_gemm(h->c2ws1, emb, L, D, W(h, "cam.h1.w"), D, epi_out(ct, D, W(h, "cam.h1.b")), st));
  LB_TRY(make_gemm(h->c2ws2, ct, L, D, W(h, "cam.h2.w"), D, epi_out(chh, D, W(h, "cam.h2.b")), st));
  LB_TRY(make_gemm(h->head, y, L, D, W(h, "head.w"), 4 * c.lat_ch,
                   epi_out(WS<float>(h, "headout"), 4 * c.lat_ch, W(h, "head.b"), EPI_F32), st));
  LB_TRY(make_gemm(h->te0, P(h, "ctx_in"), T, c.text_dim, W(h, "text.0.w"), D,
                   epi_out(WS(h, "ctx_a"), D, W(h, "text.0.b"), EPI_GELU_BF16), st));
  LB_TRY(make_gemm(h->te2, WS(h, "ctx_a"), T, D, W(h, "text.2.w"), D, epi_out(WS(h, "ctx"), D, W(h, "text.2.b")), st));
  h->layers.resize(c.layers);
  const size_t n = (size_t)L * D;
  for (int i = 0; i < c.layers; ++i) {
    Layer& ly = h->layers[i];
    const std::string p = "b" + std::to_string(i) + ".";
    GemmEpi sq = epi_out(q, D, W(h, p + "sa.qkv.b"));
    sq.out[1] = kc;
    sq.out[2] = vc;
    sq.seg_w = D;
    LB_TRY(make_gemm(ly.qkv, y, L, D, W(h, p + "sa.qkv.w"), 3 * D, sq, st));
    const float* e6 = WS<float>(h, "ee") + (size_t)i * 6 * D;
    LB_TRY(make_gemm(ly.o, ao, L, D, W(h, p + "sa.o.w"), D, epi_resid(xs, D, W(h, p + "sa.o.b"), e6 + 2 * D), st));
    LB_TRY(make_gemm(ly.caq, y, L, D, W(h, p + "ca.q.w"), D, epi_out(q, D, W(h, p + "ca.q.b")), st));
    LB_TRY(make_gemm(ly.cao, ao, L, D, W(h, p + "ca.o.w"), D, epi_resid(xs, D, W(h, p + "ca.o.b"), nullptr), st));
    LB_TRY(make_gemm(ly.ff0, y, L, D, W(h, p + "ffn.0.w"), c.ffn, epi_out(hb, c.ffn, W(h, p + "ffn.0.b"), EPI_GELU_BF16),
                     st));
    LB_TRY(make_gemm(ly.ff2, hb, L, c.ffn, W(h, p + "ffn.2.w"), D, epi_resid(xs, D, W(h, p + "ffn.2.b"), e6 + 5 * D), st));
    LB_TRY(make_gemm(ly.inj1, emb, L, D, W(h, p + "cam.inj1.w"), D, epi_out(ct, D, W(h, p + "cam.inj1.b")), st));
    LB_TRY(make_gemm(ly.inj2, ct, L, D, W(h, p + "cam.inj2.w"), D, epi_out(chh, D, W(h, p + "cam.inj2.b")), st));
    LB_TRY(make_gemm(ly.scale, chh, L, D, W(h, p + "cam.scale.w"), D,
                     epi_out(WS(h, "cam1") + (size_t)i * n, D, W(h, p + "cam.scale.b")), st));
    LB_TRY(make_gemm(ly.shift, chh, L, D, W(h, p + "cam.shift.w"), D,
                     epi_out(WS(h, "camb") + (size_t)i * n, D, W(h, p + "cam.shift.b")), st));
    GemmEpi kv = epi_out(xk + (size_t)i * T * D, D, W(h, p + "ca.kv.b"));
    kv.out[1] = xv + (size_t)i * T * D;
    kv.seg_w = D;
    LB_TRY(make_gemm(ly.cakv, WS(h, "ctx"), T, D, W(h, p + "ca.kv.w"), 2 * D, kv, st));
    // self-attention: the window's first key_len rows (plan[1]; plan[2] = 0 keys in segment 1)
    LB_TRY(make_attn(ly.self, q, L, c.heads, P(h, "K." + std::to_string(i)), P(h, "V." + std::to_string(i)), h->cap,
                     kc, vc, L, P<const int>(h, "plan") + 1, ao, st));
    LB_TRY(make_attn(ly.cross, q, L, c.heads, xk + (size_t)i * T * D, xv + (size_t)i * T * D, T, kc, vc, L, xmeta, ao,
                     st));
  }
  h->finalized = true;
  return FW_OK;
}

int fw_lb_set_prompt(fw_lb* h, void* stream) {
  if (!h || !h->finalized) return FW_EINVAL;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const fw_lb_config& c = h->cfg;
  LB_TRY(run(h->te0, s));
  LB_TRY(run(h->te2, s));
  for (int i = 0; i < c.layers; ++i) {
    const std::string p = "b" + std::to_string(i) + ".";
    LB_TRY(run(h->layers[i].cakv, s));
    __nv_bfloat16* k = P<__nv_bfloat16>(h, "xk") + (size_t)i * c.text_len * c.dim;
    LB_TRY(rms_rope2(k, W(h, p + "ca.nk.w"), k, nullptr, nullptr, nullptr, c.dim, c.text_len, c.dim, c.eps, nullptr,
                     c.head_dim, c.dim, s));
  }
  return cudaGetLastError() == cudaSuccess ? FW_OK : FW_ECUDA;
}

int fw_lb_chunk(fw_lb* h, void* stream) {
  if (!h || !h->finalized) return FW_EINVAL;
  return chunk(h, static_cast<cudaStream_t>(stream));
}

int fw_lb_roll_pieces(const fw_lb* h) { return h ? h->roll_pieces : FW_EINVAL; }

void fw_lb_destroy(fw_lb* h) { delete h; }

}  // extern "C"
