// Session engine: the chunk forward of the Matrix-Game-2-shaped causal Wan DiT as a fixed
// sequence of sm_100a kernel launches over caller-owned buffers.
//
// Mirrors StaticMG (fastworld/models/mg2/static.py:27-284): static buffers bound once
// (__init__, 28-73), `_net` (194-230) as fw_forward, `_chunk` (232-242) as fw_chunk and
// `_prefill` (244-245) as fw_prefill.  All TMA descriptors and kernel arguments are built at
// fw_finalize; a launch call only enqueues kernels, so every call is graph-capturable.
//
// Work hoisted out of the per-forward loop (exact: the inputs do not change within a chunk):
// the image-context MLP and the per-block cross-attention K/V (static.py:201,190-191) and the
// keyboard K/V of the action module (static.py:165-172) are computed once per chunk.
#include <cmath>
#include <cstring>
#include <cstdio>
#include <cstdlib>
#include <string>
#include <unordered_map>
#include <vector>

#include "../../include/fastworld_b200.h"
#include "fw_elem.h"
#include "fw_internal.h"
#include "fw_tp.h"

namespace fw {

struct Tensor {
  std::string name;
  int kind, dtype, ndim;
  int64_t shape[5];
  size_t bytes;
  void* ptr = nullptr;
};

struct GemmOp {
  CUtensorMap a, b;
  CUtensorMap c;          // fp32 residual, for EPI_RESID_TMA
  CUtensorMap o[3];       // bf16 output segments, for TMA-store epilogues (args.epi.tma_store)
  bool has_c = false;
  bool pair = false;      // 256 x 256 CTA-pair tiles (gemm2.cu)
  int bn = 256;
  GemmArgs args;
  bool valid = false;
};

struct AttnOp {
  CUtensorMap q, k0, v0, k1, v1, o;
  AttnArgs args;
};

struct Layer {
  int act = -1;   // index among action blocks, -1 if none
  GemmOp qkv, o, caq, cakv, cao, ff0, ff2;
  AttnOp self_first, self_steady, cross;
  // action module
  GemmOp mlp1, mlp2, tqkv, pmouse, mattq, pkb;
};

}  // namespace fw

struct fw_handle {
  fw_config cfg;
  std::vector<fw::Tensor> tensors;
  std::unordered_map<std::string, int> index;
  bool finalized = false;
  // dims (Hl, Dl, FFl: this rank's heads, attention width and FFN width; = H, D, FF at tp 1)
  int L, S, F, D, H, HD, FF, A, AH, Mh, Kh, nA, th, tw, Ctx, Cd, Kp, OUT, KC, PAD;
  int Hl, Dl, FFl;
  int tp = 1, tpr = 0, hc = 1;   // tensor-parallel size / rank, history window in chunks
  void* comm = nullptr;           // NCCL communicator (tp > 1)
  fw::TpPeers peers;              // the other ranks' workspaces (tp > 1, after fw_tp_peers)
  bool use_peers = false;         // reductions over peer memory instead of NCCL
  bool push = false;              // row-parallel GEMMs push their partials to the other ranks
  size_t recv_stride = 0;         // elements between the two parities of tp.recv (4 / 8 ranks)
  __nv_bfloat16* part = nullptr;  // [L, D] partial output of a row-parallel linear (tp > 1)
  float* ss = nullptr;            // [max(L, Ctx), 2] sums of squares for the sharded RMSNorms
  size_t lat_elems;
  // workspace layout (offsets into "workspace")
  std::vector<std::pair<std::string, size_t>> ws_off;
  size_t ws_bytes = 0;
  // resolved pointers
  float *xs, *headout, *rope, *acos_, *asin_, *tsin, *th_, *e, *e0, *ee, *hmod, *ke1, *ke, *kbkv, *fbias;
  __nv_bfloat16 *y, *xbf, *q, *kcur, *vcur, *ao, *hb, *hb2, *patchA, *xa, *xb, *den, *den_ctx, *ctx_a, *ctx_h,
      *ctx_o, *ctx, *ckv, *kbK, *kbV;
  int* consts;
  bool fp8 = false;         // e4m3 block linears (per-channel weight / per-token activation scales)
  bool fp8_ffn_only = false;  // ... only the FFN linears (ffn.0, ffn.2); the others stay bf16
  uint8_t* a8 = nullptr;    // e4m3 operand of the next block linear
  float* sa = nullptr;      // its per-row scales
  int* status;
  std::vector<fw::Layer> layers;
  fw::GemmOp patch, head, fc1, fc2;
  // every layer's cross-attention K/V projection as one grouped launch, and their K norms as one
  // launch (tp 1); per-layer tensor maps and vector pointers live in the workspace ("ctx.grp")
  fw::GemmOp cakv_all;
  bool ctx_grouped = false;
  const __nv_bfloat16* const* nk_grp = nullptr;
  // the action blocks' keyboard chains as four grouped launches (pointer arrays in "act.grp")
  bool kb_grouped = false;
  const __nv_bfloat16* const* kb_grp = nullptr;
  // intermediate-tensor tap of one block (fw_set_tap; eager parity checks)
  int tap_layer = -1;
  uint8_t* tap = nullptr;
};

namespace fw {

static size_t dtype_size(int dt) { return dt == FW_BF16 ? 2 : (dt == FW_U8 ? 1 : 4); }

static void add_tensor(fw_handle* h, const std::string& name, int kind, int dtype, std::vector<int64_t> shape) {
  Tensor t;
  t.name = name;
  t.kind = kind;
  t.dtype = dtype;
  t.ndim = (int)shape.size();
  size_t n = 1;
  for (int i = 0; i < 5; ++i) t.shape[i] = i < t.ndim ? shape[i] : 0;
  for (auto v : shape) n *= (size_t)v;
  t.bytes = n * dtype_size(dtype);
  h->index[name] = (int)h->tensors.size();
  h->tensors.push_back(t);
}

static void* ptr_of(fw_handle* h, const std::string& name) {
  auto it = h->index.find(name);
  return it == h->index.end() ? nullptr : h->tensors[it->second].ptr;
}
template <typename T>
static T* P(fw_handle* h, const std::string& name) {
  return reinterpret_cast<T*>(ptr_of(h, name));
}
static const __nv_bfloat16* W(fw_handle* h, const std::string& name) { return P<const __nv_bfloat16>(h, name); }

static size_t ws_add(fw_handle* h, const char* name, size_t bytes) {
  h->ws_bytes = (h->ws_bytes + 1023) & ~(size_t)1023;
  const size_t off = h->ws_bytes;
  h->ws_off.push_back({name, off});
  h->ws_bytes += bytes;
  return off;
}

static int register_tensors(fw_handle* h) {
  const fw_config& c = h->cfg;
  const int D = h->D, A = h->A, Dl = h->Dl, FFl = h->FFl;
  auto wt = [&](const std::string& n, std::vector<int64_t> s) { add_tensor(h, n, FW_KIND_WEIGHT, FW_BF16, s); };
  wt("patch.w", {D, h->Kp});
  wt("patch.b", {D});
  wt("time.0.w", {D, c.freq_dim});
  wt("time.0.b", {D});
  wt("time.2.w", {D, D});
  wt("time.2.b", {D});
  wt("tproj.w", {6 * D, D});
  wt("tproj.b", {6 * D});
  wt("img.ln0.w", {h->Cd});
  wt("img.ln0.b", {h->Cd});
  wt("img.fc1.w", {h->Cd, h->Cd});
  wt("img.fc1.b", {h->Cd});
  wt("img.fc2.w", {D, h->Cd});
  wt("img.fc2.b", {D});
  wt("img.ln1.w", {D});
  wt("img.ln1.b", {D});
  wt("head.mod", {2, D});
  wt("head.w", {h->OUT, D});
  wt("head.b", {h->OUT});
  wt("mods", {c.layers, 6, D});
  for (int i = 0; i < c.layers; ++i) {
    const std::string p = "b" + std::to_string(i) + ".";
    // with tp > 1: q/k/v, ca.q/k/v and ffn.0 are this rank's rows (column-parallel), sa.o,
    // ca.o and ffn.2 this rank's input columns (row-parallel; their biases are whole)
    wt(p + "sa.qkv.w", {3 * Dl, D});
    wt(p + "sa.qkv.b", {3 * Dl});
    wt(p + "sa.o.w", {D, Dl});
    wt(p + "sa.o.b", {D});
    wt(p + "sa.nq.w", {Dl});
    wt(p + "sa.nk.w", {Dl});
    wt(p + "n3.w", {D});
    wt(p + "n3.b", {D});
    wt(p + "ca.q.w", {Dl, D});
    wt(p + "ca.q.b", {Dl});
    wt(p + "ca.kv.w", {2 * Dl, D});
    wt(p + "ca.kv.b", {2 * Dl});
    wt(p + "ca.o.w", {D, Dl});
    wt(p + "ca.o.b", {D});
    wt(p + "ca.nq.w", {Dl});
    wt(p + "ca.nk.w", {Dl});
    wt(p + "ffn.0.w", {FFl, D});
    wt(p + "ffn.0.b", {FFl});
    wt(p + "ffn.2.w", {D, FFl});
    wt(p + "ffn.2.b", {D});
    if (h->layers[i].act >= 0) {
      const std::string a = p + "am.";
      wt(a + "mlp1.w", {h->Mh, D + c.mouse_dim * h->PAD});
      wt(a + "mlp1.b", {h->Mh});
      wt(a + "mlp2.w", {h->Mh, h->Mh});
      wt(a + "mlp2.b", {h->Mh});
      wt(a + "mln.w", {h->Mh});
      wt(a + "mln.b", {h->Mh});
      wt(a + "tqkv.w", {3 * A, h->Mh});
      wt(a + "tqkv.b", {3 * A});
      wt(a + "mqn.w", {c.act_head_dim});
      wt(a + "mkn.w", {c.act_head_dim});
      wt(a + "pmouse.w", {D, A});
      wt(a + "pmouse.b", {D});
      wt(a + "kbe1.w", {h->Kh, c.keyboard_dim});
      wt(a + "kbe1.b", {h->Kh});
      wt(a + "kbe2.w", {h->Kh, h->Kh});
      wt(a + "kbe2.b", {h->Kh});
      wt(a + "mattq.w", {A, D});
      wt(a + "mattq.b", {A});
      wt(a + "kbkv.w", {2 * A, h->Kh * h->PAD});
      wt(a + "kbkv.b", {2 * A});
      wt(a + "kqn.w", {c.act_head_dim});
      wt(a + "kkn.w", {c.act_head_dim});
      wt(a + "pkb.w", {D, A});
      wt(a + "pkb.b", {D});
    }
  }
  if (h->fp8) {   // e4m3 copies of the block linears, derived at fw_finalize
    auto der = [&](const std::string& n, int64_t N, int64_t K) {
      add_tensor(h, n + ".q8", FW_KIND_DERIVED, FW_U8, {N, K});
      add_tensor(h, n + ".sw", FW_KIND_DERIVED, FW_F32, {N});
    };
    for (int i = 0; i < c.layers; ++i) {
      const std::string p = "b" + std::to_string(i) + ".";
      der(p + "ffn.0", FFl, D);
      der(p + "ffn.2", D, FFl);
      if (h->fp8_ffn_only) continue;
      der(p + "sa.qkv", 3 * Dl, D);
      der(p + "sa.o", D, Dl);
      der(p + "ca.q", Dl, D);
      der(p + "ca.o", D, Dl);
      if (h->layers[i].act >= 0) {
        const std::string a = p + "am.";
        der(a + "mlp1", h->Mh, D);
        der(a + "mlp2", h->Mh, h->Mh);
        der(a + "tqkv", 3 * A, h->Mh);
        der(a + "pmouse", D, A);
        der(a + "mattq", A, D);
        der(a + "pkb", D, A);
      }
    }
  }
  // session state (static.py:47-54, 280-281)
  // (history window of hc chunks: hc slots of L rows; this rank's heads)
  for (int i = 0; i < c.layers; ++i)
    add_tensor(h, "hk." + std::to_string(i), FW_KIND_STATE, FW_BF16, {1, (int64_t)h->hc * h->L, h->Hl, h->HD});
  for (int i = 0; i < c.layers; ++i)
    add_tensor(h, "hv." + std::to_string(i), FW_KIND_STATE, FW_BF16, {1, (int64_t)h->hc * h->L, h->Hl, h->HD});
  const char* an[4] = {"mk.", "mv.", "kk.", "kv."};
  for (int t = 0; t < 4; ++t)
    for (int i = 0; i < c.layers; ++i)
      if (h->layers[i].act >= 0)
        add_tensor(h, an[t] + std::to_string(i), FW_KIND_STATE, FW_BF16,
                   t < 2 ? std::vector<int64_t>{h->S, h->F, h->AH, 64} : std::vector<int64_t>{1, h->F, h->AH, 64});
  // static inputs / outputs (static.py:58-72)
  const std::vector<int64_t> lat = {1, c.lat_ch, h->F, c.lat_h, c.lat_w};
  add_tensor(h, "x_in", FW_KIND_INPUT, FW_BF16, lat);
  for (int i = 0; i + 1 < c.n_steps; ++i)
    add_tensor(h, "noise." + std::to_string(i), FW_KIND_INPUT, FW_BF16, {h->F, c.lat_ch, c.lat_h, c.lat_w});
  add_tensor(h, "cc", FW_KIND_INPUT, FW_BF16, {1, c.cond_ch, h->F, c.lat_h, c.lat_w});
  add_tensor(h, "vis", FW_KIND_INPUT, FW_BF16, {1, h->Ctx, h->Cd});
  add_tensor(h, "gm", FW_KIND_INPUT, FW_BF16, {1, h->F, h->PAD, c.mouse_dim});
  add_tensor(h, "kc", FW_KIND_INPUT, FW_BF16, {1, h->KC, c.keyboard_dim});
  add_tensor(h, "lat_in", FW_KIND_INPUT, FW_BF16, lat);
  add_tensor(h, "chunk", FW_KIND_INPUT, FW_I32, {4});
  add_tensor(h, "out", FW_KIND_OUTPUT, FW_BF16, lat);
  add_tensor(h, "status", FW_KIND_STATUS, FW_I32, {4});
  // workspace
  const int L = h->L;
  const size_t bf = 2, f4 = 4;
  auto mx = [](std::initializer_list<int> v) { int m = 0; for (int x : v) m = x > m ? x : m; return m; };
  ws_add(h, "xs", (size_t)L * D * f4);
  ws_add(h, "y", (size_t)L * mx({D, h->Mh}) * bf);
  ws_add(h, "xbf", (size_t)L * D * bf);
  ws_add(h, "q", (size_t)L * Dl * bf);
  ws_add(h, "kcur", (size_t)L * Dl * bf);
  ws_add(h, "vcur", (size_t)L * Dl * bf);
  ws_add(h, "ao", (size_t)L * mx({Dl, A}) * bf);
  ws_add(h, "hb", (size_t)L * mx({FFl, 3 * A, h->Mh}) * bf);
  ws_add(h, "hb2", (size_t)L * mx({h->Mh, A}) * bf);
  ws_add(h, "patchA", (size_t)L * h->Kp * bf);
  ws_add(h, "headout", (size_t)L * h->OUT * f4);
  ws_add(h, "xa", h->lat_elems * bf);
  ws_add(h, "xb", h->lat_elems * bf);
  ws_add(h, "den", h->lat_elems * bf);
  ws_add(h, "den_ctx", h->lat_elems * bf);
  ws_add(h, "ctx_a", (size_t)h->Ctx * h->Cd * bf);
  ws_add(h, "ctx_h", (size_t)h->Ctx * h->Cd * bf);
  ws_add(h, "ctx_o", (size_t)h->Ctx * D * bf);
  ws_add(h, "ctx", (size_t)h->Ctx * D * bf);
  ws_add(h, "ckv", (size_t)c.layers * 2 * h->Ctx * Dl * bf);
  // keyboard embedding / K-V scratch, one slice per action block (the prologue runs all blocks'
  // keyboard chains together)
  const size_t nAs = h->nA ? h->nA : 1;
  ws_add(h, "ke1", nAs * h->KC * h->Kh * f4);
  ws_add(h, "ke", nAs * h->KC * h->Kh * f4);
  ws_add(h, "kbkv", nAs * h->F * 2 * A * f4);
  ws_add(h, "act.grp", nAs * 7 * sizeof(void*));   // per action block: kbe1.w/b, kbe2.w/b, kbkv.w/b, kkn.w
  ws_add(h, "kbK", (size_t)(h->nA ? h->nA : 1) * h->F * A * bf);
  ws_add(h, "kbV", (size_t)(h->nA ? h->nA : 1) * h->F * A * bf);
  ws_add(h, "fbias", (size_t)h->F * h->Mh * f4);
  ws_add(h, "rope", (size_t)L * (h->HD / 2) * 2 * f4);
  ws_add(h, "acos", (size_t)h->F * 64 * f4);
  ws_add(h, "asin", (size_t)h->F * 64 * f4);
  ws_add(h, "tsin", (size_t)c.freq_dim * f4);
  ws_add(h, "th", (size_t)D * f4);
  ws_add(h, "e", (size_t)D * f4);
  ws_add(h, "e0", (size_t)6 * D * f4);
  ws_add(h, "ee", (size_t)c.layers * 6 * D * f4);
  ws_add(h, "hmod", (size_t)2 * D * f4);
  ws_add(h, "consts", 64 * sizeof(int));
  if (h->fp8) {
    ws_add(h, "a8", (size_t)L * mx({D, FFl, h->Mh, A}));
    ws_add(h, "sa", (size_t)L * f4);
  }
  if (h->tp > 1) {
    ws_add(h, "part", (size_t)L * D * bf);
    ws_add(h, "ss", (size_t)mx({L, h->Ctx}) * 2 * f4);
    // peer-memory reductions (tp_reduce.cu): reduced sums, flags, gathered sums of squares,
    // per-CTA call counters; other ranks address these at the same offsets of their mapping
    ws_add(h, "tp.red", (size_t)L * D * bf);
    ws_add(h, "tp.flags", (size_t)3 * TP_MAX_RANKS * TP_MAX_CTAS * sizeof(unsigned));
    ws_add(h, "tp.gat", (size_t)2 * TP_MAX_RANKS * mx({L, h->Ctx}) * 2 * f4);
    ws_add(h, "tp.epoch", (size_t)2 * TP_MAX_CTAS * sizeof(unsigned));
    // partials pushed by the other ranks' GEMMs: 2 parities x tp slots x ceil(L / tp) rows
    ws_add(h, "tp.recv", (size_t)2 * h->tp * ((L + h->tp - 1) / h->tp) * D * bf);
  }
  // per-layer tensor maps (128 B each), bias and K-norm weight pointers for the grouped
  // cross-attention K/V projection
  ws_add(h, "ctx.grp", (size_t)c.layers * (sizeof(CUtensorMap) + 2 * sizeof(void*)));
  h->ws_bytes = (h->ws_bytes + 1023) & ~(size_t)1023;
  add_tensor(h, "workspace", FW_KIND_WORKSPACE, FW_U8, {(int64_t)h->ws_bytes});
  return 0;
}

static int config_check(const fw_config& c) {
  if (c.dim <= 0 || c.heads <= 0 || c.head_dim != 128 || c.dim != c.heads * c.head_dim) return FW_ESHAPE;
  if (c.layers <= 0 || c.ffn % 64 || c.dim % 256) return FW_ESHAPE;
  if (c.frames != 3 || c.lat_h % 2 || c.lat_w % 2) return FW_ESHAPE;
  if (c.act_head_dim != 64 || c.n_action < 0 || c.n_action > FW_MAX_ACTION_BLOCKS) return FW_ESHAPE;
  if (c.n_steps < 1 || c.n_steps > FW_MAX_STEPS) return FW_EINVAL;
  if (c.freq_dim % 2 || c.ctx_dim % 128) return FW_ESHAPE;
  if (c.n_action && (c.mouse_hidden % 128 || c.keyboard_hidden <= 0 || c.mouse_dim * c.time_ratio * c.window % 8))
    return FW_ESHAPE;
  for (int i = 0; i < c.n_action; ++i)
    if (c.action_blocks[i] < 0 || c.action_blocks[i] >= c.layers) return FW_EINVAL;
  if (c.hist_chunks < 1 || c.tp_size < 1 || c.tp_rank < 0 || c.tp_rank >= c.tp_size) return FW_EINVAL;
  if (c.linear_fp8 < 0 || c.linear_fp8 > 2) return FW_EINVAL;
  if (c.tp_size > 1) {   // whole heads and 32-column FFN shards per rank; no action module
    if (c.heads % c.tp_size || c.ffn % (32 * c.tp_size) || c.n_action) return FW_ESHAPE;
  }
  return 0;
}

// CTA-pair tiles (opt-in, FW_GEMM_PAIR=1) for bf16 linears with large M and N: the 14B QKV and
// FFN-up at tensor-parallel size 1-2 (4680 x 15360 x 5120: 511 us vs 586 us in isolation); the
// MG2 shapes and N = 5120 outputs keep one-CTA tiles (fewer wave-quantisation losses).
static bool use_pair(int M, int N) { return gemm_pair_enabled() && M >= 4096 && N >= 6144; }
// A residual epilogue with no bf16 mirror becomes a TMA reduce-add into the residual.
static int resid_to_tma(GemmOp& op) {
  GemmEpi& e = op.args.epi;
  if (e.mode != EPI_RESID_F32 || e.mirror || !resid_tma_enabled()) return 0;
  int rc = make_tmap_2d(&op.c, e.resid, 4, op.args.M, op.args.N, e.ld_resid, 32, 32, true);
  if (rc) return rc;
  e.mode = EPI_RESID_TMA;
  op.has_c = true;
  return 0;
}

// ---------------------------------------------------------------- op construction
static int make_gemm(GemmOp& op, const void* A, int M, int K, int lda, const void* B, int N, int ldb, int bn,
                     const GemmEpi& epi, int* status) {
  op.pair = use_pair(M, N);
  if (op.pair) bn = 256;
  op.bn = bn;
  int rc = make_tmap_2d(&op.a, A, 2, M, K, lda, 128, 64, true);
  if (rc) return rc;
  rc = make_tmap_2d(&op.b, B, 2, N, K, ldb, op.pair ? 128 : bn, 64, true);
  if (rc) return rc;
  op.args.M = M;
  op.args.N = N;
  op.args.K = K;
  op.args.epi = epi;
  op.args.status = status;
  op.args.b_static = true;   // B is always a weight (or a derived weight) in the engine
  op.valid = true;
  rc = resid_to_tma(op);
  if (!rc && !op.pair) rc = make_out_tmaps(op.args, op.o);
  if (rc) return rc;
  return gemm_check(op.args, bn);
}
static int run(const GemmOp& op, cudaStream_t s) {
  if (op.pair) return gemm_pair_launch(op.a, op.b, op.args, s, op.has_c ? &op.c : nullptr);
  return gemm_bf16_launch(op.a, op.b, op.bn, op.args, s, 0, op.has_c ? &op.c : nullptr, op.o);
}
static int pick_bn(int N) { return N >= 256 ? 256 : (N >= 128 ? 128 : 64); }

// A block linear `wname` (weight `wname.w` [N, ldb]) whose bf16 operand is A [M, lda].  With
// e4m3 linears the GEMM instead reads the handle's e4m3 activation buffer (row stride K bytes,
// per-row scales) and the derived per-channel-quantised weight `wname.q8` / `wname.sw`.
static int make_lin(fw_handle* h, GemmOp& op, const std::string& wname, const void* A, int lda, int M, int K, int N,
                    int ldb, int bn, const GemmEpi& epi);

static GemmEpi epi_bf16(void* out, int ld, const __nv_bfloat16* bias, int mode = EPI_BF16) {
  GemmEpi e;
  e.mode = mode;
  e.out[0] = out;
  e.ld_out = ld;
  e.seg_w = 1 << 30;
  e.bias = bias;
  return e;
}
static GemmEpi epi_resid(float* xs, int ld, const __nv_bfloat16* bias, const float* gate, __nv_bfloat16* mirror) {
  GemmEpi e;
  e.mode = EPI_RESID_F32;
  e.resid = xs;
  e.ld_resid = ld;
  e.bias = bias;
  e.gate = gate;
  e.gate_stride = 0;
  e.mirror = mirror;
  e.ld_mirror = ld;
  return e;
}

static int make_attn(AttnOp& op, const void* q, int Lq, int heads, const void* k0, const void* v0, int cap0,
                     const void* k1, const void* v1, int cap1, const int* meta, void* out, int* status) {
  const int cols = heads * 128;
  int rc = make_tmap_2d(&op.q, q, 2, Lq, cols, cols, 128, 64, true);
  if (!rc) rc = make_tmap_2d(&op.k0, k0, 2, cap0, cols, cols, 128, 64, true);
  if (!rc) rc = make_tmap_2d(&op.v0, v0, 2, cap0, cols, cols, 128, 64, true);
  if (!rc) rc = make_tmap_2d(&op.k1, k1, 2, cap1, cols, cols, 128, 64, true);
  if (!rc) rc = make_tmap_2d(&op.v1, v1, 2, cap1, cols, cols, 128, 64, true);
  if (!rc) rc = make_tmap_2d(&op.o, out, 2, Lq, cols, cols, 128, 64, true);
  if (rc) return rc;
  op.args.Lq = Lq;
  op.args.heads = heads;
  op.args.meta = meta;
  op.args.max_keys0 = cap0;
  op.args.max_keys1 = cap1;
  op.args.out = reinterpret_cast<__nv_bfloat16*>(out);
  op.args.ld_out = cols;
  op.args.scale_log2 = (float)(1.4426950408889634 / std::sqrt(128.0));
  op.args.status = status;
  return 0;
}
static int run(const AttnOp& op, cudaStream_t s) {
  return attention_launch(op.q, op.k0, op.v0, op.k1, op.v1, op.args, s, &op.o);
}

// With FW_TRACE_ERRORS=1 in the environment the engine names the first failing call on stderr.
static bool trace_errors() {
  static const bool on = [] {
    const char* v = getenv("FW_TRACE_ERRORS");
    return v && v[0] == '1';
  }();
  return on;
}
#define FW_TRY(x)                                                                        \
  do {                                                                                   \
    int _rc = (x);                                                                       \
    if (_rc) {                                                                           \
      if (trace_errors()) fprintf(stderr, "fastworld_b200: %s failed (%d) at engine.cu:%d\n", #x, _rc, __LINE__); \
      return _rc;                                                                        \
    }                                                                                    \
  } while (0)

static int make_lin(fw_handle* h, GemmOp& op, const std::string& wname, const void* A, int lda, int M, int K, int N,
                    int ldb, int bn, const GemmEpi& epi) {
  if (!h->fp8 || !ptr_of(h, wname + ".q8")) return make_gemm(op, A, M, K, lda, W(h, wname + ".w"), N, ldb, bn, epi,
                                                            h->status);
  if (bn == 224) bn = 256;   // the e4m3 GEMM has no 224-wide tile
  op.bn = bn;
  FW_TRY(make_tmap_2d(&op.a, h->a8, 1, M, K, K, 128, 128, true));
  FW_TRY(make_tmap_2d(&op.b, P<uint8_t>(h, wname + ".q8"), 1, N, K, K, bn, 128, true));
  op.args.M = M;
  op.args.N = N;
  op.args.K = K;
  op.args.epi = epi;
  op.args.sa = h->sa;
  op.args.sw = P<float>(h, wname + ".sw");
  op.args.status = h->status;
  op.args.b_static = true;
  op.valid = true;
  FW_TRY(resid_to_tma(op));
  FW_TRY(make_out_tmaps(op.args, op.o));
  return gemm_check(op.args, bn);
}

// The operand of an e4m3 GEMM is quantised from `src` (bf16 [M, ld]) with per-token scales;
// in bf16 mode the GEMM reads `src` directly and this only launches the GEMM.
static int run_from(fw_handle* h, const GemmOp& op, const __nv_bfloat16* src, int ld, cudaStream_t s) {
  if (op.args.sa) FW_TRY(quant_rows(src, ld, op.args.M, op.args.K, h->a8, op.args.K, h->sa, s));
  return run(op, s);
}

// LayerNorm of the fp32 residual into the next GEMM's operand (bf16 y, or e4m3 a8 + scales).
// `consumer` is the GEMM that reads the normalised rows: e4m3 (a8 + per-row scales) when it is
// an e4m3 linear, bf16 (y) otherwise.
static int ln_op(fw_handle* h, const GemmOp& consumer, int M, int D, float eps, const float* shift,
                 const float* scale, const __nv_bfloat16* w, const __nv_bfloat16* b, cudaStream_t s) {
  if (consumer.args.sa) return ln_f32_q8(h->xs, D, M, D, eps, shift, scale, w, b, h->a8, h->sa, D, s);
  return ln_f32(h->xs, D, M, D, eps, shift, scale, w, b, h->y, D, s);
}

// q/k RMSNorm over the full hidden width (+ RoPE when `rope`) of x0 (and x1), in place; rows
// of this rank's width Dl.  With tp > 1 the per-row sums of squares of the shards are
// all-reduced first (static.py:208-209, 189-190 normalise over all heads).
static int rms_norm_op(fw_handle* h, __nv_bfloat16* x0, __nv_bfloat16* x1, const __nv_bfloat16* w0,
                       const __nv_bfloat16* w1, int M, const float2* rope, cudaStream_t s) {
  const float eps = h->cfg.eps;
  const int Dl = h->Dl;
  if (h->tp == 1) return rms_rope2(x0, w0, x0, x1, w1, x1, Dl, M, Dl, eps, rope, h->HD, Dl, s);
  FW_TRY(sumsq_rows(x0, x1, Dl, M, Dl, h->ss, s));
  if (h->use_peers)
    FW_TRY(tp_sumsq(h->peers, h->ss, M, h->status, s));
  else
    FW_TRY(tp_allreduce(h->comm, h->ss, (size_t)M * 2, FW_F32, s));
  return rms_rope2_ss(x0, w0, x0, x1, w1, x1, Dl, M, Dl, h->ss, h->D, eps, rope, h->HD, Dl, s);
}

// After a row-parallel linear with tp > 1: all-reduce the partial outputs, then
// xs += gate[frame] * (sum + bias) (the epilogue the GEMM applies itself at tp 1).  With the
// peers mapped this is one fused kernel over NVLink; otherwise NCCL + resid_add.
static int row_parallel_done(fw_handle* h, const std::string& bias, const float* gate, __nv_bfloat16* mirror,
                             int parity, cudaStream_t s) {
  if (h->tp == 1) return 0;
  if (h->push && h->tp == 2)
    return tp_combine2(h->peers, parity, h->part, h->L, h->D, W(h, bias), gate, h->xs, mirror, h->status, s);
  if (h->push)
    return tp_reduce(h->peers, h->L, h->D, W(h, bias), gate, h->xs, mirror, h->status, s,
                     h->peers.recv[h->tpr] + (size_t)parity * h->recv_stride);
  if (h->use_peers) return tp_reduce(h->peers, h->L, h->D, W(h, bias), gate, h->xs, mirror, h->status, s);
  FW_TRY(tp_allreduce(h->comm, h->part, (size_t)h->L * h->D, FW_BF16, s));
  // the adaLN gate is one row for every frame (e0 is per timestep; static.py:204, 220, 225)
  return resid_add(h->xs, h->D, h->part, h->D, W(h, bias), gate, 0, h->S, mirror, h->L, h->D, s);
}

static int finalize(fw_handle* h) {
  for (auto& t : h->tensors)
    if (!t.ptr) return FW_ENOTBOUND;
  if (!get_encode_fn()) return FW_ENODRIVER;
  uint8_t* ws = P<uint8_t>(h, "workspace");
  auto WS = [&](const char* n) -> void* {
    for (auto& p : h->ws_off)
      if (p.first == n) return ws + p.second;
    return nullptr;
  };
  h->xs = (float*)WS("xs");
  h->y = (__nv_bfloat16*)WS("y");
  h->xbf = (__nv_bfloat16*)WS("xbf");
  h->q = (__nv_bfloat16*)WS("q");
  h->kcur = (__nv_bfloat16*)WS("kcur");
  h->vcur = (__nv_bfloat16*)WS("vcur");
  h->ao = (__nv_bfloat16*)WS("ao");
  h->hb = (__nv_bfloat16*)WS("hb");
  h->hb2 = (__nv_bfloat16*)WS("hb2");
  h->patchA = (__nv_bfloat16*)WS("patchA");
  h->headout = (float*)WS("headout");
  h->xa = (__nv_bfloat16*)WS("xa");
  h->xb = (__nv_bfloat16*)WS("xb");
  h->den = (__nv_bfloat16*)WS("den");
  h->den_ctx = (__nv_bfloat16*)WS("den_ctx");
  h->ctx_a = (__nv_bfloat16*)WS("ctx_a");
  h->ctx_h = (__nv_bfloat16*)WS("ctx_h");
  h->ctx_o = (__nv_bfloat16*)WS("ctx_o");
  h->ctx = (__nv_bfloat16*)WS("ctx");
  h->ckv = (__nv_bfloat16*)WS("ckv");
  h->ke1 = (float*)WS("ke1");
  h->ke = (float*)WS("ke");
  h->kbkv = (float*)WS("kbkv");
  h->kbK = (__nv_bfloat16*)WS("kbK");
  h->kbV = (__nv_bfloat16*)WS("kbV");
  h->fbias = (float*)WS("fbias");
  h->rope = (float*)WS("rope");
  h->acos_ = (float*)WS("acos");
  h->asin_ = (float*)WS("asin");
  h->tsin = (float*)WS("tsin");
  h->th_ = (float*)WS("th");
  h->e = (float*)WS("e");
  h->e0 = (float*)WS("e0");
  h->ee = (float*)WS("ee");
  h->hmod = (float*)WS("hmod");
  h->consts = (int*)WS("consts");
  h->a8 = (uint8_t*)WS("a8");
  h->sa = (float*)WS("sa");
  h->part = (__nv_bfloat16*)WS("part");
  h->ss = (float*)WS("ss");
  h->status = P<int>(h, "status");
  // device tables: attention segment lengths {first, steady, cross, steady with a history
  // window of several chunks (rewritten per chunk by hist_meta)}
  int consts[8] = {0, h->L, h->L, h->L, h->Ctx, 0, 0, h->L};
  if (cudaMemcpy(h->consts, consts, sizeof(consts), cudaMemcpyHostToDevice) != cudaSuccess) return FW_ECUDA;
  const int L = h->L, D = h->D, Ctx = h->Ctx, Dl = h->Dl, Hl = h->Hl;
  const bool tp = h->tp > 1;
  const int bnl = Dl % 256 ? 128 : 256;   // column tile that divides this rank's head width
  int* st = h->status;
  // patch embedding and head
  FW_TRY(make_gemm(h->patch, h->patchA, L, h->Kp, h->Kp, W(h, "patch.w"), D, h->Kp, pick_bn(D),
                   [&] { GemmEpi e = epi_bf16(h->xs, D, W(h, "patch.b"), EPI_F32); return e; }(), st));
  FW_TRY(make_gemm(h->head, h->y, L, D, D, W(h, "head.w"), h->OUT, D, pick_bn(h->OUT),
                   epi_bf16(h->headout, h->OUT, W(h, "head.b"), EPI_F32), st));
  // image-context MLP (M = Ctx)
  FW_TRY(make_gemm(h->fc1, h->ctx_a, Ctx, h->Cd, h->Cd, W(h, "img.fc1.w"), h->Cd, h->Cd, 128,
                   epi_bf16(h->ctx_h, h->Cd, W(h, "img.fc1.b"), EPI_GELU_ERF_BF16), st));
  FW_TRY(make_gemm(h->fc2, h->ctx_h, Ctx, h->Cd, h->Cd, W(h, "img.fc2.w"), D, h->Cd, 128,
                   epi_bf16(h->ctx_o, D, W(h, "img.fc2.b")), st));
  for (int i = 0; i < h->cfg.layers; ++i) {
    Layer& ly = h->layers[i];
    const std::string p = "b" + std::to_string(i) + ".";
    const float* ee = h->ee + (size_t)i * 6 * D;
    {
      GemmEpi e = epi_bf16(h->q, Dl, W(h, p + "sa.qkv.b"));
      e.out[1] = h->kcur;
      e.out[2] = h->vcur;
      e.seg_w = Dl;
      FW_TRY(make_lin(h, ly.qkv, p + "sa.qkv", h->y, D, L, D, 3 * Dl, D, bnl, e));
    }
    // row-parallel linears: with tp > 1 the GEMM writes this rank's partial sum (no bias);
    // the all-reduce and resid_add apply the bias and the gated residual once
    auto row_par = [&](const char* name, const float* gate, __nv_bfloat16* mirror) {
      return tp ? epi_bf16(h->part, D, nullptr) : epi_resid(h->xs, D, W(h, p + name + ".b"), gate, mirror);
    };
    // the gated-residual linears take 224-wide tiles where that fills the SMs better (bf16 only;
    // the tensor-parallel partial-sum epilogue and the e4m3 linears keep 256)
    const int bnr = tp ? 256 : gemm_resid_bn(L, D);
    FW_TRY(make_lin(h, ly.o, p + "sa.o", h->ao, Dl, L, Dl, D, Dl, bnr, row_par("sa.o", ee + 2 * D, nullptr)));
    FW_TRY(make_lin(h, ly.caq, p + "ca.q", h->y, D, L, D, Dl, D, bnl, epi_bf16(h->q, Dl, W(h, p + "ca.q.b"))));
    {
      __nv_bfloat16* ck = h->ckv + (size_t)i * 2 * Ctx * Dl;
      GemmEpi e = epi_bf16(ck, Dl, W(h, p + "ca.kv.b"));
      e.out[1] = ck + (size_t)Ctx * Dl;
      e.seg_w = Dl;
      FW_TRY(make_gemm(ly.cakv, h->ctx, Ctx, D, D, W(h, p + "ca.kv.w"), 2 * Dl, D, bnl, e, st));
    }
    FW_TRY(make_lin(h, ly.cao, p + "ca.o", h->ao, Dl, L, Dl, D, Dl, bnr,
                    row_par("ca.o", nullptr, ly.act >= 0 ? h->xbf : nullptr)));
    FW_TRY(make_lin(h, ly.ff0, p + "ffn.0", h->y, D, L, D, h->FFl, D, 256,
                    epi_bf16(h->hb, h->FFl, W(h, p + "ffn.0.b"), EPI_GELU_BF16)));
    FW_TRY(make_lin(h, ly.ff2, p + "ffn.2", h->hb, h->FFl, L, h->FFl, D, h->FFl, bnr,
                    row_par("ffn.2", ee + 5 * D, nullptr)));
    const void* hk = ptr_of(h, "hk." + std::to_string(i));
    const void* hv = ptr_of(h, "hv." + std::to_string(i));
    const int cap = h->hc * L;
    FW_TRY(make_attn(ly.self_first, h->q, L, Hl, hk, hv, cap, h->kcur, h->vcur, L, h->consts + 0, h->ao, st));
    FW_TRY(make_attn(ly.self_steady, h->q, L, Hl, hk, hv, cap, h->kcur, h->vcur, L,
                     h->consts + (h->hc > 1 ? 6 : 2), h->ao, st));
    {
      const __nv_bfloat16* ck = h->ckv + (size_t)i * 2 * Ctx * Dl;
      FW_TRY(make_attn(ly.cross, h->q, L, Hl, ck, ck + (size_t)Ctx * Dl, Ctx, ck, ck + (size_t)Ctx * Dl, Ctx,
                       h->consts + 4, h->ao, st));
    }
    if (ly.act >= 0) {
      const std::string a = p + "am.";
      const int A = h->A, Mh = h->Mh, K1 = D + h->cfg.mouse_dim * h->PAD;
      GemmEpi e1 = epi_bf16(h->hb, Mh, nullptr, EPI_GELU_BF16);
      e1.bias = nullptr;
      e1.fbias = h->fbias;
      e1.fbias_stride = Mh;
      e1.rows_per_frame = h->S;
      FW_TRY(make_lin(h, ly.mlp1, a + "mlp1", h->xbf, D, L, D, Mh, K1, pick_bn(Mh), e1));
      FW_TRY(make_lin(h, ly.mlp2, a + "mlp2", h->hb, Mh, L, Mh, Mh, Mh, pick_bn(Mh),
                      epi_bf16(h->hb2, Mh, W(h, a + "mlp2.b"))));
      FW_TRY(make_lin(h, ly.tqkv, a + "tqkv", h->y, Mh, L, Mh, 3 * A, Mh, pick_bn(3 * A),
                      epi_bf16(h->hb, 3 * A, W(h, a + "tqkv.b"))));
      FW_TRY(make_lin(h, ly.pmouse, a + "pmouse", h->ao, A, L, A, D, A, 256,
                      epi_resid(h->xs, D, W(h, a + "pmouse.b"), nullptr, h->xbf)));
      FW_TRY(make_lin(h, ly.mattq, a + "mattq", h->xbf, D, L, D, A, D, pick_bn(A),
                      epi_bf16(h->hb2, A, W(h, a + "mattq.b"))));
      FW_TRY(make_lin(h, ly.pkb, a + "pkb", h->ao, A, L, A, D, A, 256,
                      epi_resid(h->xs, D, W(h, a + "pkb.b"), nullptr, nullptr)));
    }
  }
  if (h->fp8) {   // derive the per-output-channel e4m3 weights of every block linear
    for (auto& t : h->tensors) {
      if (t.kind != FW_KIND_DERIVED || t.name.size() < 3 || t.name.compare(t.name.size() - 3, 3, ".q8")) continue;
      const std::string base = t.name.substr(0, t.name.size() - 3);
      const int idx = h->index[base + ".w"];
      const Tensor& w = h->tensors[idx];
      const int N = (int)t.shape[0], K = (int)t.shape[1];
      FW_TRY(quant_rows(reinterpret_cast<const __nv_bfloat16*>(w.ptr), (int)w.shape[1], N, K,
                        reinterpret_cast<uint8_t*>(t.ptr), K, P<float>(h, base + ".sw"), 0));
    }
    if (cudaDeviceSynchronize() != cudaSuccess) return FW_ECUDA;
  }
  if (!tp) {   // the grouped cross-attention K/V projection (all layers in one launch)
    const int nl = h->cfg.layers;
    std::vector<CUtensorMap> maps(nl);
    std::vector<const void*> ptrs(2 * (size_t)nl);
    bool ok = true;
    for (int i = 0; i < nl; ++i) {
      const GemmOp& op = h->layers[i].cakv;
      ok = ok && !op.pair && op.bn == h->layers[0].cakv.bn;
      maps[i] = op.b;
      ptrs[i] = op.args.epi.bias;
      ptrs[nl + i] = W(h, "b" + std::to_string(i) + ".ca.nk.w");
    }
    if (ok) {
      uint8_t* g = reinterpret_cast<uint8_t*>(WS("ctx.grp"));
      if (cudaMemcpy(g, maps.data(), sizeof(CUtensorMap) * nl, cudaMemcpyHostToDevice) != cudaSuccess ||
          cudaMemcpy(g + sizeof(CUtensorMap) * nl, ptrs.data(), sizeof(void*) * 2 * nl, cudaMemcpyHostToDevice) !=
              cudaSuccess)
        return FW_ECUDA;
      h->cakv_all = h->layers[0].cakv;
      GemmArgs& a = h->cakv_all.args;
      a.groups = nl;
      a.epi.tma_store = false;   // grouped outputs are written by st.global (one tensor map per layer otherwise)
      a.tmB_grp = reinterpret_cast<const CUtensorMap*>(g);
      a.bias_grp = reinterpret_cast<const __nv_bfloat16* const*>(g + sizeof(CUtensorMap) * nl);
      a.out_grp_stride = (long long)2 * Ctx * Dl;
      h->nk_grp = reinterpret_cast<const __nv_bfloat16* const*>(g + sizeof(CUtensorMap) * nl + sizeof(void*) * nl);
      FW_TRY(gemm_check(a, h->cakv_all.bn));
      h->ctx_grouped = true;
    }
  }
  if (h->nA > 0) {   // keyboard chains of every action block, in action-block order
    std::vector<const void*> ptrs(7 * (size_t)h->nA, nullptr);
    bool aligned = true;
    for (int i = 0; i < h->cfg.layers; ++i) {
      const int a = h->layers[i].act;
      if (a < 0) continue;
      const std::string p = "b" + std::to_string(i) + ".am.";
      const char* names[7] = {"kbe1.w", "kbe1.b", "kbe2.w", "kbe2.b", "kbkv.w", "kbkv.b", "kkn.w"};
      for (int k = 0; k < 7; ++k) {
        ptrs[(size_t)k * h->nA + a] = W(h, p + names[k]);
        if (k == 2 || k == 4) aligned = aligned && (reinterpret_cast<uintptr_t>(ptrs[(size_t)k * h->nA + a]) & 15u) == 0;
      }
    }
    void* g = WS("act.grp");
    if (cudaMemcpy(g, ptrs.data(), ptrs.size() * sizeof(void*), cudaMemcpyHostToDevice) != cudaSuccess)
      return FW_ECUDA;
    h->kb_grp = reinterpret_cast<const __nv_bfloat16* const*>(g);
    h->kb_grouped = aligned;
  }
  h->finalized = true;
  return 0;
}

// ---------------------------------------------------------------- launch sequence
// Per-chunk prologue: RoPE tables, image context + cross K/V, keyboard K/V.
static int prologue(fw_handle* h, cudaStream_t s) {
  const fw_config& c = h->cfg;
  const int D = h->D, Ctx = h->Ctx;
  FW_TRY(rope_tables(P<int>(h, "chunk"), h->F, h->th, h->tw, h->HD, (double)c.rope_theta,
                     reinterpret_cast<float2*>(h->rope), 64, h->acos_, h->asin_, s));
  FW_TRY(ln_bf16(P<__nv_bfloat16>(h, "vis"), h->Cd, Ctx, h->Cd, c.eps_ln, nullptr, nullptr, W(h, "img.ln0.w"),
                 W(h, "img.ln0.b"), h->ctx_a, h->Cd, s));
  FW_TRY(run(h->fc1, s));
  FW_TRY(run(h->fc2, s));
  FW_TRY(ln_bf16(h->ctx_o, D, Ctx, D, c.eps_ln, nullptr, nullptr, W(h, "img.ln1.w"), W(h, "img.ln1.b"), h->ctx, D, s));
  const int Dl = h->Dl;
  if (h->hc > 1) FW_TRY(hist_meta(P<int>(h, "chunk"), h->hc, h->L, h->consts + 6, s));
  if (h->ctx_grouped) {   // all layers' K/V projections, then all their K norms: two launches
    FW_TRY(run(h->cakv_all, s));
    FW_TRY(rms_grp(h->ckv, (long long)2 * Ctx * Dl, c.layers, h->nk_grp, Dl, Ctx, Dl, c.eps, s));
  } else {
    for (int i = 0; i < c.layers; ++i) {
      const std::string p = "b" + std::to_string(i) + ".";
      __nv_bfloat16* ck = h->ckv + (size_t)i * 2 * Ctx * Dl;
      FW_TRY(run(h->layers[i].cakv, s));
      FW_TRY(rms_norm_op(h, ck, nullptr, W(h, p + "ca.nk.w"), nullptr, Ctx, nullptr, s));
    }
  }
  if (h->kb_grouped) {   // every action block's keyboard chain in four launches (blockIdx.y = block)
    const int A = h->A, Kh = h->Kh, nA = h->nA;
    const __nv_bfloat16* const* g = h->kb_grp;   // device array: offsets only on the host
    SmallmGrp g1{g + 0 * nA, g + 1 * nA, 0, (long long)h->KC * Kh, nA, true};
    SmallmGrp g2{g + 2 * nA, g + 3 * nA, (long long)h->KC * Kh, (long long)h->KC * Kh, nA, true};
    SmallmGrp g3{g + 4 * nA, g + 5 * nA, (long long)h->KC * Kh, (long long)h->F * 2 * A, nA, true};
    FW_TRY(smallm_linear_bf16(P<__nv_bfloat16>(h, "kc"), c.keyboard_dim, h->KC, nullptr, c.keyboard_dim, nullptr, Kh,
                              c.keyboard_dim, ACT_NONE, ACT_SILU, h->ke1, nullptr, Kh, s, &g1));
    FW_TRY(smallm_linear_f32(h->ke1, Kh, h->KC, nullptr, Kh, nullptr, Kh, Kh, ACT_NONE, ACT_NONE, h->ke, nullptr, Kh,
                             s, &g2));
    FW_TRY(smallm_linear_f32(h->ke, c.time_ratio * Kh, h->F, nullptr, Kh * h->PAD, nullptr, 2 * A, Kh * h->PAD,
                             ACT_NONE, ACT_NONE, h->kbkv, nullptr, 2 * A, s, &g3));
    return kb_kv_grp(h->kbkv, g + 6 * nA, nA, h->acos_, h->asin_, h->kbK, h->kbV, h->F, h->AH, c.eps, s);
  }
  for (int i = 0; i < c.layers; ++i) {
    const Layer& ly = h->layers[i];
    if (ly.act < 0) continue;
    const std::string a = "b" + std::to_string(i) + ".am.";
    const int A = h->A, Kh = h->Kh;
    FW_TRY(smallm_linear_bf16(P<__nv_bfloat16>(h, "kc"), c.keyboard_dim, h->KC, W(h, a + "kbe1.w"), c.keyboard_dim,
                              W(h, a + "kbe1.b"), Kh, c.keyboard_dim, ACT_NONE, ACT_SILU, h->ke1, nullptr, Kh, s));
    FW_TRY(smallm_linear_f32(h->ke1, Kh, h->KC, W(h, a + "kbe2.w"), Kh, W(h, a + "kbe2.b"), Kh, Kh, ACT_NONE, ACT_NONE,
                             h->ke, nullptr, Kh, s));
    // window of frame f = pixel-frame rows [ratio * f, ratio * f + pad_t) of the embedded keys
    FW_TRY(smallm_linear_f32(h->ke, c.time_ratio * Kh, h->F, W(h, a + "kbkv.w"), Kh * h->PAD, W(h, a + "kbkv.b"),
                             2 * A, Kh * h->PAD, ACT_NONE, ACT_NONE, h->kbkv, nullptr, 2 * A, s));
    FW_TRY(kb_kv(h->kbkv, W(h, a + "kkn.w"), h->acos_, h->asin_, h->kbK + (size_t)ly.act * h->F * A,
                 h->kbV + (size_t)ly.act * h->F * A, h->F, h->AH, c.eps, s));
  }
  return 0;
}

static int action(fw_handle* h, int i, int first, int write, cudaStream_t s) {
  const fw_config& c = h->cfg;
  const Layer& ly = h->layers[i];
  const std::string a = "b" + std::to_string(i) + ".am.";
  const std::string si = std::to_string(i);
  const int D = h->D, A = h->A, Mh = h->Mh, K1 = D + c.mouse_dim * h->PAD;
  // mouse window contribution of mouse_mlp[0], one row per frame: b + gm_f . W[:, D:]
  FW_TRY(smallm_linear_bf16(P<__nv_bfloat16>(h, "gm"), c.mouse_dim * h->PAD, h->F, W(h, a + "mlp1.w") + D, K1,
                            W(h, a + "mlp1.b"), Mh, c.mouse_dim * h->PAD, ACT_NONE, ACT_NONE, h->fbias, nullptr, Mh, s));
  FW_TRY(run_from(h, ly.mlp1, h->xbf, D, s));
  FW_TRY(run_from(h, ly.mlp2, h->hb, Mh, s));
  if (ly.tqkv.args.sa)
    FW_TRY(ln_bf16_q8(h->hb2, Mh, h->L, Mh, c.eps_ln, nullptr, nullptr, W(h, a + "mln.w"), W(h, a + "mln.b"), h->a8,
                      h->sa, Mh, s));
  else
    FW_TRY(ln_bf16(h->hb2, Mh, h->L, Mh, c.eps_ln, nullptr, nullptr, W(h, a + "mln.w"), W(h, a + "mln.b"), h->y, Mh,
                   s));
  FW_TRY(run(ly.tqkv, s));
  FW_TRY(mouse_attn(h->hb, W(h, a + "mqn.w"), W(h, a + "mkn.w"), h->acos_, h->asin_, P<__nv_bfloat16>(h, "mk." + si),
                    P<__nv_bfloat16>(h, "mv." + si), first, write, h->ao, h->S, h->F, h->AH, c.eps, s));
  FW_TRY(run_from(h, ly.pmouse, h->ao, A, s));
  FW_TRY(run_from(h, ly.mattq, h->xbf, D, s));
  const __nv_bfloat16* kc = h->kbK + (size_t)ly.act * h->F * A;
  const __nv_bfloat16* vc = h->kbV + (size_t)ly.act * h->F * A;
  FW_TRY(kb_attn(h->hb2, W(h, a + "kqn.w"), h->acos_, h->asin_, P<__nv_bfloat16>(h, "kk." + si),
                 P<__nv_bfloat16>(h, "kv." + si), kc, vc, first, h->ao, h->L, h->S, h->F, h->AH, c.eps, s));
  if (write) {
    FW_TRY(copy_bytes(ptr_of(h, "kk." + si), kc, (size_t)h->F * A * 2, s));
    FW_TRY(copy_bytes(ptr_of(h, "kv." + si), vc, (size_t)h->F * A * 2, s));
  }
  FW_TRY(run_from(h, ly.pkb, h->ao, A, s));
  return 0;
}

// One `_net` (static.py:194-230) from latent `x` at timestep index `step`; writes den and,
// when `noise`, the next latent xnext = add_noise(den).
static int forward(fw_handle* h, int step, int first, int write, const __nv_bfloat16* x, __nv_bfloat16* den,
                   __nv_bfloat16* out_copy, const __nv_bfloat16* noise, float t_next, __nv_bfloat16* xnext,
                   cudaStream_t s) {
  const fw_config& c = h->cfg;
  const int L = h->L, D = h->D;
  const float t = step < c.n_steps ? c.steps[step] : 0.f;
  const int ti = (int)t;   // the forward uses int(t) (static.py:39-40)
  // time embedding and per-block adaLN tables
  FW_TRY(sinusoid((double)ti, c.freq_dim, h->tsin, s));
  FW_TRY(smallm_linear_f32(h->tsin, c.freq_dim, 1, W(h, "time.0.w"), c.freq_dim, W(h, "time.0.b"), D, c.freq_dim,
                           ACT_NONE, ACT_SILU, h->th_, nullptr, D, s));
  FW_TRY(smallm_linear_f32(h->th_, D, 1, W(h, "time.2.w"), D, W(h, "time.2.b"), D, D, ACT_NONE, ACT_NONE, h->e,
                           nullptr, D, s));
  FW_TRY(smallm_linear_f32(h->e, D, 1, W(h, "tproj.w"), D, W(h, "tproj.b"), 6 * D, D, ACT_SILU, ACT_NONE, h->e0,
                           nullptr, 6 * D, s));
  FW_TRY(modulation(W(h, "mods"), h->e0, c.layers, D, h->ee, W(h, "head.mod"), h->e, h->hmod, s));
  // patch embedding of cat([x, cc])
  FW_TRY(patchify(x, c.lat_ch, P<__nv_bfloat16>(h, "cc"), c.cond_ch, h->F, c.lat_h, c.lat_w, h->patchA, s));
  FW_TRY(run(h->patch, s));
  const float2* rope = reinterpret_cast<const float2*>(h->rope);
  for (int i = 0; i < c.layers; ++i) {
    const Layer& ly = h->layers[i];
    const std::string p = "b" + std::to_string(i) + ".";
    const float* ee = h->ee + (size_t)i * 6 * D;
    const int Dl = h->Dl;
    // tap slots: fp32 residual [L, D] at TAP_XS_IN..TAP_XS_OUT, then bf16 [L, Dl] q, k, v, attention
    const bool tap = h->tap && h->tap_layer == i;
    const size_t xs_b = (size_t)L * D * 4, qb = (size_t)L * Dl * 2;
    auto tap_xs = [&](int slot) { return tap ? copy_bytes(h->tap + slot * xs_b, h->xs, xs_b, s) : 0; };
    auto tap_bf = [&](int slot, const void* src) {
      return tap ? copy_bytes(h->tap + 5 * xs_b + slot * qb, src, qb, s) : 0;
    };
    FW_TRY(tap_xs(0));
    FW_TRY(ln_op(h, ly.qkv, L, D, c.eps, ee + 0 * D, ee + 1 * D, nullptr, nullptr, s));
    FW_TRY(run(ly.qkv, s));
    FW_TRY(rms_norm_op(h, h->q, h->kcur, W(h, p + "sa.nq.w"), W(h, p + "sa.nk.w"), L, rope, s));
    FW_TRY(tap_bf(0, h->q));
    FW_TRY(tap_bf(1, h->kcur));
    FW_TRY(tap_bf(2, h->vcur));
    FW_TRY(run(first ? ly.self_first : ly.self_steady, s));
    FW_TRY(tap_bf(3, h->ao));
    if (write) {   // the history is written after the attention read it (static.py:217-218)
      const size_t bytes = (size_t)L * Dl * 2;
      void* hk = ptr_of(h, "hk." + std::to_string(i));
      void* hv = ptr_of(h, "hv." + std::to_string(i));
      if (h->hc == 1) {
        FW_TRY(copy_bytes(hk, h->kcur, bytes, s));
        FW_TRY(copy_bytes(hv, h->vcur, bytes, s));
      } else {   // slot k % window of the history ring
        FW_TRY(slot_copy(hk, bytes, P<int>(h, "chunk"), h->hc, h->kcur, bytes, s));
        FW_TRY(slot_copy(hv, bytes, P<int>(h, "chunk"), h->hc, h->vcur, bytes, s));
      }
    }
    FW_TRY(run_from(h, ly.o, h->ao, Dl, s));
    FW_TRY(row_parallel_done(h, p + "sa.o.b", ee + 2 * D, nullptr, (3 * i) & 1, s));
    FW_TRY(tap_xs(1));
    FW_TRY(ln_op(h, ly.caq, L, D, c.eps, nullptr, nullptr, W(h, p + "n3.w"), W(h, p + "n3.b"), s));
    FW_TRY(run(ly.caq, s));
    FW_TRY(rms_norm_op(h, h->q, nullptr, W(h, p + "ca.nq.w"), nullptr, L, nullptr, s));
    FW_TRY(run(ly.cross, s));
    FW_TRY(run_from(h, ly.cao, h->ao, Dl, s));
    FW_TRY(row_parallel_done(h, p + "ca.o.b", nullptr, nullptr, (3 * i + 1) & 1, s));
    FW_TRY(tap_xs(2));
    if (ly.act >= 0) FW_TRY(action(h, i, first, write, s));
    FW_TRY(tap_xs(3));
    FW_TRY(ln_op(h, ly.ff0, L, D, c.eps, ee + 3 * D, ee + 4 * D, nullptr, nullptr, s));
    FW_TRY(run(ly.ff0, s));
    FW_TRY(run_from(h, ly.ff2, h->hb, h->FFl, s));
    FW_TRY(row_parallel_done(h, p + "ffn.2.b", ee + 5 * D, nullptr, (3 * i + 2) & 1, s));
    FW_TRY(tap_xs(4));
  }
  FW_TRY(ln_f32(h->xs, D, L, D, c.eps, h->hmod, h->hmod + D, nullptr, nullptr, h->y, D, s));
  FW_TRY(run(h->head, s));
  return scheduler(h->headout, x, (float)ti / 1000.f, den, out_copy, noise, t_next / 1000.f, xnext, c.lat_ch, h->F,
                   c.lat_h, c.lat_w, s);
}

static int chunk(fw_handle* h, int first, cudaStream_t s) {
  const fw_config& c = h->cfg;
  FW_TRY(prologue(h, s));
  const __nv_bfloat16* x = P<__nv_bfloat16>(h, "x_in");
  __nv_bfloat16* bufs[2] = {h->xa, h->xb};
  const int n = c.n_steps;
  for (int i = 0; i < n; ++i) {
    const bool last = i == n - 1;
    __nv_bfloat16* xn = last ? nullptr : bufs[i & 1];
    const __nv_bfloat16* nz = last ? nullptr : P<__nv_bfloat16>(h, "noise." + std::to_string(i));
    FW_TRY(forward(h, i, first, 0, x, h->den, last ? P<__nv_bfloat16>(h, "out") : nullptr, nz,
                   last ? 0.f : c.steps[i + 1], xn, s));
    x = xn;
  }
  // context forward at t = 0 on the final denoised latent; writes the history
  return forward(h, n, first, 1, h->den, h->den_ctx, nullptr, nullptr, 0.f, nullptr, s);
}

}  // namespace fw

// ==================================================================== C ABI
extern "C" {

int fw_abi_version(void) { return FW_ABI_VERSION; }

const char* fw_strerror(int code) {
  switch (code) {
    case FW_OK: return "ok";
    case FW_EINVAL: return "invalid argument";
    case FW_ESHAPE: return "unsupported or inconsistent shape";
    case FW_EALIGN: return "pointer or stride not 16-byte aligned";
    case FW_ECUDA: return "CUDA runtime error";
    case FW_ENOTBOUND: return "a required tensor is not bound";
    case FW_ENODRIVER: return "cuTensorMapEncodeTiled unavailable (driver entry point)";
    case FW_ESTATE: return "call out of order (finalize first / already finalized)";
    case FW_ESIZE: return "bound buffer smaller than required";
    case FW_ESCRATCH: return "problem exceeds the fixed scratch of fw_linear_e4m3_noalloc (M*K <= 32 MiB, M <= 16384)";
    case FW_ENCCL: return "NCCL unavailable (libnccl.so.2) or an NCCL call failed";
    default: return "unknown error";
  }
}

int fw_create(const fw_config* cfg, fw_handle** out) {
  if (!cfg || !out) return FW_EINVAL;
  int rc = fw::config_check(*cfg);
  if (rc) return rc;
  fw_handle* h = new fw_handle();
  h->cfg = *cfg;
  const fw_config& c = *cfg;
  h->F = c.frames;
  h->th = c.lat_h / 2;
  h->tw = c.lat_w / 2;
  h->S = h->th * h->tw;
  h->L = h->F * h->S;
  h->D = c.dim;
  h->H = c.heads;
  h->HD = c.head_dim;
  h->FF = c.ffn;
  h->AH = c.act_heads;
  h->A = c.act_heads * c.act_head_dim;
  h->Mh = c.mouse_hidden;
  h->Kh = c.keyboard_hidden;
  h->nA = c.n_action;
  h->Ctx = c.ctx_tokens;
  h->Cd = c.ctx_dim;
  h->Kp = (c.lat_ch + c.cond_ch) * 4;
  h->OUT = c.lat_ch * 4;
  h->PAD = c.time_ratio * c.window;
  h->KC = c.frames * c.time_ratio + h->PAD - 3;
  h->lat_elems = (size_t)c.lat_ch * c.frames * c.lat_h * c.lat_w;
  h->fp8 = c.linear_fp8 != 0;
  h->fp8_ffn_only = c.linear_fp8 == 2;
  h->tp = c.tp_size;
  h->tpr = c.tp_rank;
  h->hc = c.hist_chunks;
  h->Hl = c.heads / c.tp_size;
  h->Dl = h->Hl * c.head_dim;
  h->FFl = c.ffn / c.tp_size;
  h->layers.resize(c.layers);
  for (int j = 0; j < c.n_action; ++j) h->layers[c.action_blocks[j]].act = j;
  fw::register_tensors(h);
  *out = h;
  return 0;
}

int fw_tensor_count(const fw_handle* h) { return h ? (int)h->tensors.size() : FW_EINVAL; }

int fw_tensor_info_at(const fw_handle* h, int i, fw_tensor_info* info) {
  if (!h || !info || i < 0 || i >= (int)h->tensors.size()) return FW_EINVAL;
  const fw::Tensor& t = h->tensors[i];
  info->name = t.name.c_str();
  info->kind = t.kind;
  info->dtype = t.dtype;
  info->ndim = t.ndim;
  for (int k = 0; k < 5; ++k) info->shape[k] = t.shape[k];
  info->bytes = t.bytes;
  return 0;
}

int fw_bind(fw_handle* h, const char* name, void* ptr, size_t bytes) {
  if (!h || !name || !ptr) return FW_EINVAL;
  if (h->finalized) return FW_ESTATE;
  auto it = h->index.find(name);
  if (it == h->index.end()) return FW_EINVAL;
  fw::Tensor& t = h->tensors[it->second];
  if (bytes < t.bytes) return FW_ESIZE;
  if (reinterpret_cast<uintptr_t>(ptr) & 15u) return FW_EALIGN;
  t.ptr = ptr;
  return 0;
}

int fw_finalize(fw_handle* h) {
  if (!h) return FW_EINVAL;
  if (h->finalized) return FW_ESTATE;
  return fw::finalize(h);
}

int fw_chunk(fw_handle* h, int first, void* stream) {
  if (!h) return FW_EINVAL;
  if (!h->finalized || (h->tp > 1 && !h->comm && !h->use_peers)) return FW_ESTATE;
  return fw::chunk(h, first, reinterpret_cast<cudaStream_t>(stream));
}

int fw_prefill(fw_handle* h, int first, void* stream) {
  if (!h) return FW_EINVAL;
  if (!h->finalized || (h->tp > 1 && !h->comm && !h->use_peers)) return FW_ESTATE;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  int rc = fw::prologue(h, s);
  if (rc) return rc;
  return fw::forward(h, h->cfg.n_steps, first, 1, fw::P<__nv_bfloat16>(h, "lat_in"), h->den_ctx, nullptr, nullptr,
                     0.f, nullptr, s);
}

int fw_forward(fw_handle* h, int step, int first, int write, void* stream) {
  if (!h) return FW_EINVAL;
  if (!h->finalized || (h->tp > 1 && !h->comm && !h->use_peers)) return FW_ESTATE;
  if (step < 0 || step > h->cfg.n_steps) return FW_EINVAL;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  int rc = fw::prologue(h, s);
  if (rc) return rc;
  // one forward from x_in (or lat_in for the context step) into out
  const __nv_bfloat16* x = fw::P<__nv_bfloat16>(h, step < h->cfg.n_steps ? "x_in" : "lat_in");
  return fw::forward(h, step, first, write, x, h->den, fw::P<__nv_bfloat16>(h, "out"), nullptr, 0.f, nullptr, s);
}

int fw_prep(fw_handle* h, const fw_prep_args* args, void* stream) {
  if (!h || !args) return FW_EINVAL;
  if (!h->finalized) return FW_ESTATE;
  const int n = h->cfg.n_steps;   // x_in + (n_steps - 1) renoising tensors
  __nv_bfloat16* dst[FW_MAX_STEPS];
  dst[0] = fw::P<__nv_bfloat16>(h, "x_in");
  for (int i = 1; i < n; ++i) dst[i] = fw::P<__nv_bfloat16>(h, "noise." + std::to_string(i - 1));
  return fw::prep_launch(h->cfg, *args, fw::P<int>(h, "chunk"), fw::P<__nv_bfloat16>(h, "kc"),
                         fw::P<__nv_bfloat16>(h, "gm"), fw::P<__nv_bfloat16>(h, "cc"), dst, n, h->status,
                         reinterpret_cast<cudaStream_t>(stream));
}

size_t fw_tap_bytes(const fw_handle* h) {
  if (!h) return 0;
  return 5 * (size_t)h->L * h->D * 4 + 4 * (size_t)h->L * h->Dl * 2;
}

int fw_set_tap(fw_handle* h, int layer, void* buf, size_t bytes) {
  if (!h) return FW_EINVAL;
  if (!buf || layer < 0) {
    h->tap = nullptr;
    h->tap_layer = -1;
    return 0;
  }
  if (layer >= h->cfg.layers) return FW_EINVAL;
  if (bytes < fw_tap_bytes(h)) return FW_ESIZE;
  if (reinterpret_cast<uintptr_t>(buf) & 15u) return FW_EALIGN;
  h->tap = static_cast<uint8_t*>(buf);
  h->tap_layer = layer;
  return 0;
}

void fw_destroy(fw_handle* h) {
  if (!h) return;
  fw::tp_comm_destroy(h->comm);
  delete h;
}

int fw_tp_unique_id(void* id128) { return fw::tp_unique_id(id128); }

int fw_tp_init(fw_handle* h, const void* id128) {
  if (!h || !id128) return FW_EINVAL;
  if (h->tp == 1 || h->comm) return FW_ESTATE;
  return fw::tp_comm_init(&h->comm, id128, h->tpr, h->tp);
}

int fw_tp_peers(fw_handle* h, void* const* ws_bases, int n) {
  if (!h || !ws_bases) return FW_EINVAL;
  if (h->tp == 1 || !h->finalized) return FW_ESTATE;
  if (n != h->tp || n > fw::TP_MAX_RANKS) return FW_EINVAL;
  const uint8_t* own = fw::P<uint8_t>(h, "workspace");
  if (ws_bases[h->tpr] != own) return FW_EINVAL;
  auto off = [&](const char* name) -> size_t {
    for (auto& p : h->ws_off)
      if (p.first == name) return p.second;
    return (size_t)-1;
  };
  fw::TpPeers& P = h->peers;
  P.tp = h->tp;
  P.rank = h->tpr;
  P.gat_rows = h->L > h->Ctx ? h->L : h->Ctx;
  for (int j = 0; j < n; ++j) {
    uint8_t* b = reinterpret_cast<uint8_t*>(ws_bases[j]);
    if (!b || (reinterpret_cast<uintptr_t>(b) & 255u)) return FW_EALIGN;
    P.part[j] = reinterpret_cast<const __nv_bfloat16*>(b + off("part"));
    P.red[j] = reinterpret_cast<__nv_bfloat16*>(b + off("tp.red"));
    P.flags[j] = reinterpret_cast<unsigned*>(b + off("tp.flags"));
    P.gat[j] = reinterpret_cast<float*>(b + off("tp.gat"));
  }
  P.epoch = reinterpret_cast<unsigned*>(const_cast<uint8_t*>(own) + off("tp.epoch"));
  h->use_peers = true;
  // The row-parallel GEMMs (sa.o, ca.o, ffn.2 of every block; call k of a forward uses parity
  // k % 2 of the receive buffers) also store their partial into the other ranks' memory while
  // they compute: with two ranks the whole partial into the peer's recv, with more the rows of
  // each rank's slice into that rank's recv slot (reduce-scatter), so the reduction kernels
  // read the partials from local memory.
  const char* pe = getenv("FW_TP_PUSH");
  if (!(pe && pe[0] == '0') && !h->fp8) {   // (the e4m3 row-parallel GEMMs do not push)
    const int Ls = (h->L + h->tp - 1) / h->tp;
    const size_t LD = (size_t)h->L * h->D;
    h->recv_stride = (size_t)h->tp * Ls * h->D;
    for (int j = 0; j < n; ++j) P.recv[j] = reinterpret_cast<__nv_bfloat16*>(reinterpret_cast<uint8_t*>(ws_bases[j]) + off("tp.recv"));
    for (int i = 0; i < h->cfg.layers; ++i) {
      fw::GemmOp* ops[3] = {&h->layers[i].o, &h->layers[i].cao, &h->layers[i].ff2};
      for (int k = 0; k < 3; ++k) {
        fw::GemmEpi& e = ops[k]->args.epi;
        const int parity = (3 * i + k) & 1;
        if (e.mode != fw::EPI_BF16 || e.out[0] != h->part) return FW_ESTATE;
        e.mode = fw::EPI_BF16_PUSH;
        e.tma_store = false;
        if (h->tp == 2) {
          e.peer_out = P.recv[1 - h->tpr] + (size_t)parity * LD;
        } else {
          e.push_tp = h->tp;
          e.push_rank = h->tpr;
          e.push_ls = Ls;
          for (int j = 0; j < n; ++j)
            e.push_base[j] = j == h->tpr ? nullptr : P.recv[j] + (size_t)parity * h->recv_stride;
        }
        int rc = fw::gemm_check(ops[k]->args, ops[k]->bn);
        if (rc) return rc;
      }
    }
    h->push = true;
  }
  return 0;
}

int fw_tp_reduce_once(fw_handle* h, void* stream) {
  if (!h) return FW_EINVAL;
  if (h->tp == 1 || !h->finalized || !(h->use_peers || h->comm)) return FW_ESTATE;
  return fw::row_parallel_done(h, "b0.sa.o.b", nullptr, nullptr, 0, reinterpret_cast<cudaStream_t>(stream));
}

int fw_tp_allreduce(fw_handle* h, void* buf, size_t count, int dtype, void* stream) {
  if (!h) return FW_EINVAL;
  if (!h->comm) return FW_ESTATE;
  return fw::tp_allreduce(h->comm, buf, count, dtype, reinterpret_cast<cudaStream_t>(stream));
}

int fw_copy(void* dst, const void* src, size_t bytes, void* stream) {
  return fw::copy_bytes(dst, src, bytes, reinterpret_cast<cudaStream_t>(stream));
}

}  // extern "C"
