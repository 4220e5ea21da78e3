/* fastworld_b200: C ABI of the B200 (sm_100a) chunk-forward engine for the Matrix-Game-2-shaped
 * causal Wan DiT.
 *
 * The engine replaces the device work behind the reference's session object
 * (fastworld/models/mg2/static.py, class StaticMG) and keeps its calling convention: the
 * caller allocates every buffer (weights, session state, static inputs, workspace), binds
 * raw pointers once, and then launches whole chunks or single forwards on a stream.  The
 * library owns no device memory, never allocates, never synchronises inside a launch call,
 * and every launch is capturable into a CUDA graph (fastworld/graph.py:13-33).
 *
 * Return values: 0 on success, a negative FW_E* code on a host-side error.  Device-side
 * errors (a bounded wait that ran out) are written to the bound "status" word (int32[4]),
 * which the caller reads after synchronising.
 *
 * Reference interfaces replaced (file:line in StevenCYLu/fastworld):
 *   fw_create / fw_tensor_* / fw_bind / fw_finalize  StaticMG.__init__        static.py:28-73
 *   fw_chunk                                         StaticMG._chunk          static.py:232-242
 *   fw_prefill                                       StaticMG._prefill        static.py:244-245
 *   fw_forward                                       StaticMG._net            static.py:194-230
 *   fw_copy                                          StaticMG.state / load    static.py:273-278
 *   fw_graph_*                                       graph.capture            graph.py:13-33
 *   fw_gemm_bf16, fw_attention, fw_* ops             the torch / flash-attn calls inside _net
 */
#ifndef FASTWORLD_B200_H
#define FASTWORLD_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define FW_ABI_VERSION 2

/* error codes */
#define FW_OK 0
#define FW_EINVAL (-1)      /* bad argument (null pointer, unknown name, bad enum) */
#define FW_ESHAPE (-2)      /* unsupported or inconsistent shape */
#define FW_EALIGN (-3)      /* pointer or stride alignment (16 bytes for TMA / vector access) */
#define FW_ECUDA (-4)       /* a CUDA runtime call failed */
#define FW_ENOTBOUND (-5)   /* fw_finalize: a required tensor was not bound */
#define FW_ENODRIVER (-6)   /* cuTensorMapEncodeTiled unavailable */
#define FW_ESTATE (-7)      /* call out of order (e.g. launch before fw_finalize) */
#define FW_ESIZE (-8)       /* bound buffer smaller than required */
#define FW_ESCRATCH (-9)    /* problem larger than the fixed scratch of fw_linear_e4m3_noalloc */
#define FW_ENCCL (-10)      /* NCCL unavailable or an NCCL call failed */

/* tensor kinds (fw_tensor_info.kind) */
#define FW_KIND_WEIGHT 0
#define FW_KIND_STATE 1     /* session state: history K/V and action-module K/V */
#define FW_KIND_INPUT 2     /* static per-chunk inputs written by the host before a launch */
#define FW_KIND_OUTPUT 3
#define FW_KIND_WORKSPACE 4
#define FW_KIND_STATUS 5
#define FW_KIND_DERIVED 6   /* filled by fw_finalize from the weights (e4m3 copies, scales) */

/* dtypes */
#define FW_BF16 0
#define FW_F32 1
#define FW_I32 2
#define FW_U8 3
#define FW_F16 4

#define FW_MAX_ACTION_BLOCKS 64
#define FW_MAX_STEPS 16

/* Model + schedule.  Mirrors fastworld_b200.config.DiTConfig. */
typedef struct fw_config {
  int dim, heads, head_dim, ffn, layers, freq_dim;
  int lat_ch, cond_ch, frames, lat_h, lat_w;          /* patch is fixed to (1, 2, 2) */
  int ctx_tokens, ctx_dim;
  int n_action, action_blocks[FW_MAX_ACTION_BLOCKS];
  int act_heads, act_head_dim, mouse_hidden, keyboard_hidden, mouse_dim, keyboard_dim;
  int time_ratio, window;
  int n_steps;
  float steps[FW_MAX_STEPS];                          /* denoising timesteps; context forward at t = 0 */
  float eps;                                          /* block LayerNorm / RMSNorm eps */
  float eps_ln;                                       /* img_emb / mouse_mlp LayerNorm eps */
  float rope_theta;
  int linear_fp8;                                     /* 1: block linears in e4m3;
                                                         2: only the FFN linears in e4m3 */
  /* KV history window in chunks (1 = MG2: the previous chunk only).  With W > 1 the history
   * buffer holds W chunk slots; chunk k's context forward writes slot k % W and a steady
   * chunk attends to the min(k, W) filled slots and the current chunk. */
  int hist_chunks;
  /* Tensor parallelism: this handle computes heads
   * [tp_rank * heads / tp_size, ...) and the same share of the FFN columns; tensors are
   * registered with the local widths.  tp_size 1 = the whole model on one GPU. */
  int tp_size, tp_rank;
} fw_config;

typedef struct fw_tensor_info {
  const char* name;
  int kind, dtype, ndim;
  int64_t shape[5];
  size_t bytes;
} fw_tensor_info;

typedef struct fw_handle fw_handle;

int fw_abi_version(void);
const char* fw_strerror(int code);
/* Number of kernels this library has enqueued so far (all threads; monotonic). */
unsigned long long fw_launch_count(void);

/* ---- session engine (StaticMG, static.py:27-284) ---- */
int fw_create(const fw_config* cfg, fw_handle** out);
int fw_tensor_count(const fw_handle* h);
int fw_tensor_info_at(const fw_handle* h, int index, fw_tensor_info* info);
/* Bind a caller-owned device buffer of at least the reported size to a tensor name. */
int fw_bind(fw_handle* h, const char* name, void* ptr, size_t bytes);
/* Validate bindings, build TMA descriptors, upload constant tables (synchronous, once). */
int fw_finalize(fw_handle* h);
/* One chunk: n_steps denoising forwards with the flow-matching update between them, then
 * the context forward at t = 0 that writes the history (static.py:232-242).  Reads the
 * inputs x_in, noise.*, cc, vis, gm, kc, chunk; writes out and the state tensors.
 * first != 0: chunk 0 (no history keys). */
int fw_chunk(fw_handle* h, int first, void* stream);
/* Context forward over the bound lat_in only (static.py:244-245). */
int fw_prefill(fw_handle* h, int first, void* stream);
/* One forward (static.py:194-230) at timestep index `step` (n_steps = the context forward
 * at t = 0) from latent x_cur into den; write != 0 updates the history. */
int fw_forward(fw_handle* h, int step, int first, int write, void* stream);
/* Destroys the handle and, with tp_size > 1, its NCCL communicator (release every CUDA graph
 * that captured this handle's launches first). */
void fw_destroy(fw_handle* h);

/* Chunk preparation on the device (StaticMG._prep, static.py:76-127), one launch that reads no
 * host memory: writes the chunk info {k, frames * k}, the action module's keyboard / mouse
 * windows (kc, gm), the image condition slice cc = cond[:, frames * k : frames * (k + 1)] and,
 * with draw_noise, x_in and the per-step renoising noise as N(0, 1) bf16 from Philox-4x32-10
 * keyed by `seed` (a different stream from the reference's torch.randn; see prep.cu).
 * actions: chunks j_lo .. j_lo + n_act - 1, 8 floats each (keyboard then mouse values); they
 * must cover every chunk the window reads (else status DEV_PREP_ACTIONS = 8, zeros written).
 * cond: bf16 [cond_ch, cond_frames, H, W] on the device, cond_frames >= frames * (chunk + 1). */
#define FW_PREP_MAX_ACT 4
typedef struct fw_prep_args {
  int chunk;
  unsigned long long seed;
  int draw_noise;
  const void* cond;
  int cond_frames;
  int j_lo, n_act;
  float actions[FW_PREP_MAX_ACT * 8];
} fw_prep_args;
int fw_prep(fw_handle* h, const fw_prep_args* args, void* stream);
/* Philox-4x32-10 of one counter under one key (host function; the generator fw_prep uses). */
int fw_philox4x32_10(const unsigned* counter4, const unsigned* key2, unsigned* out4);

/* Parity tap (the reference's exactness ladder compares one forward layer by layer,
 * scripts/mg2/test_static.py:50-57): while set, every forward copies block `layer`'s
 * intermediates into `buf` (fw_tap_bytes(h) bytes, 16-byte aligned):
 *   fp32 [L, D] residual stream at 5 points: block input, after self-attention (+ gated o-proj),
 *   after cross-attention, after the action module (= the previous one without it), block output;
 *   then bf16 [L, Dl]: q and k after RMSNorm + RoPE, v, and the self-attention output.
 * layer < 0 or buf == NULL clears it.  Meant for eager launches; a graph recorded while a tap is
 * set replays the copies. */
size_t fw_tap_bytes(const fw_handle* h);
int fw_set_tap(fw_handle* h, int layer, void* buf, size_t bytes);

/* ---- tensor parallelism (no counterpart in the reference, whose runtimes are single-GPU;
 * BASELINE configs[4]) ----
 * NCCL is loaded at run time (libnccl.so.2: the copy already in the process if any).
 * fw_tp_unique_id: on one rank, 128 bytes to broadcast to every rank of the group.
 * fw_tp_init: on every rank (collective, blocking), after fw_create and before the first
 * launch; the engine then all-reduces (sum) the row-parallel partial outputs of sa.o,
 * ca.o and ffn.2 and the per-token sums of squares of the q/k RMSNorms over the group,
 * enqueued on the launch stream (capturable). */
int fw_tp_unique_id(void* id128);
int fw_tp_init(fw_handle* h, const void* id128);
/* Peer-memory reductions (replace NCCL for the engine's collectives): after fw_finalize on every
 * rank, pass the tp workspace base addresses as seen from this process (index = rank; this
 * rank's own binding at its index, the others mapped with fw_ipc_open).  The engine then sums
 * the row-parallel partials with one kernel per linear that reads and writes the other GPUs'
 * workspaces over NVLink and applies bias + gated residual in the same pass (two-shot), and
 * gathers the RMSNorm sums of squares the same way.  Every rank must call it, before its first
 * launch. */
int fw_tp_peers(fw_handle* h, void* const* ws_bases, int n);
/* One row-parallel reduction step of the engine (sum of every rank's partial output buffer,
 * block 0's O-projection bias, residual update of the handle's workspace), on the path the
 * handle uses (peer kernels or NCCL); for timing and tests.  Collective: every rank calls it. */
int fw_tp_reduce_once(fw_handle* h, void* stream);
/* In-place sum all-reduce over the handle's group (dtype FW_BF16 or FW_F32); for tests. */
int fw_tp_allreduce(fw_handle* h, void* buf, size_t count, int dtype, void* stream);

/* ---- checkpoint copies (state save / restore / migrate; static.py:273-278) ----
 * Vectorised device copy of `bytes` (16-byte aligned pointers; any size).  `src` may be a
 * peer GPU's memory when peer access is enabled. */
int fw_copy(void* dst, const void* src, size_t bytes, void* stream);

/* Export the cudaMalloc allocation that contains `ptr`: its 64-byte IPC handle and the byte
 * offset of `ptr` inside it (for fw_ipc_open in another process). */
int fw_ipc_get_handle(const void* ptr, void* handle, size_t* offset);
/* Map another process's device allocation (a 64-byte cudaIpcMemHandle_t of its base) into the
 * CURRENT device's address space with peer access enabled, so kernels on this GPU (fw_copy) can
 * read it over NVLink; close it with fw_ipc_close once the copy has completed. */
int fw_ipc_open(const void* handle, void** ptr);
int fw_ipc_close(void* ptr);

/* ---- CUDA graphs held by the library (replace torch.cuda.CUDAGraph in graph.capture,
 * fastworld/graph.py:13-33) ----
 * fw_graph_begin starts recording `stream` (thread-local capture: launches this thread issues on
 * `stream` are recorded, not executed; not the legacy default stream); fw_graph_end stops
 * recording and instantiates the executable graph (it always ends the capture, also on error);
 * fw_graph_launch replays it on any stream of the same device; fw_graph_destroy frees it.
 * Recorded work must only read and write buffers that outlive the graph. */
typedef struct fw_graph fw_graph;
int fw_graph_begin(void* stream);
int fw_graph_end(void* stream, fw_graph** out);
int fw_graph_launch(const fw_graph* g, void* stream);
int fw_graph_nodes(const fw_graph* g, size_t* n);
void fw_graph_destroy(fw_graph* g);
/* Let kernels on the current device read and write `peer`'s memory (checkpoints placed on
 * another GPU; fastworld/prefix_cache.py:85-87 keeps every checkpoint on the GPU that made it). */
int fw_peer_access(int peer);

/* ---- TAEHV streaming video decoder (TinyVAE, fastworld/models/mg2/vae.py:95-124) ----
 * Decodes one latent chunk "lat" [16, lat_frames, lat_h, lat_w] (fp16, as the reference casts it) into
 * lat_frames * prod(time_up) RGB frames [frames, 3, 8 lat_h, 8 lat_w] fp32 in [-1, 1], carrying
 * the streaming state (each MemBlock's last input frame, tensor "mem") from chunk to chunk.
 * Tensors are registered and bound like the session engine's (fw_taehv_tensor_info_at /
 * fw_taehv_bind): weights fp16 [Cout, taps * Cin] with K ordered (tap, input channel), biases
 * fp32; "conv_in.w" is [C0, 192]: 9 taps x 16 latent channels, then 48 zero columns;
 * "conv_out.wt" is the last conv transposed, [32, C3] with row (ky * 3 + kx) * 3 + c (27 used),
 * "conv_out.b" fp32 [32] (3 used); "work" is the activation
 * workspace and "status" the int32[4] device status word (zeroed).  fw_taehv_finalize builds the
 * TMA descriptors; fw_taehv_decode launches the whole decoder (no host synchronisation;
 * graph-capturable).
 * A zeroed "mem" is the state of a new stream; the caller drops the first
 * prod(time_up) - 1 frames of a stream's first chunk (TAEHV's frames_to_trim). */
typedef struct fw_taehv_config {
  int lat_ch;          /* 16 */
  int lat_frames;      /* latent frames per chunk (MG2: 3) */
  int lat_h, lat_w;    /* latent size (MG2: 44 x 80); lat_w a multiple of 16 */
  int channels[4];     /* stage widths (taew2_1: 256, 128, 64, 64), multiples of 64, <= 256 */
  int time_up[3];      /* frames per input frame at the three upsampling steps (1, 2, 2) */
} fw_taehv_config;
typedef struct fw_taehv fw_taehv;
int fw_taehv_create(const fw_taehv_config* cfg, fw_taehv** out);
int fw_taehv_tensor_count(const fw_taehv* h);
int fw_taehv_tensor_info_at(const fw_taehv* h, int index, fw_tensor_info* info);
int fw_taehv_bind(fw_taehv* h, const char* name, void* ptr, size_t bytes);
int fw_taehv_finalize(fw_taehv* h);
int fw_taehv_decode(fw_taehv* h, void* stream);
/* Device status word (0 = every bounded wait completed); synchronous. */
int fw_taehv_status(fw_taehv* h, int* out);
void fw_taehv_destroy(fw_taehv* h);

/* ---- LingBot-World-v2 causal runtime (StaticLingbot, fastworld/models/lingbot_v2/static.py:49-320) ----
 * A Wan-1.3B I2V DiT with a camera injector, text cross-attention and a KV window of kv_frames
 * frames with a sink of sink_frames, served chunk by chunk.  Tensors are registered and bound
 * like the session engine's (fw_lb_tensor_info_at / fw_lb_bind): packed bf16 weights
 * (b<i>.sa.qkv = q | k | v rows, b<i>.ca.kv = k | v rows), state
 * K.<i> / V.<i> [kv_frames * tokens per frame, dim], fp32 latents (x_in, noise.<i>, y_in, out),
 * bf16 Plücker features pl_in, the padded prompt ctx_in, and per chunk the device plan
 * int32[8] = {write offset, key length, 0, roll src, roll dst, roll rows, roll piece rows, 0}
 * (rows = tokens) and chunk int32[4] = {k, chunk * k, 0, 0} (RoPE frame offset).
 * fw_lb_set_prompt: text embedding and every block's cross-attention K/V (derived tensors
 * xk, xv) from ctx_in; fw_lb_chunk: one chunk (camera branch, n_steps forwards, the t = 0 key
 * refresh, the roll); both graph-capturable, no host synchronisation. */
typedef struct fw_lb_config {
  int dim, heads, head_dim, ffn, layers, freq_dim;
  int text_len, text_dim;
  int lat_ch, y_ch, cam_ch, chunk, lat_h, lat_w;
  int kv_frames, sink_frames;
  int n_steps;
  float eps;
  float timesteps[8];
  double sig_x0[8];      /* fp64 sigma of each step's x0 conversion */
  float an_alpha[8];     /* renoising to step i + 1: alpha * x0 + sigma * noise */
  float an_sigma[8];
} fw_lb_config;
typedef struct fw_lb fw_lb;
int fw_lb_create(const fw_lb_config* cfg, fw_lb** out);
int fw_lb_tensor_count(const fw_lb* h);
int fw_lb_tensor_info_at(const fw_lb* h, int index, fw_tensor_info* info);
int fw_lb_bind(fw_lb* h, const char* name, void* ptr, size_t bytes);
int fw_lb_finalize(fw_lb* h);
int fw_lb_set_prompt(fw_lb* h, void* stream);
int fw_lb_chunk(fw_lb* h, void* stream);
/* Roll launches per chunk (the most pieces any plan of this window needs). */
int fw_lb_roll_pieces(const fw_lb* h);
void fw_lb_destroy(fw_lb* h);

/* ---- failure-path self-tests (no counterpart in the reference, which has no device-side
 * failure detection) ----
 * Runs a bounded wait that nothing satisfies, so that it runs out after `limit_ns`
 * (0 < limit_ns <= 2 s): which 0 = an mbarrier wait of the kind every tcgen05 kernel's warp roles
 * use (a CTA holding TMEM; expected status DEV_TIMEOUT_TEST = 6), which 1 = the two-rank peer
 * reduction kernel waiting for a rank that never runs (its buffers are this GPU's own memory;
 * expected status DEV_TIMEOUT_PEER = 7).  `scratch`: fw_selftest_bytes(which) zeroed bytes,
 * 256-byte aligned; `status`: int32[4], zeroed.  Nothing faults; the context stays usable. */
size_t fw_selftest_bytes(int which);
int fw_selftest_wait(int which, unsigned long long limit_ns, void* scratch, size_t bytes, int* status, void* stream);

/* ---- individual kernels (used by the engine; exported for tests and reuse) ---- */
/* C[M,N] = A[M,K] B[N,K]^T (+ bias[N]) with A, B, C bf16 row-major, fp32 accumulate.
 * epilogue: 0 = store bf16, 1 = GELU(tanh) then bf16, 3 = store fp32 (out is float*).
 * tile_n: 64 / 128 / 256 = one CTA per 128 x tile_n tile; 224 = the same with 224-wide tiles
 * (fp32 output only); 512 = a CTA pair per 256 x 256 tile (tcgen05 cta_group::2); 0 = default. */
int fw_gemm_bf16(const void* A, const void* B, const void* bias, void* out, int M, int N, int K, int epilogue,
                 int tile_n, void* stream);
/* e4m3 operands (A8 [M,K], B8 [N,K] bytes, K % 16 == 0): C = (A8 B8^T) * sa[row] * sw[col] (+ bias),
 * fp32 accumulate; epilogues as fw_gemm_bf16.  BASELINE configs[2]. */
int fw_gemm_e4m3(const void* A8, const float* sa, const void* B8, const float* sw, const void* bias, void* out,
                 int M, int N, int K, int epilogue, int tile_n, void* stream);
/* Per-row e4m3 quantisation of bf16 x [M,K]: scale[row] = absmax / 448, q = e4m3(x / scale). */
int fw_quant_e4m3(const void* x, int M, int K, void* q, float* scale, void* stream);
/* e4m3 linear layer for callers that cannot allocate device memory (no counterpart in the
 * reference).  out[M,N] (bf16) = per-token-e4m3(x[M,K] bf16) * (w8[N,K] e4m3 * sw[N])^T + bias,
 * the same computation as fw_quant_e4m3 into caller scratch followed by fw_gemm_e4m3, but the
 * quantised copy of x lives in a fixed array inside the library (32 MiB of activations and
 * 16384 row scales per GPU, held until the process exits): M * K must be <= 32 MiB and
 * M <= 16384, else FW_ESCRATCH; shapes and alignments the GEMM rejects are refused before
 * anything is launched.  It calls no cudaMalloc / cudaFree.  The first call in a CUDA context
 * (with that context's device current) looks up the array's device address and caches it for
 * that context; make that first call before any stream capture.  All calls share the array and it keeps the last call's
 * contents: calls whose executions overlap on the GPU (other streams, other threads) race. */
int fw_linear_e4m3_noalloc(const void* x, const void* w8, const float* sw, const void* bias, void* out, int M, int N,
                           int K, void* stream);
/* resid[M,N] (fp32) += gate[row / rows_per_frame, N] * (A B^T + bias); gate may be NULL. */
int fw_gemm_bf16_resid(const void* A, const void* B, const void* bias, float* resid, const float* gate,
                       int rows_per_frame, int M, int N, int K, void* stream);
/* LayerNorm of fp32 rows x [M, D] (no affine) into bf16 out [M, D], fp32 statistics, followed by
 * y * (1 + scale) + shift (adaLN modulate, fp32 [D] each; norm1 / norm2, static.py:206, 224) or
 * y * w + b (bf16 [D] each; norm3, static.py:221), or neither (all four NULL). */
int fw_layernorm(const float* x, int M, int D, float eps, const float* shift, const float* scale, const void* w,
                 const void* b, void* out, void* stream);
/* RMSNorm over the full row of bf16 x [M, D] times w (bf16 [D]), then, when rope != NULL, each
 * (even, odd) pair of every head of head_dim rotated by rope[row, pair] = (cos, sin) (fp32
 * [M, head_dim / 2, 2]); bf16 out [M, D] (may equal x).  static.py:207-212 (norm_q / norm_k,
 * then _rope at static.py:130-133 in fp32 instead of fp64). */
int fw_rms_rope(const void* x, int M, int D, float eps, const void* w, const float* rope, int head_dim, void* out,
                void* stream);
/* Non-causal attention, head_dim 128: out[Lq, H*128] = softmax(q k^T / sqrt(128)) v over the
 * keys of segment 0 then segment 1.  meta = device int32 {n_keys0, n_keys1}.  max_keys0/1
 * are the row capacities of the segment buffers. */
int fw_attention(const void* q, int Lq, int heads, const void* k0, const void* v0, int max_keys0, const void* k1,
                 const void* v1, int max_keys1, const int* meta, void* out, int* status, void* stream);

#ifdef __cplusplus
}
#endif
#endif /* FASTWORLD_B200_H */
