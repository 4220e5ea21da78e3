// Internal (C++) interfaces shared by the translation units of libfastworld_b200.
#pragma once
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <utility>

namespace fw {

// ---------------------------------------------------------------- host utilities
typedef CUresult (*PFN_encodeTiled)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                    const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                    CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);
// Resolves cuTensorMapEncodeTiled through the runtime's driver entry point (no -lcuda).
PFN_encodeTiled get_encode_fn();
// 2-D row-major tensor [rows, cols] of `elem_bytes` elements with row stride `ld` elements;
// box = [box_rows, box_cols]; 128-byte swizzle (box_cols * elem_bytes must be 128) or none.
// Returns 0 or a negative FW_E* code.
int make_tmap_2d(CUtensorMap* out, const void* base, int elem_bytes, int64_t rows, int64_t cols, int64_t ld,
                 int box_rows, int box_cols, bool swizzle128);
int num_sms();
// Counts kernel launches enqueued by this library (all threads); read with fw_launch_count().
void note_launch();
// Programmatic dependent launch (on unless FW_PDL=0 in the environment): every kernel of the
// library signals griddepcontrol.launch_dependents on entry and waits (griddepcontrol.wait)
// before touching data produced upstream, so the next kernel's launch and prologue overlap the
// tail of the current one, in streams and in captured graphs alike.
bool pdl_enabled();
// Residual GEMM epilogues without a bf16 mirror add into the fp32 residual by TMA reduce-add
// (EPI_RESID_TMA) unless FW_RESID_TMA=0 in the environment (then EPI_RESID_F32).
bool resid_tma_enabled();

template <typename... KArgs, typename... Args>
inline cudaError_t launch_k(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t s,
                            Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl_enabled() ? 1 : 0;
  const cudaError_t e = cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
  note_launch();
  return e;
}

// ---------------------------------------------------------------- GEMM
enum EpiMode : int {
  EPI_BF16 = 0,        // out_bf16 = acc + bias                                   (split by column segment)
  EPI_GELU_BF16 = 1,   // out_bf16 = gelu_tanh(acc + bias)
  EPI_RESID_F32 = 2,   // resid_f32 += gate[frame] * (acc + bias); optional bf16 mirror of resid
  EPI_F32 = 3,         // out_f32 = acc + bias
  EPI_GELU_ERF_BF16 = 4,   // out_bf16 = gelu_erf(acc + bias)
  EPI_RESID_TMA = 5,   // resid_f32 += gate[frame] * (acc + bias) by TMA reduce-add (no mirror; needs tmC)
  EPI_BF16_PUSH = 6,   // out_bf16 = acc + bias, stored coalesced to out[0] and to other GPUs (see GemmEpi)
};

struct GemmEpi {
  int mode = EPI_BF16;
  void* out[3] = {nullptr, nullptr, nullptr};   // destinations by column segment
  int ld_out = 0;                               // elements
  int seg_w = 0;                                // column segment width (multiple of the tile N)
  const __nv_bfloat16* bias = nullptr;          // [N] bf16 (optional)
  const float* fbias = nullptr;                 // [frames, fbias_stride] fp32 per-frame bias (optional)
  int fbias_stride = 0;
  const float* gate = nullptr;                  // [frames, gate_stride] fp32 (EPI_RESID_F32, optional)
  int gate_stride = 0;
  float* resid = nullptr;                       // [M, ld_resid] fp32
  int ld_resid = 0;
  __nv_bfloat16* mirror = nullptr;              // [M, ld_mirror] bf16 copy of the new residual (optional)
  // EPI_BF16_PUSH, besides out[0]: either every row to peer_out [M, ld_out] (two ranks), or
  // (push_tp > 2) the rows of slice j = row / push_ls to rank j's receive buffer push_base[j],
  // at slot push_rank: push_base[j] + (push_rank * push_ls + row - j * push_ls) * ld_out
  // (this rank's own slice stays in out[0] only).
  __nv_bfloat16* peer_out = nullptr;
  __nv_bfloat16* push_base[8] = {};
  int push_tp = 0, push_rank = 0, push_ls = 0;
  int ld_mirror = 0;
  int rows_per_frame = 1 << 30;
  // bf16 output modes: store each warp's 32 x 64 box with a TMA store through the output tensor
  // maps (one per column segment, box [32 rows, 64 cols], 128-byte swizzle) instead of st.global
  bool tma_store = false;
};

struct GemmArgs {
  int M = 0, N = 0, K = 0;
  GemmEpi epi;
  // e4m3 operands (A and B are bytes) when sa != null: sa[M] per-row activation scales,
  // sw[N] per-column (output channel) weight scales; acc is multiplied by sa[row] * sw[col].
  const float* sa = nullptr;
  const float* sw = nullptr;
  int* status = nullptr;
  // Grouped launch (groups > 1; bf16 output modes, tile width >= 128): group g multiplies the
  // same A by B_g (tensor map tmB_grp[g], in device memory, 64-byte aligned), adds bias_grp[g]
  // and writes the out[] segments shifted by g * out_grp_stride elements.
  int groups = 1;
  // B is not written by any kernel of the stream (the engine's weights): its first loads may be
  // issued before the programmatic-dependent-launch wait
  bool b_static = false;
  const CUtensorMap* tmB_grp = nullptr;
  const __nv_bfloat16* const* bias_grp = nullptr;
  long long out_grp_stride = 0;
};

// C[M,N] = A[M,K] * B[N,K]^T.  tmA: box [128 rows, 64 cols]; tmB: box [bn rows, 64 cols];
// bn in {64, 128, 256}.  `ctas` = 0 uses one CTA per SM (persistent).
// tmC: the fp32 residual [M, ld_resid] with box [32 rows, 32 cols], 128-byte swizzle, for
// EPI_RESID_TMA (ignored otherwise).
// tmO: with epi.tma_store, the output tensor maps of the column segments (make_out_tmaps).
int gemm_bf16_launch(const CUtensorMap& tmA, const CUtensorMap& tmB, int bn, const GemmArgs& a, cudaStream_t s,
                     int ctas = 0, const CUtensorMap* tmC = nullptr, const CUtensorMap* tmO = nullptr);
// Output tensor maps for a bf16-output GEMM (one per column segment of a.epi) and sets
// a.epi.tma_store; leaves the st.global path (returns 0, tma_store false) for grouped launches.
int make_out_tmaps(GemmArgs& a, CUtensorMap (&o)[3]);
int gemm_check(const GemmArgs& a, int bn);
// Tile width for a bf16 GEMM with a 32-column epilogue (residual, fp32 output): 224 where it
// needs no more waves of the GPU's SMs than 256 and so gives each SM less work, else 256
// (64 / 128 for narrow outputs).
int gemm_resid_bn(int M, int N);
// CTA-pair variant (gemm2.cu): 256 x 256 tiles; tmA box [128 rows, 64 cols] as above, tmB box
// [128 rows, 64 cols] (half a tile of output columns per CTA).
int gemm_pair_launch(const CUtensorMap& tmA, const CUtensorMap& tmB, const GemmArgs& a, cudaStream_t s,
                     const CUtensorMap* tmC = nullptr);
// Pair tiles for the engine's large linears only with FW_GEMM_PAIR=1 in the environment: in
// isolation they beat one-CTA tiles on the 14B shapes by up to 13 %, but a whole 14B chunk
// (weights streamed from HBM) measured the same either way (837.9 vs 834.5 ms).
bool gemm_pair_enabled();

// ---------------------------------------------------------------- attention
struct AttnArgs {
  int Lq = 0;           // query rows
  int heads = 0;        // heads (head_dim 128)
  const int* meta = nullptr;   // device int32 {n_keys_seg0, n_keys_seg1}
  int max_keys0 = 0, max_keys1 = 0;   // capacity of each segment (host-known bound)
  __nv_bfloat16* out = nullptr;       // [Lq, heads*128]
  int ld_out = 0;
  float scale_log2 = 0.f;             // softmax scale * log2(e)
  int* status = nullptr;
};
// Q [Lq, heads*128] (tmQ box [128, 64]); K/V segments [keys, heads*128] (box [128, 64]).
// tmO (optional): the output [Lq, heads*128] with box [128, 64], 128-byte swizzle; O is then
// written by TMA stores.
int attention_launch(const CUtensorMap& tmQ, const CUtensorMap& tmK0, const CUtensorMap& tmV0,
                     const CUtensorMap& tmK1, const CUtensorMap& tmV1, const AttnArgs& a, cudaStream_t s,
                     const CUtensorMap* tmO = nullptr);

}  // namespace fw
