// Host launchers of the memory-bound kernels in elem.cu (all return 0 or a negative FW_E* code).
#pragma once
#include "../../include/fastworld_b200.h"
#include "fw_internal.h"

namespace fw {

enum : int { ACT_NONE = 0, ACT_SILU = 1, ACT_GELU_ERF = 2 };

int ln_f32(const float* x, int ldx, int M, int D, float eps, const float* shift, const float* scale,
           const __nv_bfloat16* w, const __nv_bfloat16* b, __nv_bfloat16* out, int ldo, cudaStream_t s);
int ln_bf16(const __nv_bfloat16* x, int ldx, int M, int D, float eps, const float* shift, const float* scale,
            const __nv_bfloat16* w, const __nv_bfloat16* b, __nv_bfloat16* out, int ldo, cudaStream_t s);
// LayerNorm with e4m3 output and per-row scales (out8 row stride ldo bytes).
int ln_f32_q8(const float* x, int ldx, int M, int D, float eps, const float* shift, const float* scale,
              const __nv_bfloat16* w, const __nv_bfloat16* b, uint8_t* out8, float* sa, int ldo, cudaStream_t s);
int ln_bf16_q8(const __nv_bfloat16* x, int ldx, int M, int D, float eps, const float* shift, const float* scale,
               const __nv_bfloat16* w, const __nv_bfloat16* b, uint8_t* out8, float* sa, int ldo, cudaStream_t s);
// bf16 rows -> e4m3 rows + per-row scale absmax / 448.
int quant_rows(const __nv_bfloat16* x, int ldx, int M, int K, uint8_t* q, int ldq, float* scale, cudaStream_t s);
int rms_rope(const __nv_bfloat16* x, int ldx, int M, int D, float eps, const __nv_bfloat16* w, const float2* rope,
             int hd, __nv_bfloat16* out, int ldo, cudaStream_t s);
// Two tensors of the same shape in one launch (x2 may be null).
// In-place RMSNorm (no RoPE) of `groups` row blocks: block g is x + g * grp_stride ([M, D], row
// stride ldx) with weight w_grp[g] (a device array of pointers); one launch.
int rms_grp(__nv_bfloat16* x, long long grp_stride, int groups, const __nv_bfloat16* const* w_grp, int ldx, int M,
            int D, float eps, cudaStream_t s);
int rms_rope2(const __nv_bfloat16* x, const __nv_bfloat16* w, __nv_bfloat16* out, const __nv_bfloat16* x2,
              const __nv_bfloat16* w2, __nv_bfloat16* out2, int ldx, int M, int D, float eps, const float2* rope, int hd,
              int ldo, cudaStream_t s);
// rms_rope2 with the sum of squares of each full row given (ss[row * 2 + t], all-reduced over
// the tensor-parallel group) and d_full the full normalised width.
int rms_rope2_ss(const __nv_bfloat16* x, const __nv_bfloat16* w, __nv_bfloat16* out, const __nv_bfloat16* x2,
                 const __nv_bfloat16* w2, __nv_bfloat16* out2, int ldx, int M, int D, const float* ss, int d_full,
                 float eps, const float2* rope, int hd, int ldo, cudaStream_t s);
// ss[row * 2 + t] = sum of squares of row `row` of x0 (t = 0) and x1 (t = 1, optional).
int sumsq_rows(const __nv_bfloat16* x0, const __nv_bfloat16* x1, int ld, int M, int D, float* ss, cudaStream_t s);
// xs += gate[frame * gate_stride] * (p + bias) (gate, bias, mirror optional), for all-reduced
// row-parallel outputs.
int resid_add(float* xs, int ldx, const __nv_bfloat16* p, int ldp, const __nv_bfloat16* bias, const float* gate,
              int gate_stride, int rows_per_frame, __nv_bfloat16* mirror, int M, int D, cudaStream_t s);
// History window of several chunks: meta = {min(k, window) * L, L}; slot_copy writes slot k % window.
int hist_meta(const int* chunk, int window, int L, int* meta, cudaStream_t s);
int slot_copy(void* dst_base, size_t slot_bytes, const int* chunk, int window, const void* src, size_t bytes,
              cudaStream_t s);
int rope_tables(const int* chunk, int F, int th, int tw, int hd, double theta, float2* table, int act_hd,
                float* act_cos, float* act_sin, cudaStream_t s);
// Grouped small-M linears (one launch, blockIdx.y = group g): W = w[g], bias = bias[g] (device
// arrays of pointers; bias may be null), x and the outputs advanced by g * x_stride and
// g * out_stride elements.  Every w[g] must be 16-byte aligned with ldw % 8 == 0 for the
// vectorised path (the caller checks; `aligned`).
struct SmallmGrp {
  const __nv_bfloat16* const* w = nullptr;
  const __nv_bfloat16* const* bias = nullptr;
  long long x_stride = 0, out_stride = 0;
  int groups = 1;
  bool aligned = false;
};
int smallm_linear_f32(const float* x, int ldx, int M, const __nv_bfloat16* W, int ldw, const __nv_bfloat16* b, int N,
                      int K, int act_in, int act_out, float* outf, __nv_bfloat16* outb, int ldo, cudaStream_t s,
                      const SmallmGrp* grp = nullptr);
int smallm_linear_bf16(const __nv_bfloat16* x, int ldx, int M, const __nv_bfloat16* W, int ldw,
                       const __nv_bfloat16* b, int N, int K, int act_in, int act_out, float* outf,
                       __nv_bfloat16* outb, int ldo, cudaStream_t s, const SmallmGrp* grp = nullptr);
int sinusoid(double t, int dim, float* out, cudaStream_t s);
int modulation(const __nv_bfloat16* mods, const float* e0, int layers, int D, float* ee, const __nv_bfloat16* hmod,
               const float* e, float* head, cudaStream_t s);
int patchify(const __nv_bfloat16* x, int C1, const __nv_bfloat16* cc, int C2, int F, int H, int W, __nv_bfloat16* A,
             cudaStream_t s);
int scheduler(const float* head, const __nv_bfloat16* x, float sigma, __nv_bfloat16* den, __nv_bfloat16* out_copy,
              const __nv_bfloat16* noise, float sigma_n, __nv_bfloat16* xnext, int C, int F, int H, int W,
              cudaStream_t s);
int mouse_attn(const __nv_bfloat16* qkv, const __nv_bfloat16* wq, const __nv_bfloat16* wk, const float* acos_,
               const float* asin_, __nv_bfloat16* mk, __nv_bfloat16* mv, int first, int write, __nv_bfloat16* out,
               int S, int F, int AH, float eps, cudaStream_t s);
int kb_kv(const float* kv, const __nv_bfloat16* wk, const float* acos_, const float* asin_, __nv_bfloat16* kout,
          __nv_bfloat16* vout, int F, int AH, float eps, cudaStream_t s);
// kb_kv for `groups` action layers in one launch: layer g reads kv + g * F * 2A with weight
// wk_grp[g] and writes kout / vout + g * F * A.
int kb_kv_grp(const float* kv, const __nv_bfloat16* const* wk_grp, int groups, const float* acos_,
              const float* asin_, __nv_bfloat16* kout, __nv_bfloat16* vout, int F, int AH, float eps, cudaStream_t s);
int kb_attn(const __nv_bfloat16* mq, const __nv_bfloat16* wq, const float* acos_, const float* asin_,
            const __nv_bfloat16* kh, const __nv_bfloat16* vh, const __nv_bfloat16* kc, const __nv_bfloat16* vc,
            int first, __nv_bfloat16* out, int L, int S, int F, int AH, float eps, cudaStream_t s);
int copy_bytes(void* dst, const void* src, size_t bytes, cudaStream_t s);
// fw_prep's kernel (prep.cu): noise_dst[0] = x_in, noise_dst[t] = the noise of step t - 1.
int prep_launch(const fw_config& c, const fw_prep_args& p, int* chunk, __nv_bfloat16* kc, __nv_bfloat16* gm,
                __nv_bfloat16* cc, __nv_bfloat16* const* noise_dst, int n_noise, int* status, cudaStream_t s);

}  // namespace fw
