// Host utilities (TMA descriptors, device queries) and the op-level C ABI entry points.
#include <atomic>
#include <cstdlib>
#include <cmath>
#include <cstring>

#include "../../include/fastworld_b200.h"
#include "fw_elem.h"
#include "fw_internal.h"

namespace fw {

PFN_encodeTiled get_encode_fn() {
  static PFN_encodeTiled fn = nullptr;
  if (!fn) {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_encodeTiled>(p);
  }
  return fn;
}

static std::atomic<unsigned long long> g_launches{0};
void note_launch() { g_launches.fetch_add(1, std::memory_order_relaxed); }

bool gemm_pair_enabled() {
  static const bool on = [] {
    const char* e = getenv("FW_GEMM_PAIR");
    return e && e[0] == '1';
  }();
  return on;
}

bool resid_tma_enabled() {
  static const bool on = [] {
    const char* e = getenv("FW_RESID_TMA");
    return !(e && e[0] == '0');
  }();
  return on;
}

bool pdl_enabled() {
  static const bool on = [] {
    const char* v = getenv("FW_PDL");
    return !(v && v[0] == '0');
  }();
  return on;
}

int num_sms() {
  int dev = 0, n = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return 148;
  if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) return 148;
  return n;
}

int make_tmap_2d(CUtensorMap* out, const void* base, int elem_bytes, int64_t rows, int64_t cols, int64_t ld,
                 int box_rows, int box_cols, bool swizzle128) {
  PFN_encodeTiled enc = get_encode_fn();
  if (!enc) return FW_ENODRIVER;
  if (!base || rows <= 0 || cols <= 0 || box_rows <= 0 || box_rows > 256 || box_cols <= 0) return FW_EINVAL;
  if (reinterpret_cast<uintptr_t>(base) & 15u) return FW_EALIGN;
  if ((ld * elem_bytes) % 16) return FW_EALIGN;
  if (swizzle128 && box_cols * elem_bytes != 128) return FW_EINVAL;
  CUtensorMapDataType dt = elem_bytes == 2 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16
                           : elem_bytes == 1 ? CU_TENSOR_MAP_DATA_TYPE_UINT8
                                             : CU_TENSOR_MAP_DATA_TYPE_FLOAT32;
  cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)(ld * elem_bytes)};
  cuuint32_t box[2] = {(cuuint32_t)box_cols, (cuuint32_t)box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = enc(out, dt, 2, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                   swizzle128 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_NONE,
                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? 0 : FW_EINVAL;
}

}  // namespace fw

extern "C" {

unsigned long long fw_launch_count(void) { return fw::g_launches.load(std::memory_order_relaxed); }

int fw_gemm_bf16(const void* A, const void* B, const void* bias, void* out, int M, int N, int K, int epilogue,
                 int tile_n, void* stream) {
  using namespace fw;
  if (!A || !B || !out) return FW_EINVAL;
  if (epilogue != EPI_BF16 && epilogue != EPI_GELU_BF16 && epilogue != EPI_F32 && epilogue != EPI_GELU_ERF_BF16)
    return FW_EINVAL;
  const int bn = tile_n > 0 ? tile_n : (N >= 256 ? 256 : (N >= 128 ? 128 : 64));
  if (bn != 64 && bn != 128 && bn != 224 && bn != 256 && bn != 512) return FW_EINVAL;
  if (bn == 224 && epilogue != EPI_F32) return FW_EINVAL;   // 224-wide tiles: 32-column epilogues only
  CUtensorMap ta, tb;
  int rc = make_tmap_2d(&ta, A, 2, M, K, K, 128, 64, true);
  if (!rc) rc = make_tmap_2d(&tb, B, 2, N, K, K, bn == 512 ? 128 : bn, 64, true);
  if (rc) return rc;
  GemmArgs a;
  a.M = M;
  a.N = N;
  a.K = K;
  a.epi.mode = epilogue;
  a.epi.out[0] = out;
  a.epi.ld_out = N;
  a.epi.seg_w = 1 << 30;
  a.epi.bias = reinterpret_cast<const __nv_bfloat16*>(bias);
  if (bn == 512) return gemm_pair_launch(ta, tb, a, reinterpret_cast<cudaStream_t>(stream));
  CUtensorMap to[3];
  rc = make_out_tmaps(a, to);
  if (rc) return rc;
  return gemm_bf16_launch(ta, tb, bn, a, reinterpret_cast<cudaStream_t>(stream), 0, nullptr, to);
}

int fw_gemm_e4m3(const void* A8, const float* sa, const void* B8, const float* sw, const void* bias, void* out,
                 int M, int N, int K, int epilogue, int tile_n, void* stream) {
  using namespace fw;
  if (!A8 || !sa || !B8 || !sw || !out) return FW_EINVAL;
  if (epilogue != EPI_BF16 && epilogue != EPI_GELU_BF16 && epilogue != EPI_F32 && epilogue != EPI_GELU_ERF_BF16)
    return FW_EINVAL;
  const int bn = tile_n > 0 ? tile_n : (N >= 256 ? 256 : (N >= 128 ? 128 : 64));
  if (bn != 64 && bn != 128 && bn != 256 && bn != 512) return FW_EINVAL;
  CUtensorMap ta, tb;
  int rc = make_tmap_2d(&ta, A8, 1, M, K, K, 128, 128, true);
  if (!rc) rc = make_tmap_2d(&tb, B8, 1, N, K, K, bn == 512 ? 128 : bn, 128, true);
  if (rc) return rc;
  GemmArgs a;
  a.M = M;
  a.N = N;
  a.K = K;
  a.sa = sa;
  a.sw = sw;
  a.epi.mode = epilogue;
  a.epi.out[0] = out;
  a.epi.ld_out = N;
  a.epi.seg_w = 1 << 30;
  a.epi.bias = reinterpret_cast<const __nv_bfloat16*>(bias);
  if (bn == 512) return gemm_pair_launch(ta, tb, a, reinterpret_cast<cudaStream_t>(stream));
  CUtensorMap to[3];
  rc = make_out_tmaps(a, to);
  if (rc) return rc;
  return gemm_bf16_launch(ta, tb, bn, a, reinterpret_cast<cudaStream_t>(stream), 0, nullptr, to);
}

int fw_ipc_get_handle(const void* ptr, void* handle, size_t* offset) {
  typedef CUresult (*PFN_range)(CUdeviceptr*, size_t*, CUdeviceptr);
  static PFN_range range = nullptr;
  if (!ptr || !handle || !offset) return FW_EINVAL;
  if (!range) {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuMemGetAddressRange", &p, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess)
      return FW_ENODRIVER;
    range = reinterpret_cast<PFN_range>(p);
  }
  CUdeviceptr base = 0;
  size_t size = 0;
  if (range(&base, &size, reinterpret_cast<CUdeviceptr>(ptr)) != CUDA_SUCCESS) return FW_EINVAL;
  cudaIpcMemHandle_t h;
  if (cudaIpcGetMemHandle(&h, reinterpret_cast<void*>(base)) != cudaSuccess) return FW_ECUDA;
  memcpy(handle, &h, sizeof(h));
  *offset = (size_t)(reinterpret_cast<uintptr_t>(ptr) - (uintptr_t)base);
  return 0;
}

int fw_ipc_open(const void* handle, void** ptr) {
  if (!handle || !ptr) return FW_EINVAL;
  cudaIpcMemHandle_t h;
  memcpy(&h, handle, sizeof(h));
  return cudaIpcOpenMemHandle(ptr, h, cudaIpcMemLazyEnablePeerAccess) == cudaSuccess ? 0 : FW_ECUDA;
}

int fw_ipc_close(void* ptr) {
  if (!ptr) return FW_EINVAL;
  return cudaIpcCloseMemHandle(ptr) == cudaSuccess ? 0 : FW_ECUDA;
}

int fw_quant_e4m3(const void* x, int M, int K, void* q, float* scale, void* stream) {
  if (!x || !q || !scale || M <= 0 || K <= 0) return FW_EINVAL;
  return fw::quant_rows(reinterpret_cast<const __nv_bfloat16*>(x), K, M, K, reinterpret_cast<uint8_t*>(q), K, scale,
                        reinterpret_cast<cudaStream_t>(stream));
}

int fw_gemm_bf16_resid(const void* A, const void* B, const void* bias, float* resid, const float* gate,
                       int rows_per_frame, int M, int N, int K, void* stream) {
  using namespace fw;
  if (!A || !B || !resid || rows_per_frame <= 0 || M <= 0 || N <= 0) return FW_EINVAL;
  const int bn = gemm_resid_bn(M, N);
  CUtensorMap ta, tb;
  int rc = make_tmap_2d(&ta, A, 2, M, K, K, 128, 64, true);
  if (!rc) rc = make_tmap_2d(&tb, B, 2, N, K, K, bn, 64, true);
  if (rc) return rc;
  GemmArgs a;
  a.M = M;
  a.N = N;
  a.K = K;
  a.epi.mode = EPI_RESID_F32;
  a.epi.resid = resid;
  a.epi.ld_resid = N;
  a.epi.bias = reinterpret_cast<const __nv_bfloat16*>(bias);
  a.epi.gate = gate;
  a.epi.gate_stride = N;
  a.epi.rows_per_frame = rows_per_frame;
  if (!resid_tma_enabled()) return gemm_bf16_launch(ta, tb, bn, a, reinterpret_cast<cudaStream_t>(stream));
  // the residual is added by TMA reduce-add (EPI_RESID_TMA)
  CUtensorMap tc;
  rc = make_tmap_2d(&tc, resid, 4, M, N, N, 32, 32, true);
  if (rc) return rc;
  a.epi.mode = EPI_RESID_TMA;
  return gemm_bf16_launch(ta, tb, bn, a, reinterpret_cast<cudaStream_t>(stream), 0, &tc);
}

int fw_layernorm(const float* x, int M, int D, float eps, const float* shift, const float* scale, const void* w,
                 const void* b, void* out, void* stream) {
  if (!x || !out || M <= 0 || D <= 0 || (!shift) != (!scale) || (!w) != (!b)) return FW_EINVAL;
  return fw::ln_f32(x, D, M, D, eps, shift, scale, reinterpret_cast<const __nv_bfloat16*>(w),
                    reinterpret_cast<const __nv_bfloat16*>(b), reinterpret_cast<__nv_bfloat16*>(out), D,
                    reinterpret_cast<cudaStream_t>(stream));
}

int fw_rms_rope(const void* x, int M, int D, float eps, const void* w, const float* rope, int head_dim, void* out,
                void* stream) {
  if (!x || !w || !out || M <= 0 || D <= 0 || head_dim <= 0 || D % head_dim) return FW_EINVAL;
  return fw::rms_rope2(reinterpret_cast<const __nv_bfloat16*>(x), reinterpret_cast<const __nv_bfloat16*>(w),
                       reinterpret_cast<__nv_bfloat16*>(out), nullptr, nullptr, nullptr, D, M, D, eps,
                       reinterpret_cast<const float2*>(rope), head_dim, D, reinterpret_cast<cudaStream_t>(stream));
}

int fw_attention(const void* q, int Lq, int heads, const void* k0, const void* v0, int max_keys0, const void* k1,
                 const void* v1, int max_keys1, const int* meta, void* out, int* status, void* stream) {
  using namespace fw;
  if (!q || !k0 || !v0 || !k1 || !v1 || !meta || !out || Lq <= 0 || heads <= 0 || max_keys0 <= 0 || max_keys1 <= 0)
    return FW_EINVAL;
  const int cols = heads * 128;
  CUtensorMap tq, tk0, tv0, tk1, tv1;
  int rc = make_tmap_2d(&tq, q, 2, Lq, cols, cols, 128, 64, true);
  if (!rc) rc = make_tmap_2d(&tk0, k0, 2, max_keys0, cols, cols, 128, 64, true);
  if (!rc) rc = make_tmap_2d(&tv0, v0, 2, max_keys0, cols, cols, 128, 64, true);
  if (!rc) rc = make_tmap_2d(&tk1, k1, 2, max_keys1, cols, cols, 128, 64, true);
  if (!rc) rc = make_tmap_2d(&tv1, v1, 2, max_keys1, cols, cols, 128, 64, true);
  CUtensorMap to;
  if (!rc) rc = make_tmap_2d(&to, out, 2, Lq, cols, cols, 128, 64, true);
  if (rc) return rc;
  AttnArgs a;
  a.Lq = Lq;
  a.heads = heads;
  a.meta = meta;
  a.max_keys0 = max_keys0;
  a.max_keys1 = max_keys1;
  a.out = reinterpret_cast<__nv_bfloat16*>(out);
  a.ld_out = cols;
  a.scale_log2 = (float)(1.4426950408889634 / std::sqrt(128.0));
  a.status = status;
  return attention_launch(tq, tk0, tv0, tk1, tv1, a, reinterpret_cast<cudaStream_t>(stream), &to);
}

}  // extern "C"
