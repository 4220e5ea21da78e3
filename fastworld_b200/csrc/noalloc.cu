// An e4m3 linear layer that needs no device allocation from its caller.
//
// The regular path (fw_quant_e4m3 + fw_gemm_e4m3, and the engine's block linears) quantises the
// bf16 activations per token into scratch memory that the caller allocates, then runs the e4m3
// tensor-core GEMM on that copy.  Some callers cannot provide that scratch: a host that embeds
// this library into a process whose device memory is entirely owned by another framework's
// pool, or a latency-critical loop where calling cudaMalloc (which can synchronise the device)
// is not acceptable.  fw_linear_e4m3_noalloc keeps the quantised copy in a fixed array that is
// part of the library image instead: every GPU that loads the library holds it until the
// process exits, and the entry point itself never allocates or frees device memory.
#include <mutex>

#include "../../include/fastworld_b200.h"
#include "fw_elem.h"
#include "fw_internal.h"

namespace fw {

// Upper bounds of one call: M * K bytes of e4m3 activations and M per-row scales.
constexpr size_t kNoAllocActBytes = size_t(32) << 20;   // 32 MiB
constexpr int kNoAllocMaxRows = 16384;

static __device__ __align__(256) uint8_t g_noalloc_act[kNoAllocActBytes];
static __device__ __align__(256) float g_noalloc_scale[kNoAllocMaxRows];

// Host code may not pass the array names to a kernel (on the host they only stand for the
// symbols): the device addresses are looked up with cudaGetSymbolAddress, once per CUDA
// context (a device's primary context, or a context that a host framework created and made
// current), and cached under that context.  A context created later on the same device (for
// instance after a device reset) misses the cache and gets its own lookup.
typedef CUresult (*PFN_ctxGetCurrent)(CUcontext*);

static CUcontext current_context() {
  static PFN_ctxGetCurrent fn = [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &p, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess)
      return static_cast<PFN_ctxGetCurrent>(nullptr);
    return reinterpret_cast<PFN_ctxGetCurrent>(p);
  }();
  CUcontext c = nullptr;
  if (fn && fn(&c) != CUDA_SUCCESS) c = nullptr;
  return c;
}

struct NoAllocScratch {
  CUcontext ctx;
  void* act;
  float* scale;
};
static std::mutex g_noalloc_mu;
static NoAllocScratch g_noalloc[64];
static int g_noalloc_n = 0;

static int noalloc_scratch(void** act, float** scale) {
  std::lock_guard<std::mutex> lock(g_noalloc_mu);
  CUcontext ctx = current_context();
  for (int i = 0; ctx && i < g_noalloc_n; ++i)
    if (g_noalloc[i].ctx == ctx) {
      *act = g_noalloc[i].act;
      *scale = g_noalloc[i].scale;
      return 0;
    }
  // set-up for this context: look the arrays up with the caller's device current (the lookup
  // also binds the device's primary context when the thread had none)
  void* a = nullptr;
  void* s = nullptr;
  if (cudaGetSymbolAddress(&a, g_noalloc_act) != cudaSuccess) return FW_ECUDA;
  if (cudaGetSymbolAddress(&s, g_noalloc_scale) != cudaSuccess) return FW_ECUDA;
  if (!ctx) ctx = current_context();
  if (ctx && g_noalloc_n < 64) g_noalloc[g_noalloc_n++] = {ctx, a, reinterpret_cast<float*>(s)};
  *act = a;
  *scale = reinterpret_cast<float*>(s);
  return 0;
}

}  // namespace fw

extern "C" int fw_linear_e4m3_noalloc(const void* x, const void* w8, const float* sw, const void* bias, void* out,
                                      int M, int N, int K, void* stream) {
  using namespace fw;
  if (!x || !w8 || !sw || !out || M <= 0 || N <= 0 || K <= 0) return FW_EINVAL;
  if ((size_t)M * (size_t)K > kNoAllocActBytes || M > kNoAllocMaxRows) return FW_ESCRATCH;
  if (K % 16) return FW_ESHAPE;
  // Every check that the GEMM launch makes runs before the quantisation, so a rejected call
  // launches nothing and leaves the shared array as it was.  (Looking the array's address up
  // reads no device memory.)
  void* act = nullptr;
  float* scale = nullptr;
  int rc = noalloc_scratch(&act, &scale);
  if (rc) return rc;
  const int bn = N >= 256 ? 256 : (N >= 128 ? 128 : 64);
  GemmArgs a;
  a.M = M;
  a.N = N;
  a.K = K;
  a.sa = scale;
  a.sw = sw;
  a.epi.mode = EPI_BF16;
  a.epi.out[0] = out;
  a.epi.ld_out = N;
  a.epi.seg_w = 1 << 30;
  a.epi.bias = reinterpret_cast<const __nv_bfloat16*>(bias);
  rc = gemm_check(a, bn);
  if (rc) return rc;
  if (reinterpret_cast<uintptr_t>(x) & 15u) return FW_EALIGN;
  CUtensorMap ta, tb;
  rc = make_tmap_2d(&ta, act, 1, M, K, K, 128, 128, true);
  if (!rc) rc = make_tmap_2d(&tb, w8, 1, N, K, K, bn, 128, true);
  if (rc) return rc;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  // every byte of the scratch this call reads is written first: no clearing is needed
  rc = quant_rows(reinterpret_cast<const __nv_bfloat16*>(x), K, M, K, reinterpret_cast<uint8_t*>(act), K, scale, s);
  if (rc) return rc;
  return gemm_bf16_launch(ta, tb, bn, a, s);
}
