// Failure-path self-tests on one GPU: bounded waits that nothing satisfies must run out,
// record their code in the status word, unwind and leave the context usable.
//
//   which 0 (mbarrier): each CTA allocates TMEM, then one thread waits on an mbarrier that no
//     thread or copy ever completes (the wait every warp role of the GEMM and attention kernels
//     uses, fw_ptx.cuh mbar_wait).  It gives up after `limit_ns`, records DEV_TIMEOUT_TEST and
//     raises the CTA's abort flag; a second waiter of the same CTA sees the flag and leaves
//     without waiting out its own limit; the CTA frees its TMEM and exits.
//   which 1 (peer flag): the real two-rank reduction kernel (tp_reduce2_kernel) runs as rank 0
//     of a two-rank group whose "rank 1" buffers are this GPU's own memory and which nobody
//     plays: both of its waits for rank 1's epoch flags run out after `limit_ns`, record
//     DEV_TIMEOUT_PEER, and the kernel completes without the missing data.
// Nothing here faults: every access is in the buffers the host carves from `scratch`.
#include "../../include/fastworld_b200.h"
#include "fw_internal.h"
#include "fw_ptx.cuh"
#include "fw_tp.h"

namespace fw {

namespace {

constexpr int kSelfTestCtas = 4;
constexpr int kPeerRows = 64, kPeerCols = 256;

__global__ void __launch_bounds__(128) mbar_timeout_kernel(uint64_t limit_ns, int* status, int* outcome) {
  pdl_wait();
  __shared__ __align__(8) uint64_t bar;
  __shared__ uint32_t tmem_base;
  __shared__ int abort_flag;
  const int warp = threadIdx.x / 32;
  if (warp == 0) {
    tmem_alloc(&tmem_base, 32);
    tmem_relinquish();
  }
  if (threadIdx.x == 32) {
    mbar_init(&bar, 1);   // one arrival expected; none ever comes
    fence_mbar_init();
    abort_flag = 0;
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  int ok = -1;
  if (threadIdx.x == 64)   // the first waiter runs out after limit_ns
    ok = mbar_wait(&bar, 0, &abort_flag, status, DEV_TIMEOUT_TEST, limit_ns);
  if (threadIdx.x == 96)   // the second gives up once the CTA's abort flag is raised (bounded by 2 limits)
    ok = mbar_wait(&bar, 0, &abort_flag, status, DEV_TIMEOUT_TEST, 2 * limit_ns);
  if (ok >= 0) outcome[blockIdx.x * 2 + (threadIdx.x == 96)] = ok ? 1 : 2;
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tmem_base, 32);
  }
}

struct PeerScratch {
  size_t part, flags, epoch, xs, end;
};

PeerScratch peer_layout() {
  PeerScratch l;
  const size_t part_b = (size_t)kPeerRows * kPeerCols * 2;
  const size_t flag_b = (size_t)3 * TP_MAX_RANKS * TP_MAX_CTAS * 4;
  l.part = 0;                       // 2 x [rows, cols] bf16 partials
  l.flags = l.part + 2 * part_b;    // 2 x [3][TP_MAX_RANKS][TP_MAX_CTAS] epoch flags
  l.epoch = l.flags + 2 * flag_b;   // [2][TP_MAX_CTAS] call counters
  l.xs = l.epoch + 2 * TP_MAX_CTAS * 4;
  l.end = l.xs + (size_t)kPeerRows * kPeerCols * 4;   // [rows, cols] fp32 residual
  return l;
}

}  // namespace

}  // namespace fw

extern "C" size_t fw_selftest_bytes(int which) {
  if (which == 0) return fw::kSelfTestCtas * 2 * sizeof(int);
  if (which == 1) return fw::peer_layout().end;
  return 0;
}

extern "C" int fw_selftest_wait(int which, unsigned long long limit_ns, void* scratch, size_t bytes, int* status,
                                void* stream) {
  using namespace fw;
  if (!scratch || !status || limit_ns == 0 || limit_ns > FW_WAIT_LIMIT_NS) return FW_EINVAL;
  if (bytes < fw_selftest_bytes(which) || fw_selftest_bytes(which) == 0) return FW_ESIZE;
  if (reinterpret_cast<uintptr_t>(scratch) & 255u) return FW_EALIGN;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  if (which == 0) {
    launch_k(mbar_timeout_kernel, kSelfTestCtas, 128, 0, s, (uint64_t)limit_ns, status,
             reinterpret_cast<int*>(scratch));
    return cudaGetLastError() == cudaSuccess ? 0 : FW_ECUDA;
  }
  // which == 1: rank 0 of a two-rank group whose other rank never runs (scratch zeroed by the caller)
  uint8_t* base = static_cast<uint8_t*>(scratch);
  const PeerScratch l = peer_layout();
  const size_t part_b = (size_t)kPeerRows * kPeerCols * 2;
  const size_t flag_b = (size_t)3 * TP_MAX_RANKS * TP_MAX_CTAS * 4;
  TpPeers p;
  p.tp = 2;
  p.rank = 0;
  for (int j = 0; j < 2; ++j) {
    p.part[j] = reinterpret_cast<const __nv_bfloat16*>(base + l.part + j * part_b);
    p.flags[j] = reinterpret_cast<unsigned*>(base + l.flags + j * flag_b);
  }
  p.epoch = reinterpret_cast<unsigned*>(base + l.epoch);
  p.wait_ns = limit_ns;
  return tp_reduce(p, kPeerRows, kPeerCols, nullptr, nullptr, reinterpret_cast<float*>(base + l.xs), nullptr, status,
                   s);
}
