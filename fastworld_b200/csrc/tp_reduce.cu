// Tensor-parallel reductions over NVLink peer memory (sm_100a), fused with their epilogues.
//
// With tp_size > 1 the row-parallel linears (sa.o, ca.o, ffn.2) leave a bf16 partial sum
// [L, D] on every rank, and the q/k RMSNorms a per-row partial sum of squares.  Instead of a
// library all-reduce followed by a separate residual kernel, every rank maps the other ranks'
// engine workspaces (CUDA IPC; identical layouts, so a buffer's address on rank j is rank j's
// workspace base + the same offset) and these kernels move the data with plain loads and
// stores over NVLink:
//
// tp_reduce_kernel (two-shot all-reduce + residual epilogue), CTA c of G on every rank:
//   A. signal "my partials are final" (flagA) to every rank, wait for every rank's flagA;
//   1. rows chunk c of this rank's row slice: sum the tp partials (own + remote loads) in
//      fp32, add the bias, round to bf16 and push the result into every rank's `red`
//      buffer (remote stores); fence, signal flagB to every rank;
//   2. wait for every rank's flagB, then for every slice j, rows chunk c of slice j:
//      xs += gate * red (local reads), optional bf16 mirror.
// Every rank computes xs from the same bf16 `red` values with the same arithmetic, so the
// residual stream stays identical on all ranks.
//
// With two ranks tp_reduce2_kernel does the same in one shot (below).
//
// tp_sumsq_kernel (all-gather + local sum of [M, 2] fp32): CTA c pushes rows chunk c of its
// partial sums into every rank's gather slot (double-buffered by epoch parity), signals, waits
// for every rank and sums the slots into `ss`.
//
// Synchronisation: flags are per (source rank, CTA index) monotonically increasing epochs; CTA
// c only waits for CTA c of the other ranks and only reads rows those CTAs wrote, so no grid-
// wide barrier is needed.  Epochs live in this rank's workspace (one counter per CTA, touched
// by that CTA only) and advance by one per call, identically on every rank because every rank
// issues the same call sequence.  Buffer reuse is safe without further barriers: a rank
// reaches flagA of call e only after its call e-1 finished, and its next GEMM overwrites
// `part` only after every rank's phase 1 (the only reader of `part`) signalled flagB.
// Stores of data are ordered before the flag by __syncthreads + a system-scope fence and a
// release store; the waiter uses acquire loads.  Every wait is bounded (FW_WAIT_LIMIT_NS):
// on timeout the CTA records DEV_TIMEOUT_PEER in the status word and carries on without the
// missing data, so no GPU is left spinning.  (The limit is TpPeers::wait_ns; a self-test
// shortens it.)
#include "../../include/fastworld_b200.h"
#include "fw_internal.h"
#include "fw_ptx.cuh"
#include "fw_tp.h"

namespace fw {

namespace {

__device__ __forceinline__ void st_release_sys(unsigned* p, unsigned v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ unsigned ld_acquire_sys(const unsigned* p) {
  unsigned v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// Threads 0..tp-1 each wait until flags[t * TP_MAX_CTAS + c] >= e; then the CTA syncs.
__device__ __forceinline__ void wait_peers(const unsigned* flags, int tp, int c, unsigned e, int* status,
                                           uint64_t limit_ns) {
  const int t = threadIdx.x;
  if (t < tp) {
    const unsigned* f = flags + (size_t)t * TP_MAX_CTAS + c;
    if ((int)(ld_acquire_sys(f) - e) < 0) {
      const uint64_t t0 = globaltimer();
      for (uint32_t i = 1;; ++i) {
        if ((int)(ld_acquire_sys(f) - e) >= 0) break;
        if ((i & 63u) == 0 && globaltimer() - t0 > limit_ns) {
          record_status(status, DEV_TIMEOUT_PEER);
          break;
        }
      }
    }
  }
  __syncthreads();
}

// Thread 0: after the CTA's stores (ordered by the caller's __syncthreads), publish epoch e in
// slot (rank, c) of `off` in every rank's flag area.
__device__ __forceinline__ void signal_peers(const TpPeers& p, size_t off, int c, unsigned e) {
  if (threadIdx.x == 0) {
    __threadfence_system();
    for (int j = 0; j < p.tp; ++j) st_release_sys(p.flags[j] + off + (size_t)p.rank * TP_MAX_CTAS + c, e);
  }
}

__device__ __forceinline__ void add8(float (&a)[8], const uint4& u) {
  const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 f = unpack_bf16(w[i]);
    a[2 * i] += f.x;
    a[2 * i + 1] += f.y;
  }
}

}  // namespace

// One-shot variant for two ranks: each rank reads the other's whole partial (the NVLink load
// per direction equals the two-shot's, without the reduced-sum buffer and its extra pass).
// CTA c: A. signal/await "partials final"; rows chunk c of all L: xs += gate * (part[0] +
// part[1] + bias) in rank order (identical on both ranks); B. signal "done reading your
// partial" and await the same from the other rank before exiting, so neither rank's next GEMM
// overwrites a partial the other is still reading.
__global__ void __launch_bounds__(512) tp_reduce2_kernel(TpPeers p, int L, int D, const __nv_bfloat16* __restrict__ bias,
                                                         const float* __restrict__ gate, float* __restrict__ xs,
                                                         __nv_bfloat16* __restrict__ mirror, int* status) {
  pdl_wait();
  const int c = blockIdx.x, G = gridDim.x, r = p.rank;
  __shared__ unsigned s_e;
  if (threadIdx.x == 0) {
    unsigned* ep = p.epoch + c;
    s_e = *ep + 1u;
    *ep = s_e;
  }
  __syncthreads();
  const unsigned e = s_e;
  const int nv = D / 8;
  signal_peers(p, 0, c, e);
  wait_peers(p.flags[r] + 0, 2, c, e, status, p.wait_ns);
  constexpr int U = 4;
  const int rows_c = (L + G - 1) / G;
  const int r0 = c * rows_c, r1 = min(r0 + rows_c, L);
  const size_t base = (size_t)r0 * D;
  const int n = max(r1 - r0, 0) * nv;
  const uint4* p0 = reinterpret_cast<const uint4*>(p.part[0] + base);
  const uint4* p1 = reinterpret_cast<const uint4*>(p.part[1] + base);
  for (int i0 = threadIdx.x; i0 < n; i0 += U * blockDim.x) {
    uint4 w0[U], w1[U];
    float4 x0[U], x1[U];
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int i = i0 + u * blockDim.x;
      if (i < n) {
        w0[u] = __ldcg(p0 + i);
        w1[u] = __ldcg(p1 + i);
        const float4* xr = reinterpret_cast<const float4*>(xs + base + (size_t)i * 8);
        x0[u] = xr[0];
        x1[u] = xr[1];
      }
    }
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int i = i0 + u * blockDim.x;
      if (i >= n) continue;
      const int col = (i % nv) * 8;
      float v[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
      add8(v, w0[u]);
      add8(v, w1[u]);
      if (bias) add8(v, *reinterpret_cast<const uint4*>(bias + col));
      float4 a0 = x0[u], a1 = x1[u];
      if (gate) {
        const float4 g0 = *reinterpret_cast<const float4*>(gate + col), g1 = *reinterpret_cast<const float4*>(gate + col + 4);
        a0.x += g0.x * v[0]; a0.y += g0.y * v[1]; a0.z += g0.z * v[2]; a0.w += g0.w * v[3];
        a1.x += g1.x * v[4]; a1.y += g1.y * v[5]; a1.z += g1.z * v[6]; a1.w += g1.w * v[7];
      } else {
        a0.x += v[0]; a0.y += v[1]; a0.z += v[2]; a0.w += v[3];
        a1.x += v[4]; a1.y += v[5]; a1.z += v[6]; a1.w += v[7];
      }
      float4* xw = reinterpret_cast<float4*>(xs + base + (size_t)i * 8);
      xw[0] = a0;
      xw[1] = a1;
      if (mirror)
        *reinterpret_cast<uint4*>(mirror + base + (size_t)i * 8) =
            make_uint4(pack_bf16(a0.x, a0.y), pack_bf16(a0.z, a0.w), pack_bf16(a1.x, a1.y), pack_bf16(a1.z, a1.w));
    }
  }
  __syncthreads();
  signal_peers(p, (size_t)TP_MAX_RANKS * TP_MAX_CTAS, c, e);
  wait_peers(p.flags[r] + (size_t)TP_MAX_RANKS * TP_MAX_CTAS, 2, c, e, status, p.wait_ns);
  pdl_trigger();
}

// Two ranks with the transfer folded into the GEMMs: each rank's row-parallel GEMM already
// stored its partial into the other rank's recv[parity] (EPI_BF16_PUSH), so CTA c only signals
// "my GEMM is complete" (its stores into the other GPU were issued by the finished kernel),
// waits for the other rank's signal, and updates rows chunk c of xs from local memory.  recv is
// double-buffered by call parity: the other rank's GEMM of call e+2 writes recv[parity(e)] only
// after its combine of call e+1, which waits for this rank's signal of call e+1, given after
// this rank's combine of call e finished reading.
__global__ void __launch_bounds__(512) tp_combine2_kernel(TpPeers p, const __nv_bfloat16* __restrict__ own_part,
                                                          const __nv_bfloat16* __restrict__ recv, int L, int D,
                                                          const __nv_bfloat16* __restrict__ bias,
                                                          const float* __restrict__ gate, float* __restrict__ xs,
                                                          __nv_bfloat16* __restrict__ mirror, int* status) {
  pdl_wait();
  const int c = blockIdx.x, G = gridDim.x, r = p.rank;
  __shared__ unsigned s_e;
  if (threadIdx.x == 0) {
    unsigned* ep = p.epoch + c;
    s_e = *ep + 1u;
    *ep = s_e;
  }
  __syncthreads();
  const unsigned e = s_e;
  signal_peers(p, 0, c, e);
  wait_peers(p.flags[r] + 0, 2, c, e, status, p.wait_ns);
  const int nv = D / 8;
  constexpr int U = 4;
  const int rows_c = (L + G - 1) / G;
  const int r0 = c * rows_c, r1 = min(r0 + rows_c, L);
  const size_t base = (size_t)r0 * D;
  const int n = max(r1 - r0, 0) * nv;
  // rank order: part of rank 0 first
  const uint4* p0 = reinterpret_cast<const uint4*>((r == 0 ? own_part : recv) + base);
  const uint4* p1 = reinterpret_cast<const uint4*>((r == 0 ? recv : own_part) + base);
  for (int i0 = threadIdx.x; i0 < n; i0 += U * blockDim.x) {
    uint4 w0[U], w1[U];
    float4 x0[U], x1[U];
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int i = i0 + u * blockDim.x;
      if (i < n) {
        w0[u] = __ldcg(p0 + i);
        w1[u] = __ldcg(p1 + i);
        const float4* xr = reinterpret_cast<const float4*>(xs + base + (size_t)i * 8);
        x0[u] = xr[0];
        x1[u] = xr[1];
      }
    }
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int i = i0 + u * blockDim.x;
      if (i >= n) continue;
      const int col = (i % nv) * 8;
      float v[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
      add8(v, w0[u]);
      add8(v, w1[u]);
      if (bias) add8(v, *reinterpret_cast<const uint4*>(bias + col));
      float4 a0 = x0[u], a1 = x1[u];
      if (gate) {
        const float4 g0 = *reinterpret_cast<const float4*>(gate + col), g1 = *reinterpret_cast<const float4*>(gate + col + 4);
        a0.x += g0.x * v[0]; a0.y += g0.y * v[1]; a0.z += g0.z * v[2]; a0.w += g0.w * v[3];
        a1.x += g1.x * v[4]; a1.y += g1.y * v[5]; a1.z += g1.z * v[6]; a1.w += g1.w * v[7];
      } else {
        a0.x += v[0]; a0.y += v[1]; a0.z += v[2]; a0.w += v[3];
        a1.x += v[4]; a1.y += v[5]; a1.z += v[6]; a1.w += v[7];
      }
      float4* xw = reinterpret_cast<float4*>(xs + base + (size_t)i * 8);
      xw[0] = a0;
      xw[1] = a1;
      if (mirror)
        *reinterpret_cast<uint4*>(mirror + base + (size_t)i * 8) =
            make_uint4(pack_bf16(a0.x, a0.y), pack_bf16(a0.z, a0.w), pack_bf16(a1.x, a1.y), pack_bf16(a1.z, a1.w));
    }
  }
  pdl_trigger();
}

// recv != null: the row-parallel GEMMs already pushed every rank's partial rows of this rank's
// slice into recv (slot j = rank j's rows, [tp][slice][D], EPI_BF16_PUSH with push_tp > 2), so
// phase 1 reads local memory only; this rank's own partial is p.part[rank].
template <int TP>
__global__ void __launch_bounds__(512) tp_reduce_kernel(TpPeers p, int L, int D, const __nv_bfloat16* __restrict__ bias,
                                                        const float* __restrict__ gate, float* __restrict__ xs,
                                                        __nv_bfloat16* __restrict__ mirror, int* status,
                                                        const __nv_bfloat16* __restrict__ recv) {
  pdl_wait();
  const int c = blockIdx.x, G = gridDim.x, tp = TP, r = p.rank;
  __shared__ unsigned s_e;
  if (threadIdx.x == 0) {
    unsigned* ep = p.epoch + c;
    s_e = *ep + 1u;
    *ep = s_e;
  }
  __syncthreads();
  const unsigned e = s_e;
  const int slice = (L + tp - 1) / tp;
  const int rows_c = (slice + G - 1) / G;
  const int nv = D / 8;                       // 16-byte vectors per row
  // A: partials are final on this rank (the GEMM that wrote them completed before this kernel)
  signal_peers(p, 0, c, e);
  wait_peers(p.flags[r] + 0, tp, c, e, status, p.wait_ns);
  // 1: reduce rows chunk c of slice r, push bf16(sum + bias) to every rank.  U vectors of each
  // of the TP partials per thread per step (8 loads), all issued before any use so the NVLink
  // latency overlaps.
  constexpr int U = TP >= 8 ? 1 : 8 / TP;
  {
    const int r0 = r * slice + c * rows_c;
    const int r1 = min(min(r0 + rows_c, (r + 1) * slice), L);
    const size_t base = (size_t)r0 * D;
    const int n = max(r1 - r0, 0) * nv;
    for (int i0 = threadIdx.x; i0 < n; i0 += U * blockDim.x) {
      float a[U][8];
      uint4 w[TP][U];
#pragma unroll
      for (int j = 0; j < TP; ++j) {
        const __nv_bfloat16* src =
            (recv && j != r) ? recv + ((size_t)j * slice + (r0 - r * slice)) * D : p.part[j] + base;
#pragma unroll
        for (int u = 0; u < U; ++u) {
          const int i = i0 + u * blockDim.x;
          w[j][u] = i < n ? __ldcg(reinterpret_cast<const uint4*>(src) + i) : make_uint4(0, 0, 0, 0);
        }
      }
#pragma unroll
      for (int u = 0; u < U; ++u) {
#pragma unroll
        for (int k = 0; k < 8; ++k) a[u][k] = 0.f;
#pragma unroll
        for (int j = 0; j < TP; ++j) add8(a[u], w[j][u]);
      }
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const int i = i0 + u * blockDim.x;
        if (i >= n) continue;
        if (bias) add8(a[u], *reinterpret_cast<const uint4*>(bias + (size_t)(i % nv) * 8));
        const uint4 o = make_uint4(pack_bf16(a[u][0], a[u][1]), pack_bf16(a[u][2], a[u][3]),
                                   pack_bf16(a[u][4], a[u][5]), pack_bf16(a[u][6], a[u][7]));
#pragma unroll
        for (int j = 0; j < TP; ++j) reinterpret_cast<uint4*>(p.red[j] + base)[i] = o;
      }
    }
  }
  __syncthreads();
  signal_peers(p, (size_t)TP_MAX_RANKS * TP_MAX_CTAS, c, e);
  wait_peers(p.flags[r] + (size_t)TP_MAX_RANKS * TP_MAX_CTAS, tp, c, e, status, p.wait_ns);
  // 2: residual update of rows chunk c of every slice from the local `red`
  constexpr int U2 = 4;
  const __nv_bfloat16* red = p.red[r];
  for (int j = 0; j < tp; ++j) {
    const int r0 = j * slice + c * rows_c;
    const int r1 = min(min(r0 + rows_c, (j + 1) * slice), L);
    const int n = max(r1 - r0, 0) * nv;
    for (int i0 = threadIdx.x; i0 < n; i0 += U2 * blockDim.x) {
      uint4 w[U2];
      float4 x0[U2], x1[U2];
#pragma unroll
      for (int u = 0; u < U2; ++u) {
        const int i = i0 + u * blockDim.x;
        if (i < n) {
          const size_t e8 = (size_t)r0 * D + (size_t)i * 8;
          w[u] = __ldcg(reinterpret_cast<const uint4*>(red + e8));
          const float4* xr = reinterpret_cast<const float4*>(xs + e8);
          x0[u] = xr[0];
          x1[u] = xr[1];
        }
      }
#pragma unroll
      for (int u = 0; u < U2; ++u) {
        const int i = i0 + u * blockDim.x;
        if (i >= n) continue;
        const int col = (i % nv) * 8;
        const size_t e8 = (size_t)r0 * D + (size_t)i * 8;
        float v[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
        add8(v, w[u]);
        float4 a0 = x0[u], a1 = x1[u];
        if (gate) {
          const float4 g0 = *reinterpret_cast<const float4*>(gate + col), g1 = *reinterpret_cast<const float4*>(gate + col + 4);
          a0.x += g0.x * v[0]; a0.y += g0.y * v[1]; a0.z += g0.z * v[2]; a0.w += g0.w * v[3];
          a1.x += g1.x * v[4]; a1.y += g1.y * v[5]; a1.z += g1.z * v[6]; a1.w += g1.w * v[7];
        } else {
          a0.x += v[0]; a0.y += v[1]; a0.z += v[2]; a0.w += v[3];
          a1.x += v[4]; a1.y += v[5]; a1.z += v[6]; a1.w += v[7];
        }
        float4* xw = reinterpret_cast<float4*>(xs + e8);
        xw[0] = a0;
        xw[1] = a1;
        if (mirror)
          *reinterpret_cast<uint4*>(mirror + e8) =
              make_uint4(pack_bf16(a0.x, a0.y), pack_bf16(a0.z, a0.w), pack_bf16(a1.x, a1.y), pack_bf16(a1.z, a1.w));
      }
    }
  }
  pdl_trigger();
}

__global__ void __launch_bounds__(256) tp_sumsq_kernel(TpPeers p, float* __restrict__ ss, int M, int* status) {
  pdl_wait();
  const int c = blockIdx.x, G = gridDim.x, tp = p.tp, r = p.rank;
  __shared__ unsigned s_e;
  if (threadIdx.x == 0) {
    unsigned* ep = p.epoch + TP_MAX_CTAS + c;
    s_e = *ep + 1u;
    *ep = s_e;
  }
  __syncthreads();
  const unsigned e = s_e;
  const int rows_c = (M + G - 1) / G;
  const int r0 = c * rows_c, r1 = min(r0 + rows_c, M);
  const int n = max(r1 - r0, 0) * 2;
  const size_t slot = (size_t)p.gat_rows * 2;                     // floats per (parity, rank) slot
  const size_t par = (size_t)(e & 1u) * TP_MAX_RANKS * slot;
  for (int i = threadIdx.x; i < n; i += blockDim.x) {
    const float v = ss[(size_t)r0 * 2 + i];
    for (int j = 0; j < tp; ++j) p.gat[j][par + (size_t)r * slot + (size_t)r0 * 2 + i] = v;
  }
  __syncthreads();
  const size_t foff = (size_t)2 * TP_MAX_RANKS * TP_MAX_CTAS;
  signal_peers(p, foff, c, e);
  wait_peers(p.flags[r] + foff, tp, c, e, status, p.wait_ns);
  const float* g = p.gat[r] + par;
  for (int i = threadIdx.x; i < n; i += blockDim.x) {
    float s = 0.f;
    for (int j = 0; j < tp; ++j) s += g[(size_t)j * slot + (size_t)r0 * 2 + i];
    ss[(size_t)r0 * 2 + i] = s;
  }
  pdl_trigger();
}

static int tp_grid() { return num_sms() < TP_MAX_CTAS ? num_sms() : TP_MAX_CTAS; }

int tp_reduce(const TpPeers& p, int L, int D, const __nv_bfloat16* bias, const float* gate, float* xs,
              __nv_bfloat16* mirror, int* status, cudaStream_t s, const __nv_bfloat16* recv) {
  if (D % 8) return FW_EINVAL;
  switch (p.tp) {
    case 2: launch_k(tp_reduce2_kernel, tp_grid(), 512, 0, s, p, L, D, bias, gate, xs, mirror, status); break;
    case 4: launch_k(tp_reduce_kernel<4>, tp_grid(), 512, 0, s, p, L, D, bias, gate, xs, mirror, status, recv); break;
    case 8: launch_k(tp_reduce_kernel<8>, tp_grid(), 512, 0, s, p, L, D, bias, gate, xs, mirror, status, recv); break;
    default: return FW_EINVAL;
  }
  return cudaGetLastError() == cudaSuccess ? 0 : FW_ECUDA;
}

int tp_combine2(const TpPeers& p, int parity, const __nv_bfloat16* own_part, int L, int D,
                const __nv_bfloat16* bias, const float* gate, float* xs, __nv_bfloat16* mirror, int* status,
                cudaStream_t s) {
  if (p.tp != 2 || !p.recv[p.rank] || D % 8 || (parity & ~1)) return FW_EINVAL;
  const __nv_bfloat16* recv = p.recv[p.rank] + (size_t)parity * L * D;
  launch_k(tp_combine2_kernel, tp_grid(), 512, 0, s, p, own_part, recv, L, D, bias, gate, xs, mirror, status);
  return cudaGetLastError() == cudaSuccess ? 0 : FW_ECUDA;
}

int tp_sumsq(const TpPeers& p, float* ss, int M, int* status, cudaStream_t s) {
  if (p.tp < 2 || p.tp > TP_MAX_RANKS || M > p.gat_rows) return FW_EINVAL;
  launch_k(tp_sumsq_kernel, tp_grid(), 256, 0, s, p, ss, M, status);
  return cudaGetLastError() == cudaSuccess ? 0 : FW_ECUDA;
}

}  // namespace fw
