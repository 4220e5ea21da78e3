// Tensor parallelism: NCCL wrappers (tp.cu) and the peer-memory reductions (tp_reduce.cu).
// All functions return 0 or a negative FW_E* code.
#pragma once
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stddef.h>

namespace fw {

int tp_unique_id(void* id128);
int tp_comm_init(void** comm, const void* id128, int rank, int world);
// In-place sum over the communicator's ranks; dtype FW_BF16 or FW_F32.
int tp_allreduce(void* comm, void* buf, size_t count, int dtype, cudaStream_t s);
void tp_comm_destroy(void* comm);

constexpr int TP_MAX_RANKS = 8;
constexpr int TP_MAX_CTAS = 160;   // >= SMs per GPU; CTA c of every rank pairs with CTA c of the others

// Every rank's buffers as seen from this rank (index = rank; own rank = local pointers, the
// others mapped peer memory).
struct TpPeers {
  int tp = 0, rank = 0;
  int gat_rows = 0;                              // rows per gather slot (>= every M of tp_sumsq)
  const __nv_bfloat16* part[TP_MAX_RANKS] = {};  // [L, D] bf16 partial sums of a row-parallel linear
  __nv_bfloat16* red[TP_MAX_RANKS] = {};         // [L, D] bf16 reduced sums (+ bias)
  unsigned* flags[TP_MAX_RANKS] = {};            // [3][TP_MAX_RANKS][TP_MAX_CTAS] epochs
  float* gat[TP_MAX_RANKS] = {};                 // [2][TP_MAX_RANKS][gat_rows][2] gathered sums of squares
  __nv_bfloat16* recv[TP_MAX_RANKS] = {};        // [2 parities] x (2 ranks: [L, D]; more: [tp][ceil(L/tp)][D]) pushed partials
  unsigned* epoch = nullptr;                     // this rank's [2][TP_MAX_CTAS] call counters
  unsigned long long wait_ns = 2000000000ull;    // bound of every wait on another rank's flag (2 s)
};

// xs[L, D] += gate * (sum over ranks of part + bias) on every rank (two-shot over NVLink);
// mirror (optional) = bf16 copy of the new xs.  gate: one [D] row for all tokens, or null.
// recv (4 or 8 ranks, optional): this rank's receive buffer holding the other ranks' partial
// rows of its slice, pushed by their GEMMs ([tp][ceil(L / tp)][D]); phase 1 then reads locally.
int tp_reduce(const TpPeers& p, int L, int D, const __nv_bfloat16* bias, const float* gate, float* xs,
              __nv_bfloat16* mirror, int* status, cudaStream_t s, const __nv_bfloat16* recv = nullptr);
// Two ranks, after row-parallel GEMMs that pushed their partial sums into the other rank's
// recv[parity] (EPI_BF16_PUSH): xs += gate * (part[0] + part[1] + bias) from local memory only,
// the partials summed in rank order (identical on both ranks).
int tp_combine2(const TpPeers& p, int parity, const __nv_bfloat16* own_part, int L, int D,
                const __nv_bfloat16* bias, const float* gate, float* xs, __nv_bfloat16* mirror, int* status,
                cudaStream_t s);
// ss[M, 2] (fp32, in place) = sum over ranks of ss.
int tp_sumsq(const TpPeers& p, float* ss, int M, int* status, cudaStream_t s);

}  // namespace fw
