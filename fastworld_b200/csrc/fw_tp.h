// NCCL wrappers for tensor parallelism (tp.cu).  All return 0 or a negative FW_E* code.
#pragma once
#include <cuda_runtime.h>
#include <stddef.h>

namespace fw {

int tp_unique_id(void* id128);
int tp_comm_init(void** comm, const void* id128, int rank, int world);
// In-place sum over the communicator's ranks; dtype FW_BF16 or FW_F32.
int tp_allreduce(void* comm, void* buf, size_t count, int dtype, cudaStream_t s);
void tp_comm_destroy(void* comm);

}  // namespace fw
