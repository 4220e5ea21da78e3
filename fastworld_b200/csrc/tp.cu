// NCCL for tensor parallelism, loaded at run time.
//
// The library does not link against NCCL: fw_tp_* resolve the handful of entry points they
// need from libnccl.so.2 with dlopen.  In a PyTorch process that is the NCCL build torch
// already loaded (RTLD_NOLOAD finds it), so one NCCL runs in the process; a C host gets the
// system library.  Types and enum values are those of nccl.h (stable across NCCL 2.x).
#include <dlfcn.h>
#include <nccl.h>

#include <cstring>
#include <mutex>

#include "../../include/fastworld_b200.h"
#include "fw_tp.h"

namespace fw {

namespace {
struct NcclApi {
  ncclResult_t (*get_unique_id)(ncclUniqueId*) = nullptr;
  ncclResult_t (*comm_init_rank)(ncclComm_t*, int, ncclUniqueId, int) = nullptr;
  ncclResult_t (*all_reduce)(const void*, void*, size_t, ncclDataType_t, ncclRedOp_t, ncclComm_t,
                             cudaStream_t) = nullptr;
  ncclResult_t (*comm_destroy)(ncclComm_t) = nullptr;
  bool ok = false;
};

const NcclApi& nccl() {
  static NcclApi api;
  static std::once_flag once;
  std::call_once(once, [] {
    void* lib = dlopen("libnccl.so.2", RTLD_NOW | RTLD_NOLOAD);
    if (!lib) lib = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
    if (!lib) return;
    api.get_unique_id = reinterpret_cast<decltype(api.get_unique_id)>(dlsym(lib, "ncclGetUniqueId"));
    api.comm_init_rank = reinterpret_cast<decltype(api.comm_init_rank)>(dlsym(lib, "ncclCommInitRank"));
    api.all_reduce = reinterpret_cast<decltype(api.all_reduce)>(dlsym(lib, "ncclAllReduce"));
    api.comm_destroy = reinterpret_cast<decltype(api.comm_destroy)>(dlsym(lib, "ncclCommDestroy"));
    api.ok = api.get_unique_id && api.comm_init_rank && api.all_reduce && api.comm_destroy;
  });
  return api;
}
}  // namespace

int tp_unique_id(void* id128) {
  if (!id128) return FW_EINVAL;
  const NcclApi& n = nccl();
  if (!n.ok) return FW_ENCCL;
  ncclUniqueId id;
  if (n.get_unique_id(&id) != ncclSuccess) return FW_ENCCL;
  memcpy(id128, id.internal, sizeof(id.internal));
  return 0;
}

int tp_comm_init(void** comm, const void* id128, int rank, int world) {
  if (!comm || !id128 || world < 1 || rank < 0 || rank >= world) return FW_EINVAL;
  const NcclApi& n = nccl();
  if (!n.ok) return FW_ENCCL;
  ncclUniqueId id;
  memcpy(id.internal, id128, sizeof(id.internal));
  ncclComm_t c = nullptr;
  if (n.comm_init_rank(&c, world, id, rank) != ncclSuccess) return FW_ENCCL;
  *comm = c;
  return 0;
}

int tp_allreduce(void* comm, void* buf, size_t count, int dtype, cudaStream_t s) {
  if (!comm || !buf) return FW_EINVAL;
  if (count == 0) return 0;
  const NcclApi& n = nccl();
  if (!n.ok) return FW_ENCCL;
  ncclDataType_t t;
  if (dtype == FW_BF16)
    t = ncclBfloat16;
  else if (dtype == FW_F32)
    t = ncclFloat32;
  else
    return FW_EINVAL;
  return n.all_reduce(buf, buf, count, t, ncclSum, reinterpret_cast<ncclComm_t>(comm), s) == ncclSuccess ? 0
                                                                                                        : FW_ENCCL;
}

void tp_comm_destroy(void* comm) {
  if (!comm) return;
  const NcclApi& n = nccl();
  if (n.ok) n.comm_destroy(reinterpret_cast<ncclComm_t>(comm));
}

}  // namespace fw
