// NCCL for tensor-parallel contexts, loaded at run time (dlopen), so the
// library itself needs no NCCL unless a tensor-parallel context is made.
// Tries the NCCL that ships with the Python environment's CUDA wheels, then
// the system one.
#include "tp.h"

#include <dlfcn.h>
#include <stdlib.h>
#include <string.h>

#include <mutex>
#include <string>

namespace myos {
namespace {

struct Nccl {
  void* lib = nullptr;
  ncclResult_t (*get_unique_id)(ncclUniqueId*) = nullptr;
  ncclResult_t (*comm_init_rank)(ncclComm_t*, int, ncclUniqueId, int) = nullptr;
  ncclResult_t (*comm_destroy)(ncclComm_t) = nullptr;
  ncclResult_t (*all_reduce)(const void*, void*, size_t, ncclDataType_t, ncclRedOp_t, ncclComm_t,
                             cudaStream_t) = nullptr;
  ncclResult_t (*all_gather)(const void*, void*, size_t, ncclDataType_t, ncclComm_t,
                             cudaStream_t) = nullptr;
  const char* (*error_string)(ncclResult_t) = nullptr;
  std::string why;
};

Nccl& nccl() {
  static Nccl n;
  static std::once_flag once;
  std::call_once(once, [] {
    const char* names[] = {getenv("MYOS_NCCL_LIB"), "libnccl.so.2", "libnccl.so"};
    for (const char* name : names) {
      if (!name || !*name) continue;
      n.lib = dlopen(name, RTLD_NOW | RTLD_GLOBAL);
      if (n.lib) break;
    }
    if (!n.lib) {
      n.why = "libnccl.so.2 not found (set MYOS_NCCL_LIB)";
      return;
    }
    n.get_unique_id = (decltype(n.get_unique_id))dlsym(n.lib, "ncclGetUniqueId");
    n.comm_init_rank = (decltype(n.comm_init_rank))dlsym(n.lib, "ncclCommInitRank");
    n.comm_destroy = (decltype(n.comm_destroy))dlsym(n.lib, "ncclCommDestroy");
    n.all_reduce = (decltype(n.all_reduce))dlsym(n.lib, "ncclAllReduce");
    n.all_gather = (decltype(n.all_gather))dlsym(n.lib, "ncclAllGather");
    n.error_string = (decltype(n.error_string))dlsym(n.lib, "ncclGetErrorString");
    if (!n.get_unique_id || !n.comm_init_rank || !n.comm_destroy || !n.all_reduce ||
        !n.all_gather || !n.error_string) {
      n.why = "libnccl lacks a needed symbol";
      n.lib = nullptr;
    }
  });
  return n;
}

std::string say(ncclResult_t r) {
  Nccl& n = nccl();
  return n.error_string ? n.error_string(r) : "nccl error";
}

}  // namespace

bool tp_unique_id(uint8_t out[128], std::string* why) {
  Nccl& n = nccl();
  if (!n.lib) {
    *why = n.why;
    return false;
  }
  ncclUniqueId id;
  const ncclResult_t r = n.get_unique_id(&id);
  if (r != ncclSuccess) {
    *why = say(r);
    return false;
  }
  memcpy(out, id.internal, sizeof id.internal);
  return true;
}

bool tp_comm_init(ncclComm_t* comm, int size, int rank, const uint8_t id_bytes[128],
                  std::string* why) {
  Nccl& n = nccl();
  if (!n.lib) {
    *why = n.why;
    return false;
  }
  ncclUniqueId id;
  memcpy(id.internal, id_bytes, sizeof id.internal);
  const ncclResult_t r = n.comm_init_rank(comm, size, id, rank);
  if (r != ncclSuccess) {
    *why = say(r);
    return false;
  }
  return true;
}

void tp_comm_destroy(ncclComm_t comm) {
  if (comm && nccl().lib) nccl().comm_destroy(comm);
}

bool tp_allreduce_sum(const float* in, float* out, size_t n, ncclComm_t comm, cudaStream_t st) {
  return nccl().all_reduce(in, out, n, ncclFloat32, ncclSum, comm, st) == ncclSuccess;
}

bool tp_allgather(const void* in, void* out, size_t bytes, ncclComm_t comm, cudaStream_t st) {
  return nccl().all_gather(in, out, bytes, ncclUint8, comm, st) == ncclSuccess;
}

}  // namespace myos
