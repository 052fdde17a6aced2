// comm.cuh — a library-owned NCCL communicator for the collective route of
// the sequence-sharded decode: every rank's packed (m, l, o) shard partial is
// all-gathered, then pu_decode_combine merges them.  This replaces the
// gather the reference leaves to `jax.lax.psum` / documents as the split-KV
// merge (README.md:41-46; distributed/collectives.py), for callers (a JAX FFI
// handler, a C runtime) that have no communicator of their own.
//
// NCCL is loaded at the first call with dlopen("libnccl.so.2"), taking the
// copy the process has already loaded (torch's, for instance) when there is
// one, so the library has no link-time dependency on NCCL and loads on hosts
// without it; the entry points then return PU_ERR_UNSUPPORTED.
#pragma once

#include <dlfcn.h>
#include <nccl.h>

#include <cstring>
#include <mutex>

#include "pu_host.cuh"

namespace pu {
namespace comm {

static_assert(sizeof(ncclUniqueId) == PU_COMM_ID_BYTES, "NCCL unique id size");

struct Api {
  decltype(&ncclGetUniqueId) get_unique_id = nullptr;
  decltype(&ncclCommInitRank) init_rank = nullptr;
  decltype(&ncclAllGather) all_gather = nullptr;
  decltype(&ncclCommDestroy) destroy = nullptr;
  decltype(&ncclGetErrorString) error_string = nullptr;
  bool ok = false;
};

inline const Api& api() {
  static Api a;
  static std::once_flag once;
  std::call_once(once, [] {
    void* h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL | RTLD_NOLOAD);
    if (!h) h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
    if (!h) return;
    a.get_unique_id = reinterpret_cast<decltype(a.get_unique_id)>(dlsym(h, "ncclGetUniqueId"));
    a.init_rank = reinterpret_cast<decltype(a.init_rank)>(dlsym(h, "ncclCommInitRank"));
    a.all_gather = reinterpret_cast<decltype(a.all_gather)>(dlsym(h, "ncclAllGather"));
    a.destroy = reinterpret_cast<decltype(a.destroy)>(dlsym(h, "ncclCommDestroy"));
    a.error_string = reinterpret_cast<decltype(a.error_string)>(dlsym(h, "ncclGetErrorString"));
    a.ok = a.get_unique_id && a.init_rank && a.all_gather && a.destroy && a.error_string;
  });
  return a;
}

inline int unavailable() {
  return set_error(PU_ERR_UNSUPPORTED, "NCCL (libnccl.so.2) could not be loaded");
}

inline int check_nccl(ncclResult_t r, const char* what) {
  if (r == ncclSuccess) return PU_OK;
  return set_error(PU_ERR_CUDA, "%s: %s", what, api().error_string(r));
}

}  // namespace comm
}  // namespace pu

extern "C" {

int pu_comm_unique_id(void* id) {
  using namespace pu::comm;
  if (!id) return pu::set_error(PU_ERR_INVALID_ARGUMENT, "null id buffer");
  if (!api().ok) return unavailable();
  ncclUniqueId u;
  const int rc = check_nccl(api().get_unique_id(&u), "ncclGetUniqueId");
  if (!rc) std::memcpy(id, &u, sizeof(u));
  return rc;
}

int pu_comm_init(const void* id, int64_t nranks, int64_t rank, void** comm) {
  using namespace pu::comm;
  if (!id || !comm) return pu::set_error(PU_ERR_INVALID_ARGUMENT, "null id or comm pointer");
  if (nranks < 1 || nranks > 1024 || rank < 0 || rank >= nranks)
    return pu::set_error(PU_ERR_INVALID_ARGUMENT, "rank %lld of %lld ranks", (long long)rank,
                         (long long)nranks);
  if (!api().ok) return unavailable();
  ncclUniqueId u;
  std::memcpy(&u, id, sizeof(u));
  ncclComm_t c = nullptr;
  const int rc = check_nccl(api().init_rank(&c, (int)nranks, u, (int)rank), "ncclCommInitRank");
  *comm = rc ? nullptr : static_cast<void*>(c);
  return rc;
}

int pu_allgather_partials(const float* partial, float* gathered, int64_t B, int64_t H, int64_t D,
                          void* comm, void* stream) {
  using namespace pu::comm;
  if (!partial || !gathered || !comm)
    return pu::set_error(PU_ERR_INVALID_ARGUMENT, "null partial, gathered or comm pointer");
  if (B <= 0 || H <= 0 || D <= 0) return pu::set_error(PU_ERR_INVALID_ARGUMENT, "B, H, D must be positive");
  if (!api().ok) return unavailable();
  const size_t count = (size_t)B * H * (D + 2);
  return check_nccl(api().all_gather(partial, gathered, count, ncclFloat32, static_cast<ncclComm_t>(comm),
                                     static_cast<cudaStream_t>(stream)),
                    "ncclAllGather");
}

int pu_comm_destroy(void* comm) {
  using namespace pu::comm;
  if (!comm) return PU_OK;
  if (!api().ok) return unavailable();
  return check_nccl(api().destroy(static_cast<ncclComm_t>(comm)), "ncclCommDestroy");
}

}  // extern "C"
