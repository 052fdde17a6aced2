// pu_status.cuh — error reporting shared by every kernel and entry point.
//
// Device side: one status word per device (a __device__ variable of this
// library's module).  A kernel that gives up on a bounded wait writes
// PU_ERR_DEVICE_TIMEOUT and a location code there and returns normally, so
// the CUDA context stays usable; pu_device_status() reads and clears it.
//
// Host side: a thread-local last-error message behind pu_last_error().
#pragma once

#include <cstdint>
#include <cuda_runtime.h>

#include "pu_attn.h"

namespace pu {

// Longest a kernel waits on any single mbarrier or counter before it gives
// up (nanoseconds of %globaltimer).  Correct code never gets near it.
constexpr uint64_t kWaitTimeoutNs = 2000000000ull;  // 2 s

// Location codes written to the status detail word.
enum WaitSite : int {
  kSiteFwdQ = 101,
  kSiteFwdKFull = 102,
  kSiteFwdVFull = 103,
  kSiteFwdKEmpty = 104,
  kSiteFwdVEmpty = 105,
  kSiteFwdSFull = 106,
  kSiteFwdPFull = 107,
  kSiteFwdODone = 108,
  kSiteBwdLoad = 201,
  kSiteBwdEmpty = 202,
  kSiteBwdMma = 203,
  kSiteBwdSoftmax = 204,
  kSiteBwdDs = 205,
  kSiteBwdDq = 206,
  kSiteBwdKV = 207,
  kSiteDecodeCounter = 301,
  kSiteDecodePage = 302,
  kSiteAppendPage = 303,
  kSiteDecodePeer = 304,
  kSiteDecodeTc = 305,
  kSiteOutProj = 401,
  kSiteSelfTest = 901,
};

// Defined once: the library is a single translation unit.
__device__ int g_device_status[2];

__device__ __forceinline__ void record_device_error(int code, int where) {
  if (atomicCAS(&g_device_status[0], 0, code) == 0) {
    atomicExch(&g_device_status[1], where);
  }
}

// Host helpers (defined in capi.cu).
int set_error(int code, const char* fmt, ...);
int check_cuda(cudaError_t e, const char* what);

}  // namespace pu
