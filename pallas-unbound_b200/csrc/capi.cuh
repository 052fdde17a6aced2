// capi.cuh — library identity, error surface, device status word and the
// TMA tensor-map helpers.  Compiled once, inside pu_attn.cu.
#pragma once

#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <set>
#include <utility>

#include "pu_host.cuh"
#include "pu_ptx.cuh"

namespace pu {

namespace {
thread_local char t_last_error[512] = {0};
}

int set_error(int code, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(t_last_error, sizeof(t_last_error), fmt, ap);
  va_end(ap);
  return code;
}

int check_cuda(cudaError_t e, const char* what) {
  if (e == cudaSuccess) return PU_OK;
  return set_error(PU_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
}

namespace {

PFN_cuTensorMapEncodeTiled_v12000 g_encode_tiled = nullptr;
std::once_flag g_encode_once;
cudaError_t g_encode_status = cudaSuccess;

PFN_cuTensorMapEncodeTiled_v12000 get_encode_tiled() {
  std::call_once(g_encode_once, []() {
    void* fn = nullptr;
    cudaDriverEntryPointQueryResult q = cudaDriverEntryPointSymbolNotFound;
    g_encode_status =
        cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &fn, 12000, cudaEnableDefault, &q);
    if (g_encode_status == cudaSuccess && q == cudaDriverEntryPointSuccess) {
      g_encode_tiled = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
    }
  });
  return g_encode_tiled;
}

int make_tmap_3d(CUtensorMap* map, CUtensorMapDataType dt, uint32_t elem_bytes, const void* base,
                 uint64_t cols, uint64_t rows, uint64_t outer, uint32_t box_cols,
                 uint32_t box_rows, bool swizzle128) {
  auto enc = get_encode_tiled();
  if (!enc) {
    return set_error(PU_ERR_CUDA, "cuTensorMapEncodeTiled unavailable (driver entry point: %s)",
                     cudaGetErrorString(g_encode_status));
  }
  if (!aligned16(base)) {
    return set_error(PU_ERR_INVALID_ARGUMENT, "TMA base address %p is not 16-byte aligned", base);
  }
  if ((cols * elem_bytes) % 16 != 0) {
    return set_error(PU_ERR_INVALID_ARGUMENT, "row pitch %llu bytes is not a multiple of 16",
                     static_cast<unsigned long long>(cols * elem_bytes));
  }
  cuuint64_t dims[3] = {cols, rows, outer};
  cuuint64_t strides[2] = {cols * elem_bytes, cols * rows * elem_bytes};
  cuuint32_t box[3] = {box_cols, box_rows, 1};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = enc(map, dt, 3, const_cast<void*>(base), dims, strides, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE,
                   swizzle128 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_NONE,
                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    return set_error(PU_ERR_CUDA, "cuTensorMapEncodeTiled failed (CUresult %d)", static_cast<int>(r));
  }
  return PU_OK;
}

}  // namespace

int make_tmap_bf16_3d(CUtensorMap* map, const void* base, uint64_t cols, uint64_t rows,
                      uint64_t outer, uint32_t box_cols, uint32_t box_rows, bool swizzle128) {
  return make_tmap_3d(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, base, cols, rows, outer, box_cols,
                      box_rows, swizzle128);
}

int make_tmap_u8_3d(CUtensorMap* map, const void* base, uint64_t cols, uint64_t rows, uint64_t outer,
                    uint32_t box_cols, uint32_t box_rows, bool swizzle128) {
  return make_tmap_3d(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, base, cols, rows, outer, box_cols, box_rows,
                      swizzle128);
}

int make_tmap_f32_3d(CUtensorMap* map, const void* base, uint64_t cols, uint64_t rows,
                     uint64_t outer, uint32_t box_cols, uint32_t box_rows, bool swizzle128) {
  return make_tmap_3d(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, base, cols, rows, outer, box_cols,
                      box_rows, swizzle128);
}

int current_device() {
  int dev = -1;
  if (cudaGetDevice(&dev) != cudaSuccess) {
    set_error(PU_ERR_CUDA, "cudaGetDevice failed");
    return -1;
  }
  return dev;
}

int set_max_dynamic_smem(const void* func, int bytes, const char* what) {
  static std::mutex mu;
  static std::set<std::pair<const void*, int>> done;
  const int dev = current_device();
  if (dev < 0) return PU_ERR_CUDA;
  std::lock_guard<std::mutex> lock(mu);
  if (done.count({func, dev})) return PU_OK;
  const int rc =
      check_cuda(cudaFuncSetAttribute(func, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes), what);
  if (!rc) done.insert({func, dev});
  return rc;
}

int sm_count() {
  static int cache[64] = {0};
  int dev = current_device();
  if (dev < 0) return 148;
  if (dev < 64 && cache[dev] > 0) return cache[dev];
  int n = 0;
  if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) {
    n = 148;
  }
  if (dev < 64) cache[dev] = n;
  return n;
}

}  // namespace pu

extern "C" {

const char* pu_version(void) { return "pu_attn 0.1 sm_100a (tcgen05/TMA attention, split-KV decode)"; }

const char* pu_last_error(void) { return pu::t_last_error; }

int pu_device_status(int* detail) {
  cudaError_t e = cudaDeviceSynchronize();
  if (e != cudaSuccess) return pu::check_cuda(e, "cudaDeviceSynchronize");
  int host[2] = {0, 0};
  e = cudaMemcpyFromSymbol(host, pu::g_device_status, sizeof(host));
  if (e != cudaSuccess) return pu::check_cuda(e, "read device status");
  if (host[0] != 0) {
    int zero[2] = {0, 0};
    e = cudaMemcpyToSymbol(pu::g_device_status, zero, sizeof(zero));
    if (e != cudaSuccess) return pu::check_cuda(e, "clear device status");
  }
  if (detail) *detail = host[1];
  if (host[0] != 0) {
    return pu::set_error(host[0], "device reported status %d at site %d", host[0], host[1]);
  }
  return PU_OK;
}

}  // extern "C"

// ---------------------------------------------------------------------------
// Failure-detection self-test: one CTA waits on an mbarrier that nothing
// completes, with the given bound, exactly as the attention kernels wait on
// their pipelines.  The wait runs out, the kernel records
// PU_ERR_DEVICE_TIMEOUT at kSiteSelfTest and returns; the context stays usable.
// ---------------------------------------------------------------------------
namespace pu {
__global__ void selftest_timeout_kernel(uint64_t timeout_ns) {
  __shared__ uint64_t bar;
  __shared__ int abort_flag;
  if (threadIdx.x == 0) {
    mbar_init(&bar, 1);      // expects one arrival that never comes
    abort_flag = 0;
    fence_barrier_init();
  }
  __syncthreads();
  mbar_wait(&bar, 0, &abort_flag, kSiteSelfTest, timeout_ns);
}
}  // namespace pu

extern "C" int pu_selftest_wait_timeout(uint64_t timeout_ns, void* stream) {
  if (timeout_ns == 0 || timeout_ns > pu::kWaitTimeoutNs)
    return pu::set_error(PU_ERR_INVALID_ARGUMENT, "self-test timeout must be in (0, %llu] ns",
                         static_cast<unsigned long long>(pu::kWaitTimeoutNs));
  pu::selftest_timeout_kernel<<<1, 32, 0, static_cast<cudaStream_t>(stream)>>>(timeout_ns);
  return pu::check_cuda(cudaGetLastError(), "self-test launch");
}
