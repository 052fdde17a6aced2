// pu_attn.cu — the single translation unit of libpu_attn.so.  The kernels
// share one per-device status word (a __device__ variable), so they are
// compiled together instead of with relocatable device code.
#include "capi.cuh"
#include "decode.cuh"
#include "paged.cuh"
#include "gqa_tc.cuh"
#include "peer.cuh"
#include "outproj.cuh"
#include "attn_fwd.cuh"
#include "attn_bwd.cuh"
#include "comm.cuh"

// ---------------------------------------------------------------------------
// Allocation-free decode step (pu_decode_noalloc).
//
// Same kernel as pu_decode, but its scratch (split records and arrival
// counters) lives in the file-scope device array below instead of a
// caller-provided workspace, for callers that cannot allocate device memory.
// The array's host-side name is only a stand-in for the symbol; the device
// address is looked up once per device with cudaGetSymbolAddress (while that
// device is current) and cached.
// ---------------------------------------------------------------------------
#include <mutex>

namespace pu {
namespace noalloc {

constexpr size_t kScratchBytes = size_t(8) << 20;  // 8 MiB per device that loads the library
constexpr int kMaxDevices = 64;

static __device__ __align__(256) unsigned char g_decode_scratch[kScratchBytes];

std::mutex g_mutex;
void* g_scratch_ptr[kMaxDevices] = {nullptr};

// Device address of this device's scratch array (looked up on first use).
int scratch_for_current_device(void** out) {
  const int dev = current_device();
  if (dev < 0) return PU_ERR_CUDA;
  if (dev >= kMaxDevices) return set_error(PU_ERR_UNSUPPORTED, "device ordinal %d >= %d", dev, kMaxDevices);
  std::lock_guard<std::mutex> lock(g_mutex);
  if (g_scratch_ptr[dev] == nullptr) {
    void* p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, g_decode_scratch);
    if (e != cudaSuccess) return check_cuda(e, "cudaGetSymbolAddress(decode scratch)");
    g_scratch_ptr[dev] = p;
  }
  *out = g_scratch_ptr[dev];
  return PU_OK;
}

}  // namespace noalloc
}  // namespace pu

extern "C" int pu_decode_noalloc(const void* q, int q_dtype, const void* k_cache,
                                 const void* v_cache, int kv_dtype, const int32_t* kv_lens, void* o,
                                 float* lse, int64_t B, int64_t H, int64_t n, int64_t D,
                                 float sm_scale, void* stream) {
  using namespace pu::decode;
  int rc = check_args(q, q_dtype, k_cache, v_cache, kv_dtype, B, H, n, D);
  if (rc) return rc;
  if (!o) return pu::set_error(PU_ERR_INVALID_ARGUMENT, "null output");
  const Plan pl = make_plan(B * H, n, D, pu::sm_count(), kv_lens != nullptr);
  if (pl.total_bytes > pu::noalloc::kScratchBytes)
    return pu::set_error(PU_ERR_WORKSPACE,
                         "pu_decode_noalloc: B*H=%lld with %d splits needs %zu bytes of scratch, above "
                         "the fixed %zu-byte static scratch; use pu_decode with a workspace",
                         (long long)(B * H), pl.splits, pl.total_bytes, pu::noalloc::kScratchBytes);
  void* scratch = nullptr;
  rc = pu::noalloc::scratch_for_current_device(&scratch);
  if (rc) return rc;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  // The arrival counters must start at zero; the array keeps whatever the
  // previous call left, so clear them on the caller's stream.
  rc = pu::check_cuda(cudaMemsetAsync(scratch, 0, (size_t)(B * H) * sizeof(int), st),
                      "clear decode scratch counters");
  if (rc) return rc;
  Params prm{};
  prm.q = q;
  prm.k = k_cache;
  prm.v = v_cache;
  prm.lens = kv_lens;
  prm.kv_offset = 0;
  prm.n_local = (int)n;
  prm.H = (int)H;
  prm.splits = pl.splits;
  prm.chunk = pl.chunk;
  prm.scale_log2 = sm_scale * kLog2e;
  prm.ws_rec = reinterpret_cast<float*>(static_cast<char*>(scratch) + pl.rec_off);
  prm.ws_count = static_cast<int*>(scratch);
  prm.o = static_cast<__nv_bfloat16*>(o);
  prm.lse = lse;
  return launch<true>(prm, q_dtype, kv_dtype, (int)D, (int)(B * H), st);
}

// Binary architecture of the loaded kernels (one of each family).
extern "C" int pu_binary_arch(int* arch) {
  if (!arch) return pu::set_error(PU_ERR_INVALID_ARGUMENT, "null arch");
  const void* kernels[] = {
      reinterpret_cast<const void*>(pu::fwd::attn_fwd_kernel<128>),
      reinterpret_cast<const void*>(pu::bwd::attn_bwd_fused_kernel),
      reinterpret_cast<const void*>(pu::bwd::attn_bwd_dkdv_kernel<128>),
      reinterpret_cast<const void*>(pu::outproj::outproj_gemm_kernel),
  };
  int seen = -1;
  for (const void* k : kernels) {
    cudaFuncAttributes a{};
    const int rc = pu::check_cuda(cudaFuncGetAttributes(&a, k), "cudaFuncGetAttributes");
    if (rc) return rc;
    if (seen >= 0 && a.binaryVersion != seen)
      return pu::set_error(PU_ERR_UNSUPPORTED, "kernels built for different architectures (%d, %d)", seen,
                           a.binaryVersion);
    seen = a.binaryVersion;
  }
  *arch = seen;
  return PU_OK;
}
