// paged.cuh — paged KV cache: append of the new token's K/V, and the split-KV
// decode over the page pool.
//
// The reference's decode reads a dense, padded [B, H, N, D] cache
// (src/pallas_flash/kernels/decoding.py:86-103, 113-115); serving stacks keep
// the cache in fixed-size pages instead so that sequences grow without
// copies.  Layout here:
//   pools      k_pool, v_pool: [num_pages][H][page_size][D] (fp16 or bf16),
//              one page = page_size consecutive tokens of one sequence, all
//              heads (each (page, head) slab is contiguous for streaming)
//   page table int32 [B][max_pages]: physical page of logical page i of b
//   lengths    int32 [B]: tokens held by each sequence
// Page numbers are checked on the device: an entry outside [0, num_pages)
// is reported through the status word and its tokens are skipped, so a
// corrupt table cannot make the kernels read or write outside the pools.
#pragma once

#include "decode.cuh"

namespace pu {
namespace paged {

inline int log2_exact(long long x) {
  int s = 0;
  while ((1ll << s) < x) ++s;
  return ((1ll << s) == x) ? s : -1;
}

// One CTA per sequence b: all H heads of the new token are written, then the
// length is advanced (after every thread's write of this CTA).
template <typename T>
__global__ void __launch_bounds__(256) append_kernel(const T* __restrict__ k_new, const T* __restrict__ v_new,
                                                     T* __restrict__ k_pool, T* __restrict__ v_pool,
                                                     const int32_t* __restrict__ page_table, int max_pages,
                                                     int num_pages, int page_shift, int32_t* __restrict__ lens,
                                                     int H, int D) {
  __shared__ int s_pos;
  __shared__ int s_page;
  const int b = blockIdx.x;
  if (threadIdx.x == 0) {
    const int pos = lens[b];
    int pg = -1;
    if (pos >= 0 && (pos >> page_shift) < max_pages) pg = page_table[(size_t)b * max_pages + (pos >> page_shift)];
    if ((unsigned)pg >= (unsigned)num_pages) {
      record_device_error(PU_ERR_INVALID_ARGUMENT, kSiteAppendPage);
      pg = -1;
    }
    s_pos = pos;
    s_page = pg;
  }
  __syncthreads();
  const int pos = s_pos, pg = s_page;
  if (pg < 0) return;
  const int vec = D / 8;                               // 16-byte vectors per row
  const size_t row = (size_t)(pos & ((1 << page_shift) - 1));
  for (int i = threadIdx.x; i < H * vec; i += blockDim.x) {
    const int h = i / vec, c = i % vec;
    const size_t src = ((size_t)b * H + h) * D + (size_t)c * 8;
    const size_t dst = ((((size_t)pg * H + h) << page_shift) + row) * D + (size_t)c * 8;
    *reinterpret_cast<uint4*>(k_pool + dst) = *reinterpret_cast<const uint4*>(k_new + src);
    *reinterpret_cast<uint4*>(v_pool + dst) = *reinterpret_cast<const uint4*>(v_new + src);
  }
  __syncthreads();
  if (threadIdx.x == 0) lens[b] = pos + 1;
}

inline int check_pages(const int32_t* table, long long max_pages, long long num_pages, long long page_size,
                       int* shift) {
  if (!table) return set_error(PU_ERR_INVALID_ARGUMENT, "null page table");
  if (max_pages <= 0 || num_pages <= 0) return set_error(PU_ERR_INVALID_ARGUMENT, "page counts must be positive");
  const int s = log2_exact(page_size);
  if (s < 4 || s > 12) return set_error(PU_ERR_UNSUPPORTED, "page size %lld (power of two in [16, 4096])", page_size);
  if (num_pages * page_size > (1ll << 31) || max_pages * page_size > (1ll << 30))
    return set_error(PU_ERR_UNSUPPORTED, "page pool too large");
  *shift = s;
  return PU_OK;
}

}  // namespace paged
}  // namespace pu

extern "C" size_t pu_decode_paged_workspace_size(int64_t B, int64_t H, int64_t max_pages_per_seq,
                                                 int64_t page_size, int64_t D) {
  if (B <= 0 || H <= 0 || max_pages_per_seq <= 0 || page_size <= 0 || D <= 0) return 0;
  return pu::decode::make_plan(B * H, max_pages_per_seq * page_size, D, pu::sm_count(), true, page_size).total_bytes;
}

extern "C" int pu_decode_paged(const void* q, int q_dtype, const void* k_pool, const void* v_pool, int kv_dtype,
                               const int32_t* page_table, int64_t max_pages_per_seq, int64_t num_pages,
                               int64_t page_size, const int32_t* kv_lens, void* o, float* lse, void* workspace,
                               size_t workspace_bytes, int64_t B, int64_t H, int64_t D, float sm_scale,
                               void* stream) {
  using namespace pu::decode;
  const long long n_cap = max_pages_per_seq * page_size;
  int rc = check_args(q, q_dtype, k_pool, v_pool, kv_dtype, B, H, n_cap > 0 ? n_cap : 1, D);
  if (rc) return rc;
  int shift = 0;
  rc = pu::paged::check_pages(page_table, max_pages_per_seq, num_pages, page_size, &shift);
  if (rc) return rc;
  if (!o || !kv_lens) return pu::set_error(PU_ERR_INVALID_ARGUMENT, "null output or lengths");
  const Plan pl = make_plan(B * H, n_cap, D, pu::sm_count(), true, page_size);
  if (!workspace || workspace_bytes < pl.total_bytes)
    return pu::set_error(PU_ERR_WORKSPACE, "paged decode workspace needs %zu bytes, got %zu", pl.total_bytes,
                         workspace_bytes);
  Params prm{};
  prm.q = q;
  prm.k = k_pool;
  prm.v = v_pool;
  prm.lens = kv_lens;
  prm.kv_offset = 0;
  prm.n_local = (int)n_cap;
  prm.H = (int)H;
  prm.splits = pl.splits;
  prm.chunk = pl.chunk;
  prm.scale_log2 = sm_scale * kLog2e;
  prm.ws_rec = reinterpret_cast<float*>(static_cast<char*>(workspace) + pl.rec_off);
  prm.ws_count = static_cast<int*>(workspace);
  prm.o = static_cast<__nv_bfloat16*>(o);
  prm.lse = lse;
  prm.page_table = page_table;
  prm.max_pages = (int)max_pages_per_seq;
  prm.num_pages = (int)num_pages;
  prm.page_shift = shift;
  return launch<true, true>(prm, q_dtype, kv_dtype, (int)D, (int)(B * H), static_cast<cudaStream_t>(stream));
}

extern "C" int pu_kv_append(const void* k_new, const void* v_new, int kv_dtype, void* k_pool, void* v_pool,
                            const int32_t* page_table, int64_t max_pages_per_seq, int64_t num_pages,
                            int64_t page_size, int32_t* kv_lens, int64_t B, int64_t H, int64_t D, void* stream) {
  if (!k_new || !v_new || !k_pool || !v_pool || !kv_lens)
    return pu::set_error(PU_ERR_INVALID_ARGUMENT, "null k/v/pool/lengths pointer");
  if (B <= 0 || H <= 0) return pu::set_error(PU_ERR_INVALID_ARGUMENT, "B and H must be positive");
  if (D % 8 != 0 || D <= 0 || D > 256) return pu::set_error(PU_ERR_UNSUPPORTED, "head size %lld", (long long)D);
  if (kv_dtype != PU_DTYPE_F16 && kv_dtype != PU_DTYPE_BF16)
    return pu::set_error(PU_ERR_UNSUPPORTED, "cache dtype must be f16 or bf16");
  if (!pu::aligned16(k_new) || !pu::aligned16(v_new) || !pu::aligned16(k_pool) || !pu::aligned16(v_pool))
    return pu::set_error(PU_ERR_INVALID_ARGUMENT, "k/v/pools must be 16-byte aligned");
  if (B > 2147483647ll) return pu::set_error(PU_ERR_UNSUPPORTED, "batch too large");
  int shift = 0;
  int rc = pu::paged::check_pages(page_table, max_pages_per_seq, num_pages, page_size, &shift);
  if (rc) return rc;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  // 16-bit element types share one kernel: the copy moves raw 16-byte vectors
  pu::paged::append_kernel<__half><<<(unsigned)B, 256, 0, st>>>(
      static_cast<const __half*>(k_new), static_cast<const __half*>(v_new), static_cast<__half*>(k_pool),
      static_cast<__half*>(v_pool), page_table, (int)max_pages_per_seq, (int)num_pages, shift, kv_lens, (int)H,
      (int)D);
  return pu::check_cuda(cudaGetLastError(), "kv append launch");
}
