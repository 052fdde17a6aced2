// peer.cuh — sequence-sharded decode whose partials travel by NVLink peer
// stores instead of a collective.
//
// The reference documents the split-KV merge as a psum of LogSumExp terms
// across the devices that hold the cache shards (README.md:41-46); the NCCL
// path of this library all-gathers the packed (m, l, o) records
// (pu_decode_partial + an all-gather + pu_decode_combine).  Here the split
// kernel's last CTA of each (b, h) stores the record straight into every
// rank's exchange buffer (this process's IPC mapping of it); a second kernel
// on each rank waits, bounded, until all G records of its (b, h) have
// arrived and merges them.  No NCCL call, no host round trip, no multicast,
// no fence: every record word is a 64-bit {value, epoch} pair written with
// one store, so the reader knows a word has arrived when its epoch matches
// (the low-latency protocol of collective libraries, here for one record).
//
// Exchange buffer of one rank (zeroed once when allocated):
//   [2][G][B*H][D+2] u64 words {fp32 bits, epoch}, slot (epoch & 1):
//       double-buffered so that a fast rank's next call never overwrites
//       words a slow rank is still merging (a rank starts call e+1 only
//       after its merge of e, which needed every rank's push of e, so a push
//       of e+2 follows every rank's merge of e)
// Epochs start at 1 and grow by one per call, in lockstep on all ranks.
#pragma once

#include "decode.cuh"

namespace pu {
namespace peer {

inline size_t exchange_bytes(long long BH, long long D, long long G) {
  return decode::round_up((size_t)2 * G * BH * (D + 2) * sizeof(unsigned long long), 256);
}

}  // namespace peer
}  // namespace pu

extern "C" {

int pu_peer_alloc(size_t bytes, void** dev_ptr, void* ipc_handle) {
  if (!dev_ptr || !ipc_handle || bytes == 0) return pu::set_error(PU_ERR_INVALID_ARGUMENT, "bad peer alloc args");
  static_assert(sizeof(cudaIpcMemHandle_t) == PU_IPC_HANDLE_BYTES, "IPC handle size");
  void* p = nullptr;
  int rc = pu::check_cuda(cudaMalloc(&p, bytes), "cudaMalloc (exchange buffer)");
  if (rc) return rc;
  // cudaMemset of device memory may return before the zeros land; finish it
  // here so a peer that opens the handle can never have its first records
  // erased by a zeroing still in flight
  rc = pu::check_cuda(cudaMemset(p, 0, bytes), "cudaMemset (exchange buffer)");
  if (!rc) rc = pu::check_cuda(cudaDeviceSynchronize(), "synchronize after zeroing the exchange buffer");
  if (!rc) {
    cudaIpcMemHandle_t h;
    rc = pu::check_cuda(cudaIpcGetMemHandle(&h, p), "cudaIpcGetMemHandle");
    if (!rc) memcpy(ipc_handle, &h, sizeof(h));
  }
  if (rc) {
    cudaFree(p);
    return rc;
  }
  *dev_ptr = p;
  return PU_OK;
}

int pu_peer_free(void* dev_ptr) { return pu::check_cuda(cudaFree(dev_ptr), "cudaFree (exchange buffer)"); }

int pu_peer_open(const void* ipc_handle, void** dev_ptr) {
  if (!ipc_handle || !dev_ptr) return pu::set_error(PU_ERR_INVALID_ARGUMENT, "bad peer open args");
  cudaIpcMemHandle_t h;
  memcpy(&h, ipc_handle, sizeof(h));
  return pu::check_cuda(cudaIpcOpenMemHandle(dev_ptr, h, cudaIpcMemLazyEnablePeerAccess),
                        "cudaIpcOpenMemHandle");
}

int pu_peer_close(void* dev_ptr) { return pu::check_cuda(cudaIpcCloseMemHandle(dev_ptr), "cudaIpcCloseMemHandle"); }

size_t pu_decode_exchange_bytes(int64_t B, int64_t H, int64_t D, int64_t G) {
  if (B <= 0 || H <= 0 || D <= 0 || G <= 0) return 0;
  return pu::peer::exchange_bytes(B * H, D, G);
}

}  // extern "C"

namespace pu {
namespace peer {

// The split-KV pass in push mode; with `o` set, its last CTAs also wait for
// and merge the other ranks' records (fused step).
inline int push(const void* q, int q_dtype, const void* k_cache, const void* v_cache, int kv_dtype,
                const int32_t* kv_lens, int64_t kv_offset, void* const* exchange, int64_t G, int64_t rank,
                uint32_t epoch, void* o, float* lse, uint64_t timeout_ns, void* workspace, size_t workspace_bytes,
                int64_t B, int64_t H, int64_t n_local, int64_t D, float sm_scale, void* stream) {
  using namespace pu::decode;
  int rc = check_args(q, q_dtype, k_cache, v_cache, kv_dtype, B, H, n_local, D);
  if (rc) return rc;
  if (!exchange) return set_error(PU_ERR_INVALID_ARGUMENT, "null exchange pointer array");
  if (G < 1 || G > kMaxPeers) return set_error(PU_ERR_UNSUPPORTED, "%lld ranks (1..%d)", (long long)G, kMaxPeers);
  if (rank < 0 || rank >= G) return set_error(PU_ERR_INVALID_ARGUMENT, "rank %lld of %lld", (long long)rank, (long long)G);
  if (epoch == 0) return set_error(PU_ERR_INVALID_ARGUMENT, "epochs start at 1");
  if (kv_offset < 0) return set_error(PU_ERR_INVALID_ARGUMENT, "negative kv_offset");
  const Plan pl = make_plan(B * H, n_local, D, sm_count(), kv_lens != nullptr);
  if (!workspace || workspace_bytes < pl.total_bytes)
    return set_error(PU_ERR_WORKSPACE, "decode workspace needs %zu bytes, got %zu", pl.total_bytes, workspace_bytes);
  Params prm{};
  prm.q = q;
  prm.k = k_cache;
  prm.v = v_cache;
  prm.lens = kv_lens;
  prm.kv_offset = kv_offset;
  prm.n_local = (int)n_local;
  prm.H = (int)H;
  prm.splits = pl.splits;
  prm.chunk = pl.chunk;
  prm.scale_log2 = sm_scale * kLog2e;
  prm.ws_rec = reinterpret_cast<float*>(static_cast<char*>(workspace) + pl.rec_off);
  prm.ws_count = static_cast<int*>(workspace);
  for (int g = 0; g < G; ++g) {
    if (!exchange[g] || !aligned16(exchange[g]))
      return set_error(PU_ERR_INVALID_ARGUMENT, "exchange buffer %d null or unaligned", g);
    prm.peer_rec[g] = static_cast<unsigned long long*>(exchange[g]);
  }
  prm.n_peers = (int)G;
  prm.rank = (int)rank;
  prm.epoch = epoch;
  prm.o = static_cast<__nv_bfloat16*>(o);
  prm.lse = lse;
  prm.timeout_ns = timeout_ns;
  return launch<false, false, true>(prm, q_dtype, kv_dtype, (int)D, (int)(B * H), static_cast<cudaStream_t>(stream));
}

inline int check_timeout(uint64_t timeout_ns) {
  if (timeout_ns == 0 || timeout_ns > kWaitTimeoutNs)
    return set_error(PU_ERR_INVALID_ARGUMENT, "timeout must be in (0, 2 s]");
  return PU_OK;
}

}  // namespace peer
}  // namespace pu

extern "C" {

int pu_decode_push(const void* q, int q_dtype, const void* k_cache, const void* v_cache, int kv_dtype,
                   const int32_t* kv_lens, int64_t kv_offset, void* const* exchange, int64_t G,
                   int64_t rank, uint32_t epoch, void* workspace, size_t workspace_bytes, int64_t B,
                   int64_t H, int64_t n_local, int64_t D, float sm_scale, void* stream) {
  return pu::peer::push(q, q_dtype, k_cache, v_cache, kv_dtype, kv_lens, kv_offset, exchange, G, rank, epoch,
                        nullptr, nullptr, 0, workspace, workspace_bytes, B, H, n_local, D, sm_scale, stream);
}

int pu_decode_pull(const void* exchange, int64_t G, uint32_t epoch, void* o, float* lse, int64_t B, int64_t H,
                   int64_t D, uint64_t timeout_ns, void* stream) {
  if (!exchange || !o) return pu::set_error(PU_ERR_INVALID_ARGUMENT, "null exchange buffer or output");
  if (G < 1 || G > pu::decode::kMaxPeers) return pu::set_error(PU_ERR_UNSUPPORTED, "%lld ranks", (long long)G);
  if (D != 64 && D != 128) return pu::set_error(PU_ERR_UNSUPPORTED, "head size %lld", (long long)D);
  if (B <= 0 || H <= 0 || B * H > pu::decode::kMaxBH) return pu::set_error(PU_ERR_INVALID_ARGUMENT, "bad B*H");
  if (epoch == 0) return pu::set_error(PU_ERR_INVALID_ARGUMENT, "epochs start at 1");
  if (int rc = pu::peer::check_timeout(timeout_ns)) return rc;
  if (!pu::aligned16(exchange)) return pu::set_error(PU_ERR_INVALID_ARGUMENT, "exchange buffer unaligned");
  const auto* words = static_cast<const unsigned long long*>(exchange);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  auto* out = static_cast<__nv_bfloat16*>(o);
  if (D == 128)
    pu::decode::peer_combine_kernel<128><<<(unsigned)(B * H), 128, 0, st>>>(words, (int)G, (int)(B * H), epoch,
                                                                           timeout_ns, out, lse);
  else
    pu::decode::peer_combine_kernel<64><<<(unsigned)(B * H), 64, 0, st>>>(words, (int)G, (int)(B * H), epoch,
                                                                         timeout_ns, out, lse);
  return pu::check_cuda(cudaGetLastError(), "peer combine launch");
}

int pu_decode_sharded(const void* q, int q_dtype, const void* k_cache, const void* v_cache, int kv_dtype,
                      const int32_t* kv_lens, int64_t kv_offset, void* const* exchange, int64_t G, int64_t rank,
                      uint32_t epoch, void* o, float* lse, void* workspace, size_t workspace_bytes, int64_t B,
                      int64_t H, int64_t n_local, int64_t D, float sm_scale, uint64_t timeout_ns, void* stream) {
  if (!o) return pu::set_error(PU_ERR_INVALID_ARGUMENT, "null output");
  if (int rc = pu::peer::check_timeout(timeout_ns)) return rc;
  // The fused merge makes the last CTA of each (b, h) wait for the other
  // ranks; with at most half of the resident CTA slots waiting, every rank's
  // other CTAs always find room to run.
  const long long slots = (long long)pu::sm_count() * pu::decode::kCtasPerSm;
  if (2 * B * H <= slots)
    return pu::peer::push(q, q_dtype, k_cache, v_cache, kv_dtype, kv_lens, kv_offset, exchange, G, rank, epoch, o,
                          lse, timeout_ns, workspace, workspace_bytes, B, H, n_local, D, sm_scale, stream);
  int rc = pu::peer::push(q, q_dtype, k_cache, v_cache, kv_dtype, kv_lens, kv_offset, exchange, G, rank, epoch,
                          nullptr, nullptr, 0, workspace, workspace_bytes, B, H, n_local, D, sm_scale, stream);
  if (rc) return rc;
  return pu_decode_pull(exchange[rank], G, epoch, o, lse, B, H, D, timeout_ns, stream);
}

}  // extern "C"
