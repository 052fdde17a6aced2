// decode.cuh — split-KV flash decode (one query token per (b, h)).
//
// Reference: decoding_kv_loop / flash_decoding_kernel
// (src/pallas_flash/kernels/decoding.py:19-84) walk the whole cache of one
// (b, h) in 128-token blocks with an online softmax and return (o, m, l).
// Here the cache of each (b, h) is cut into `splits` contiguous chunks, one
// CTA per chunk, so every SM streams K/V at once.  The kernel is HBM-bound:
// each K/V row (D fp16/bf16 values) is read exactly once with 128-bit
// streaming loads, D/8 lanes per row, 8 rows in flight per lane group.
//
// Per CTA: lane groups keep (m, l, o) in registers (log2 domain), merge
// through shared memory, and write one split record to the workspace.  The
// last CTA of each (b, h) (an atomic counter in the workspace, reset by that
// CTA) merges the split records: into the bf16 output and LSE (single-GPU
// step), or into the shard's packed partial {m, l, o[D]} that an NCCL
// all-gather carries to the other ranks (sequence-sharded step).
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_fp8.h>

#include "pu_host.cuh"
#include "pu_ptx.cuh"

namespace pu {
namespace decode {

constexpr int kThreads = 256;
constexpr int kWarps = kThreads / 32;
constexpr int kCtasPerSm = 2;     // occupancy the launch bounds ask for
constexpr int kWaves = 4;         // CTAs per SM slot the split heuristic aims at
constexpr int kMinChunk = 256;    // fewest tokens one CTA is given
constexpr float kLog2e = 1.4426950408889634f;
constexpr float kLn2 = 0.6931471805599453f;
constexpr int kMaxPeers = 8;      // ranks of a push-mode exchange (one NVLink domain)

struct Params {
  const void* q;
  const void* k;
  const void* v;
  const int32_t* lens;   // [B] global lengths or nullptr
  long long kv_offset;   // global position of local token 0
  int n_local;           // tokens in this shard's cache
  int H;                 // query heads
  int group = 1;         // query heads per K/V head (GQA / MQA); K/V head = h / group
  float o_scale = 1.f;   // factor on every output record (the fp8 V scale)
  int splits;            // CTAs per (b, h)
  int chunk;             // tokens per CTA (multiple of 16)
  float scale_log2;      // sm_scale * log2(e)
  float* ws_rec;         // [BH][splits][D+2] split records (log2-domain m)
  int* ws_count;         // [BH] arrival counters (zero between calls)
  // outputs
  __nv_bfloat16* o;      // final mode: [BH][D]
  float* lse;            // final mode: [BH] or nullptr
  float* partial;        // partial mode: [BH][D+2] (natural-log m)
  // paged cache: k / v are page pools [num_pages][H][page_size][D]; token t of
  // sequence b lives in page page_table[b * max_pages + t / page_size]
  const int32_t* page_table;
  int max_pages;
  int num_pages;
  int page_shift;        // log2(page_size)
  // push mode (sequence-sharded decode over peer memory): the shard's record
  // for (b, h) goes to slot [epoch & 1][rank][bh] of every rank's exchange
  // buffer as 64-bit words {value bits, epoch} (one store each, so a reader
  // that sees the epoch sees the value: no fence, no separate flag)
  unsigned long long* peer_rec[kMaxPeers];
  int n_peers;
  int rank;
  unsigned epoch;
  uint64_t timeout_ns;   // bound of the fused merge's wait
};

template <typename T>
__device__ __forceinline__ void unpack8(const uint4& w, float (&f)[8]);

template <>
__device__ __forceinline__ void unpack8<__half>(const uint4& w, float (&f)[8]) {
  const uint32_t u[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    __half2 h = *reinterpret_cast<const __half2*>(&u[i]);
    float2 x = __half22float2(h);
    f[2 * i] = x.x;
    f[2 * i + 1] = x.y;
  }
}

template <>
__device__ __forceinline__ void unpack8<__nv_bfloat16>(const uint4& w, float (&f)[8]) {
  const uint32_t u[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    // bf16 -> fp32 is a 16-bit shift
    f[2 * i] = __uint_as_float(u[i] << 16);
    f[2 * i + 1] = __uint_as_float(u[i] & 0xFFFF0000u);
  }
}

__device__ __forceinline__ uint4 ld_stream(const uint4* p) {
  uint4 r;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0, %1, %2, %3}, [%4];"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
               : "l"(p));
  return r;
}

// ld_stream when `pred`, else zeros; a predicated load, not a branch.
__device__ __forceinline__ uint4 ld_stream_if(const uint4* p, bool pred) {
  uint4 r = make_uint4(0, 0, 0, 0);
  asm volatile(
      "{\n .reg .pred q;\n setp.ne.b32 q, %5, 0;\n"
      " @q ld.global.nc.L1::no_allocate.v4.u32 {%0, %1, %2, %3}, [%4];\n}"
      : "+r"(r.x), "+r"(r.y), "+r"(r.z), "+r"(r.w)
      : "l"(p), "r"((int)pred));
  return r;
}

// ld_stream_if for 8-byte rows pieces (fp8 caches: 8 elements per lane).
__device__ __forceinline__ uint2 ld_stream_if(const uint2* p, bool pred) {
  uint2 r = make_uint2(0, 0);
  asm volatile(
      "{\n .reg .pred q;\n setp.ne.b32 q, %3, 0;\n"
      " @q ld.global.nc.L1::no_allocate.v2.u32 {%0, %1}, [%2];\n}"
      : "+r"(r.x), "+r"(r.y)
      : "l"(p), "r"((int)pred));
  return r;
}

// Cache element types: the load word of 8 elements and its unpacking.
template <typename T>
struct KVIO {
  using W = uint4;
  static constexpr int kUnroll = 8;   // rows in flight per lane group
  __device__ __forceinline__ static W ld(const T* p, bool pred) {
    return ld_stream_if(reinterpret_cast<const uint4*>(p), pred);
  }
  __device__ __forceinline__ static void unpack(const W& w, float (&f)[8]) { unpack8<T>(w, f); }
};

// fp8 e4m3: 8 bytes per lane, twice the rows in flight for the same bytes
template <>
struct KVIO<__nv_fp8_e4m3> {
  using W = uint2;
  static constexpr int kUnroll = 16;
  __device__ __forceinline__ static W ld(const __nv_fp8_e4m3* p, bool pred) {
    return ld_stream_if(reinterpret_cast<const uint2*>(p), pred);
  }
  __device__ __forceinline__ static void unpack(const W& w, float (&f)[8]) {
    const uint32_t u[2] = {w.x, w.y};
#pragma unroll
    for (int i = 0; i < 2; ++i) {
      const __half2 lo(__nv_cvt_fp8x2_to_halfraw2((__nv_fp8x2_storage_t)(u[i] & 0xFFFFu), __NV_E4M3));
      const __half2 hi(__nv_cvt_fp8x2_to_halfraw2((__nv_fp8x2_storage_t)(u[i] >> 16), __NV_E4M3));
      const float2 a = __half22float2(lo), b = __half22float2(hi);
      f[4 * i] = a.x;
      f[4 * i + 1] = a.y;
      f[4 * i + 2] = b.x;
      f[4 * i + 3] = b.y;
    }
  }
};

// Merge the nrec split records {m (log2 units), l, o[D]} of one (b, h) with a
// stable LogSumExp.  Thread d < D reads the records kMergeBatch at a time,
// every load of a batch in flight together (one L2 round trip per batch, at
// the end of the kernel where nothing hides it), and folds them in record
// order into a running maximum M, sum L and column d's sum O; threads d >= D
// return M = -inf, L = O = 0.  No barrier inside.
constexpr int kMergeBatch = 16;

template <int D>
__device__ __forceinline__ void block_merge(const float* rec, int nrec, float& M, float& L, float& O) {
  constexpr int stride = D + 2;
  const int d = threadIdx.x;
  M = -INFINITY;
  L = 0.f;
  O = 0.f;
  if (d >= D) return;
  for (int c = 0; c < nrec; c += kMergeBatch) {
    float m[kMergeBatch], l[kMergeBatch], x[kMergeBatch];
#pragma unroll
    for (int u = 0; u < kMergeBatch; ++u) {
      const bool ok = c + u < nrec;
      const float* r = rec + (size_t)(c + u) * stride;
      m[u] = ok ? __ldcg(r) : -INFINITY;
      l[u] = ok ? __ldcg(r + 1) : 0.f;
      x[u] = ok ? __ldcg(r + 2 + d) : 0.f;
    }
    float bm = M;
#pragma unroll
    for (int u = 0; u < kMergeBatch; ++u) bm = fmaxf(bm, m[u]);
    if (bm == -INFINITY) continue;              // every record so far is empty
    const float a = (M == -INFINITY) ? 0.f : ex2(M - bm);
    L *= a;
    O *= a;
#pragma unroll
    for (int u = 0; u < kMergeBatch; ++u) {
      const float w = (m[u] == -INFINITY) ? 0.f : ex2(m[u] - bm);
      L = fmaf(w, l[u], L);
      O = fmaf(w, x[u], O);
    }
    M = bm;
  }
}

// Push-mode merge for one (b, h): wait (bounded) until the words of every
// rank's record in the local exchange buffer carry `epoch`, then merge in
// rank order (the arithmetic of combine_kernel).  Called by every thread of
// the block (d = thread index; threads d >= D only join the vote).  A wait
// that runs out records PU_ERR_DEVICE_TIMEOUT (detail kSiteDecodePeer) and
// the output is zeros.
template <int D>
__device__ __forceinline__ void peer_merge(const unsigned long long* exch, int G, int BH, int bh, unsigned epoch,
                                           uint64_t timeout_ns, __nv_bfloat16* o, float* lse, int d) {
  const unsigned long long* base = exch + (size_t)(epoch & 1u) * G * BH * (D + 2);
  float mg[kMaxPeers], lg[kMaxPeers], og[kMaxPeers];
  unsigned long long wm[kMaxPeers], wl[kMaxPeers], wo[kMaxPeers];
  // first reads of every rank's words, all in flight together
#pragma unroll
  for (int g = 0; g < kMaxPeers; ++g) {
    wm[g] = wl[g] = wo[g] = 0ull;
    if (d < D && g < G) {
      const unsigned long long* r = base + ((size_t)g * BH + bh) * (D + 2);
      wm[g] = ld_volatile_u64(r);
      wl[g] = ld_volatile_u64(r + 1);
      wo[g] = ld_volatile_u64(r + 2 + d);
    }
  }
  // Poll in rounds: every word whose epoch is not yet this call's is read
  // again, all such reads of a round in flight together, so the wait ends one
  // L2 round trip after the last rank's record lands (settling the words one
  // at a time would chain up to three round trips per rank).
  bool ok = true;
  if (d < D) {
    const uint64_t t0 = global_timer_ns();
    while (true) {
      bool pending = false;
#pragma unroll
      for (int g = 0; g < kMaxPeers; ++g)
        if (g < G)
          pending |= ((unsigned)(wm[g] >> 32) != epoch) | ((unsigned)(wl[g] >> 32) != epoch) |
                     ((unsigned)(wo[g] >> 32) != epoch);
      if (!pending) break;
      if (global_timer_ns() - t0 > timeout_ns) {
        ok = false;
        break;
      }
#pragma unroll
      for (int g = 0; g < kMaxPeers; ++g) {
        if (g >= G) continue;
        const unsigned long long* r = base + ((size_t)g * BH + bh) * (D + 2);
        if ((unsigned)(wm[g] >> 32) != epoch) wm[g] = ld_volatile_u64(r);
        if ((unsigned)(wl[g] >> 32) != epoch) wl[g] = ld_volatile_u64(r + 1);
        if ((unsigned)(wo[g] >> 32) != epoch) wo[g] = ld_volatile_u64(r + 2 + d);
      }
    }
  }
#pragma unroll
  for (int g = 0; g < kMaxPeers; ++g) {
    const bool have = ok && d < D && g < G;
    mg[g] = have ? __uint_as_float((unsigned)wm[g]) : -INFINITY;
    lg[g] = have ? __uint_as_float((unsigned)wl[g]) : 0.f;
    og[g] = have ? __uint_as_float((unsigned)wo[g]) : 0.f;
  }
  if (!__syncthreads_and(ok)) {
    if (d == 0) record_device_error(PU_ERR_DEVICE_TIMEOUT, kSiteDecodePeer);
    if (d < D) o[(size_t)bh * D + d] = __float2bfloat16_rn(0.f);
    if (d == 0 && lse != nullptr) lse[bh] = -INFINITY;
    return;
  }
  if (d >= D) return;
  float M = -INFINITY;
#pragma unroll
  for (int g = 0; g < kMaxPeers; ++g) M = fmaxf(M, mg[g]);
  float L = 0.f, O = 0.f;
  if (M != -INFINITY) {
#pragma unroll
    for (int g = 0; g < kMaxPeers; ++g) {
      if (g >= G || mg[g] == -INFINITY) continue;
      const float w = ex2((mg[g] - M) * kLog2e);
      L += w * lg[g];
      O += w * og[g];
    }
  }
  o[(size_t)bh * D + d] = __float2bfloat16_rn(L > 0.f ? O / L : 0.f);
  if (d == 0 && lse != nullptr) lse[bh] = (L > 0.f) ? M + logf(L) : -INFINITY;
}

template <int D>
__global__ void __launch_bounds__(D) peer_combine_kernel(const unsigned long long* __restrict__ exch, int G,
                                                         int BH, unsigned epoch, uint64_t timeout_ns,
                                                         __nv_bfloat16* __restrict__ o,
                                                         float* __restrict__ lse) {
  peer_merge<D>(exch, G, BH, blockIdx.x, epoch, timeout_ns, o, lse, threadIdx.x);
}

// kFinal: write the bf16 output; else the shard partial (to `partial`, or to
// every peer's exchange buffer when kPush).
template <typename QT, typename KVT, int D, bool kFinal, bool kPaged, bool kPush = false>
__global__ void __launch_bounds__(kThreads, kCtasPerSm) split_kv_kernel(const Params p) {
  using IO = KVIO<KVT>;
  constexpr int kUnroll = IO::kUnroll;
  constexpr int LPR = D / 8;        // lanes per cache row
  constexpr int RPW = 32 / LPR;     // rows per warp instruction
  constexpr int ROWS_PER_ITER = kWarps * RPW * kUnroll;
  constexpr int NGROUP = kWarps * RPW;  // lane groups per CTA
  static_assert(D == 64 || D == 128, "head size");

  __shared__ float sm_m[NGROUP];
  __shared__ float sm_l[NGROUP];
  __shared__ float sm_o[NGROUP][D];
  __shared__ int sm_last;

  const int tid = threadIdx.x;
  const int warp = tid >> 5;
  const int lane = tid & 31;
  const int sub = lane % LPR;       // which 8 columns of the row
  const int rw = lane / LPR;        // which row of the warp instruction
  const int split = blockIdx.x;
  const int bh = blockIdx.y;
  const int b = bh / p.H;
  // launched with programmatic stream serialization: the CTAs may start while
  // the previous kernel of the stream finishes; nothing in global memory is
  // touched before this wait
  grid_dep_wait();
  grid_dep_launch_dependents();

  int len = p.n_local;
  if (p.lens != nullptr) {
    long long g = (long long)p.lens[b] - p.kv_offset;
    len = g < 0 ? 0 : (g > p.n_local ? p.n_local : (int)g);
  }
  const int t_begin = split * p.chunk;
  const int t_end = min(t_begin + p.chunk, len);

  // query slice, pre-scaled into log2 units
  float qf[8];
  {
    const uint4 w = *reinterpret_cast<const uint4*>(static_cast<const QT*>(p.q) + (size_t)bh * D + sub * 8);
    unpack8<QT>(w, qf);
#pragma unroll
    for (int i = 0; i < 8; ++i) qf[i] *= p.scale_log2;
  }

  // K/V head of this query head (GQA / MQA: `group` query heads share one)
  const int h = bh % p.H;
  const int h_kv = h / p.group;
  const int H_kv = p.H / p.group;
  const size_t kv_head = (size_t)b * H_kv + h_kv;
  const KVT* kb = static_cast<const KVT*>(p.k) + kv_head * p.n_local * D + sub * 8;
  const KVT* vb = static_cast<const KVT*>(p.v) + kv_head * p.n_local * D + sub * 8;
  // paged cache: token t of sequence b is row t % page_size of page
  // page_table[b][t / page_size]; out-of-range page numbers are reported
  // and their tokens skipped.  A warp's tokens of one iteration are TW
  // consecutive tokens starting at a multiple of TW (chunks are multiples of
  // the page size), so when page_size >= TW they share one page: its entry
  // is read once, one iteration ahead of its use.
  constexpr int TW = RPW * kUnroll;
  const int32_t* table_b = nullptr;
  bool one_page = false;
  int pg_next = 0;
  if constexpr (kPaged) {
    kb = static_cast<const KVT*>(p.k) + sub * 8;
    vb = static_cast<const KVT*>(p.v) + sub * 8;
    table_b = p.page_table + (size_t)b * p.max_pages;
    one_page = (1 << p.page_shift) >= TW;
    const int base0 = t_begin + warp * TW;
    if (one_page && base0 < t_end) pg_next = __ldg(table_b + (base0 >> p.page_shift));
  }
  const int page_mask = (1 << p.page_shift) - 1;
  auto page_row = [&](int pg, int t) -> size_t {
    return ((((size_t)pg * H_kv + h_kv) << p.page_shift) + (t & page_mask)) * D;
  };

  float m = -INFINITY, l = 0.f;
  float o[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) o[i] = 0.f;

  for (int base = t_begin + warp * TW; base < t_end; base += ROWS_PER_ITER) {
    typename IO::W kw[kUnroll], vw[kUnroll];
    bool tok_ok[kUnroll];
    if constexpr (kPaged) {
      if (one_page) {
        const int pg = pg_next;
        // next iteration's entry (clamped to this chunk: always a valid index)
        pg_next = __ldg(table_b + (min(base + ROWS_PER_ITER, t_end - 1) >> p.page_shift));
        const bool page_ok = (unsigned)pg < (unsigned)p.num_pages;
        if (!page_ok && lane == 0) record_device_error(PU_ERR_INVALID_ARGUMENT, kSiteDecodePage);
        const size_t row0 = page_ok ? page_row(pg, base) : 0;
#pragma unroll
        for (int u = 0; u < kUnroll; ++u) {
          tok_ok[u] = page_ok && (base + u * RPW + rw < t_end);
          const size_t off = row0 + (size_t)(u * RPW + rw) * D;
          kw[u] = IO::ld(kb + off, tok_ok[u]);
          vw[u] = IO::ld(vb + off, tok_ok[u]);
        }
      } else {
#pragma unroll
        for (int u = 0; u < kUnroll; ++u) {
          const int t = base + u * RPW + rw;
          int pg = -1;
          if (t < t_end) pg = __ldg(table_b + (t >> p.page_shift));
          tok_ok[u] = (unsigned)pg < (unsigned)p.num_pages;
          if (t < t_end && !tok_ok[u]) record_device_error(PU_ERR_INVALID_ARGUMENT, kSiteDecodePage);
          const size_t off = tok_ok[u] ? page_row(pg, t) : 0;
          kw[u] = IO::ld(kb + off, tok_ok[u]);
          vw[u] = IO::ld(vb + off, tok_ok[u]);
        }
      }
    } else {
#pragma unroll
      for (int u = 0; u < kUnroll; ++u) {
        const int t = base + u * RPW + rw;
        tok_ok[u] = t < t_end;
        kw[u] = IO::ld(kb + (size_t)t * D, tok_ok[u]);
        vw[u] = IO::ld(vb + (size_t)t * D, tok_ok[u]);
      }
    }
    float s[kUnroll];
#pragma unroll
    for (int u = 0; u < kUnroll; ++u) {
      float kf[8];
      IO::unpack(kw[u], kf);
      float acc = 0.f;
#pragma unroll
      for (int i = 0; i < 8; ++i) acc = fmaf(qf[i], kf[i], acc);
      s[u] = acc;
    }
#pragma unroll
    for (int off = LPR / 2; off > 0; off >>= 1) {
#pragma unroll
      for (int u = 0; u < kUnroll; ++u) s[u] += __shfl_xor_sync(0xffffffffu, s[u], off);
    }
    float gmax = -INFINITY;
#pragma unroll
    for (int u = 0; u < kUnroll; ++u) {
      if (!tok_ok[u]) s[u] = -INFINITY;
      gmax = fmaxf(gmax, s[u]);
    }
    const float m_new = fmaxf(m, gmax);
    if (m_new == -INFINITY) continue;  // nothing valid yet in this lane group
    const float alpha = ex2(m - m_new);
    l *= alpha;
#pragma unroll
    for (int i = 0; i < 8; ++i) o[i] *= alpha;
#pragma unroll
    for (int u = 0; u < kUnroll; ++u) {
      const float pu_ = ex2(s[u] - m_new);
      l += pu_;
      float vf[8];
      IO::unpack(vw[u], vf);
#pragma unroll
      for (int i = 0; i < 8; ++i) o[i] = fmaf(pu_, vf[i], o[i]);
    }
    m = m_new;
  }

  // merge the lane groups of this CTA
  const int grp = warp * RPW + rw;
  if (sub == 0) {
    sm_m[grp] = m;
    sm_l[grp] = l;
  }
#pragma unroll
  for (int i = 0; i < 8; ++i) sm_o[grp][sub * 8 + i] = o[i];
  __syncthreads();

  float* rec = p.ws_rec + ((size_t)bh * p.splits + split) * (D + 2);
  if (tid < D) {
    float M = -INFINITY;
#pragma unroll
    for (int g = 0; g < NGROUP; ++g) M = fmaxf(M, sm_m[g]);
    float L = 0.f, O = 0.f;
    if (M != -INFINITY) {
#pragma unroll
      for (int g = 0; g < NGROUP; ++g) {
        const float w = (sm_m[g] == -INFINITY) ? 0.f : ex2(sm_m[g] - M);
        L += w * sm_l[g];
        O += w * sm_o[g][tid];
      }
    }
    rec[2 + tid] = O * p.o_scale;
    if (tid == 0) {
      rec[0] = M;
      rec[1] = L;
    }
  }
  __syncthreads();
  if (tid == 0) {
    // the barrier orders every thread's record stores before this fence, so
    // one device-scope fence publishes the CTA's record before its count
    __threadfence();
    const int prev = atomicAdd(p.ws_count + bh, 1);
    sm_last = (prev == p.splits - 1);
  }
  __syncthreads();
  if (!sm_last) return;
  __threadfence();

  // last CTA of this (b, h): merge every split record
  float M, L, O;
  block_merge<D>(p.ws_rec + (size_t)bh * p.splits * (D + 2), p.splits, M, L, O);
  if (tid < D) {
    if constexpr (kFinal) {
      const float out = (L > 0.f) ? O / L : 0.f;
      p.o[(size_t)bh * D + tid] = __float2bfloat16_rn(out);
      if (tid == 0 && p.lse != nullptr) {
        p.lse[bh] = (L > 0.f) ? (M + lg2(L)) * kLn2 : -INFINITY;
      }
    } else if constexpr (kPush) {
      const float m_nat = (M == -INFINITY) ? -INFINITY : M * kLn2;
      const size_t slot = ((size_t)((p.epoch & 1u) * p.n_peers + p.rank) * gridDim.y + bh) * (D + 2);
#pragma unroll 1
      for (int g = 0; g < p.n_peers; ++g) {
        unsigned long long* out = p.peer_rec[g] + slot;
        st_volatile_u64(out + 2 + tid, ll_word(O, p.epoch));
        if (tid == 0) {
          st_volatile_u64(out, ll_word(m_nat, p.epoch));
          st_volatile_u64(out + 1, ll_word(L, p.epoch));
        }
      }
    } else {
      float* out = p.partial + (size_t)bh * (D + 2);
      out[2 + tid] = O;
      if (tid == 0) {
        out[0] = (M == -INFINITY) ? -INFINITY : M * kLn2;
        out[1] = L;
      }
    }
  }
  if (tid == 0) p.ws_count[bh] = 0;  // leave the workspace zeroed for the next call
  if constexpr (kPush) {
    // fused merge (p.o set): this CTA waits for the other ranks' records of
    // (b, h); the host enables it only while the waiting CTAs (at most B*H)
    // leave most CTA slots free, so every rank's remaining CTAs still run
    if (p.o != nullptr)
      peer_merge<D>(p.peer_rec[p.rank], p.n_peers, gridDim.y, bh, p.epoch, p.timeout_ns, p.o, p.lse, tid);
  }
}

// Merge G gathered shard records {m (natural log), l, o[D]} per (b, h).
template <int D>
__global__ void __launch_bounds__(D) combine_kernel(const float* __restrict__ parts, int G, int BH,
                                                    __nv_bfloat16* __restrict__ o,
                                                    float* __restrict__ lse) {
  const int bh = blockIdx.x;
  const int d = threadIdx.x;
  const size_t stride = (size_t)BH * (D + 2);
  float M = -INFINITY;
  for (int g = 0; g < G; ++g) M = fmaxf(M, parts[g * stride + (size_t)bh * (D + 2)]);
  float L = 0.f, O = 0.f;
  if (M != -INFINITY) {
    for (int g = 0; g < G; ++g) {
      const float* r = parts + g * stride + (size_t)bh * (D + 2);
      if (r[0] == -INFINITY) continue;
      const float w = ex2((r[0] - M) * kLog2e);
      L += w * r[1];
      O += w * r[2 + d];
    }
  }
  o[(size_t)bh * D + d] = __float2bfloat16_rn(L > 0.f ? O / L : 0.f);
  if (d == 0 && lse != nullptr) lse[bh] = (L > 0.f) ? M + logf(L) : -INFINITY;
}

// Workspace layout: [0, kCountBytes) arrival counters, one int per (b, h),
// at a fixed place so that calls of different shapes sharing one workspace
// never see another call's split records as counters; then the records.
constexpr int kMaxBH = 65535;
constexpr size_t kCountBytes = 256 * 1024;  // >= kMaxBH * sizeof(int), 256-aligned

struct Plan {
  int splits;
  int chunk;
  size_t rec_off;      // byte offset of the split records
  size_t total_bytes;
};

inline size_t round_up(size_t x, size_t a) { return (x + a - 1) / a * a; }

// Split plan.  Without per-sequence lengths every (b, h) has the same work:
// exactly one full wave of CTAs (splits = floor(resident CTAs / BH)) streams
// best, since each CTA then pays its start-up and merge once.  With lengths
// (ragged batches) the work per (b, h) is unknown on the host, so chunks are
// finer (about kWaves waves) and CTAs past a sequence's end finish at once.
inline Plan make_plan(long long BH, long long n_local, long long D, int num_sms, bool ragged,
                      long long align = 16) {
  Plan pl{};
  const long long slots = (long long)num_sms * kCtasPerSm;
  long long splits = ragged ? (slots * kWaves + BH - 1) / BH : std::max<long long>(1, slots / BH);
  const long long max_splits = std::max<long long>(1, (n_local + kMinChunk - 1) / kMinChunk);
  splits = std::max<long long>(1, std::min(splits, max_splits));
  long long chunk = (n_local + splits - 1) / splits;
  chunk = std::max<long long>(align, (chunk + align - 1) / align * align);
  splits = std::max<long long>(1, (n_local + chunk - 1) / chunk);
  pl.splits = (int)splits;
  pl.chunk = (int)chunk;
  pl.rec_off = kCountBytes;
  pl.total_bytes = pl.rec_off + round_up((size_t)BH * splits * (D + 2) * sizeof(float), 256);
  return pl;
}

// Workspace that serves a call with or without lengths.
inline size_t workspace_bytes_any(long long BH, long long n_local, long long D, int num_sms) {
  return std::max(make_plan(BH, n_local, D, num_sms, false).total_bytes,
                  make_plan(BH, n_local, D, num_sms, true).total_bytes);
}

// Launch with programmatic stream serialization: the kernel's CTAs may be
// placed on SMs while the previous kernel of the stream finishes (the kernel
// waits in grid_dep_wait before it touches global memory).
template <typename... Args>
inline cudaError_t launch_pdl(void (*kernel)(Args...), dim3 grid, dim3 block, size_t smem, cudaStream_t st,
                              Args... args) {
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kernel, args...);
}

template <bool kFinal, bool kPaged, bool kPush, typename QT, int DD>
int launch_kv(const Params& prm, int kv_dtype, dim3 grid, cudaStream_t st) {
  cudaError_t e;
  if (kv_dtype == PU_DTYPE_F16) {
    e = launch_pdl(split_kv_kernel<QT, __half, DD, kFinal, kPaged, kPush>, grid, dim3(kThreads), 0, st, prm);
  } else if (kv_dtype == PU_DTYPE_BF16) {
    e = launch_pdl(split_kv_kernel<QT, __nv_bfloat16, DD, kFinal, kPaged, kPush>, grid, dim3(kThreads), 0, st, prm);
  } else {
    // fp8 caches are read by the single-GPU final-output step
    if constexpr (kFinal && !kPaged && !kPush) {
      e = launch_pdl(split_kv_kernel<QT, __nv_fp8_e4m3, DD, kFinal, kPaged, kPush>, grid, dim3(kThreads), 0, st,
                     prm);
    } else {
      return set_error(PU_ERR_UNSUPPORTED, "fp8 caches: single-GPU dense decode only");
    }
  }
  return check_cuda(e, "split-KV decode launch");
}

template <bool kFinal, bool kPaged = false, bool kPush = false>
int launch(const Params& prm, int q_dtype, int kv_dtype, int D, int BH, cudaStream_t st) {
  const dim3 grid(prm.splits, BH);
  const bool qh = (q_dtype == PU_DTYPE_F16);
  if (D == 128)
    return qh ? launch_kv<kFinal, kPaged, kPush, __half, 128>(prm, kv_dtype, grid, st)
              : launch_kv<kFinal, kPaged, kPush, __nv_bfloat16, 128>(prm, kv_dtype, grid, st);
  return qh ? launch_kv<kFinal, kPaged, kPush, __half, 64>(prm, kv_dtype, grid, st)
            : launch_kv<kFinal, kPaged, kPush, __nv_bfloat16, 64>(prm, kv_dtype, grid, st);
}

inline int check_args(const void* q, int q_dtype, const void* k, const void* v, int kv_dtype,
                      long long B, long long H, long long n, long long D, bool allow_fp8 = false) {
  if (allow_fp8 && kv_dtype == PU_DTYPE_FP8_E4M3) kv_dtype = PU_DTYPE_F16;  // same checks otherwise
  if (!q || !k || !v) return set_error(PU_ERR_INVALID_ARGUMENT, "null q/k/v pointer");
  if (B <= 0 || H <= 0 || n <= 0) return set_error(PU_ERR_INVALID_ARGUMENT, "B, H and the cache length must be positive");
  if (D != 128 && D != 64) return set_error(PU_ERR_UNSUPPORTED, "decode head size %lld (supported: 64, 128)", D);
  if ((q_dtype != PU_DTYPE_F16 && q_dtype != PU_DTYPE_BF16) ||
      (kv_dtype != PU_DTYPE_F16 && kv_dtype != PU_DTYPE_BF16))
    return set_error(PU_ERR_UNSUPPORTED, "decode dtypes must be f16 or bf16");
  if (!aligned16(q) || !aligned16(k) || !aligned16(v))
    return set_error(PU_ERR_INVALID_ARGUMENT, "q/k/v must be 16-byte aligned");
  if (B * H > kMaxBH) return set_error(PU_ERR_UNSUPPORTED, "B*H = %lld exceeds %d", B * H, kMaxBH);
  if (n > (1ll << 30)) return set_error(PU_ERR_UNSUPPORTED, "cache length too large");
  return PU_OK;
}

}  // namespace decode
}  // namespace pu

extern "C" {

size_t pu_decode_workspace_size(int64_t B, int64_t H, int64_t n_local, int64_t D) {
  if (B <= 0 || H <= 0 || n_local <= 0 || D <= 0) return 0;
  return pu::decode::workspace_bytes_any(B * H, n_local, D, pu::sm_count());
}

int pu_decode_partial(const void* q, int q_dtype, const void* k_cache, const void* v_cache,
                      int kv_dtype, const int32_t* kv_lens, int64_t kv_offset, float* partial,
                      void* workspace, size_t workspace_bytes, int64_t B, int64_t H,
                      int64_t n_local, int64_t D, float sm_scale, void* stream) {
  using namespace pu::decode;
  int rc = check_args(q, q_dtype, k_cache, v_cache, kv_dtype, B, H, n_local, D);
  if (rc) return rc;
  if (!partial) return pu::set_error(PU_ERR_INVALID_ARGUMENT, "null partial output");
  if (kv_offset < 0) return pu::set_error(PU_ERR_INVALID_ARGUMENT, "negative kv_offset");
  const Plan pl = make_plan(B * H, n_local, D, pu::sm_count(), kv_lens != nullptr);
  if (!workspace || workspace_bytes < pl.total_bytes)
    return pu::set_error(PU_ERR_WORKSPACE, "decode workspace needs %zu bytes, got %zu", pl.total_bytes,
                         workspace_bytes);
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
  prm.partial = partial;
  return launch<false>(prm, q_dtype, kv_dtype, (int)D, (int)(B * H), static_cast<cudaStream_t>(stream));
}

int pu_decode(const void* q, int q_dtype, const void* k_cache, const void* v_cache, int kv_dtype,
              const int32_t* kv_lens, void* o, float* lse, void* workspace, size_t workspace_bytes,
              int64_t B, int64_t H, int64_t n, int64_t D, float sm_scale, void* stream) {
  using namespace pu::decode;
  int rc = check_args(q, q_dtype, k_cache, v_cache, kv_dtype, B, H, n, D);
  if (rc) return rc;
  if (!o) return pu::set_error(PU_ERR_INVALID_ARGUMENT, "null output");
  const Plan pl = make_plan(B * H, n, D, pu::sm_count(), kv_lens != nullptr);
  if (!workspace || workspace_bytes < pl.total_bytes)
    return pu::set_error(PU_ERR_WORKSPACE, "decode workspace needs %zu bytes, got %zu", pl.total_bytes,
                         workspace_bytes);
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
  prm.ws_rec = reinterpret_cast<float*>(static_cast<char*>(workspace) + pl.rec_off);
  prm.ws_count = static_cast<int*>(workspace);
  prm.o = static_cast<__nv_bfloat16*>(o);
  prm.lse = lse;
  return launch<true>(prm, q_dtype, kv_dtype, (int)D, (int)(B * H), static_cast<cudaStream_t>(stream));
}

int pu_decode_combine(const float* partials, int64_t G, void* o, float* lse, int64_t B, int64_t H,
                      int64_t D, void* stream) {
  using namespace pu::decode;
  if (!partials || !o) return pu::set_error(PU_ERR_INVALID_ARGUMENT, "null partials/output");
  if (G <= 0 || B <= 0 || H <= 0) return pu::set_error(PU_ERR_INVALID_ARGUMENT, "G, B, H must be positive");
  if (D != 128 && D != 64) return pu::set_error(PU_ERR_UNSUPPORTED, "combine head size %lld", (long long)D);
  const int BH = (int)(B * H);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (D == 128)
    combine_kernel<128><<<BH, 128, 0, st>>>(partials, (int)G, BH, static_cast<__nv_bfloat16*>(o), lse);
  else
    combine_kernel<64><<<BH, 64, 0, st>>>(partials, (int)G, BH, static_cast<__nv_bfloat16*>(o), lse);
  return pu::check_cuda(cudaGetLastError(), "decode combine launch");
}


}  // extern "C"
