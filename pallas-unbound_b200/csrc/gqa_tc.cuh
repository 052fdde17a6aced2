// gqa_tc.cuh — grouped-head split-KV decode on the tensor core (D = 128,
// q and cache of one 16-bit type, G = H / H_kv >= 2 query heads per K/V head).
//
// No counterpart in the reference (one K/V head per query head;
// src/pallas_flash/kernels/decoding.py:105-115 is the per-head math).  One
// CTA per (split, b, K/V head, slice of at most 16 query heads) streams its
// chunk of the cache once, in tiles of 128 rows, and computes the heads of
// its slice:
//
//   S   [128 rows x 16 heads] = K_tile · Qsᵀ      A = K tile (K-major), B = the
//                                                slice's queries, zero-padded
//   Oᵀ  [128 dims x 16 heads] += V_tileᵀ · Pᵀ     A = V tile read MN-major,
//                                                B = Pᵀ (heads x rows, K-major)
//
// so the rows of the tile are the MMA's M and the heads its N: ~4·16·D flops
// per cache row, far below what HBM delivers — the kernel is bound by the
// K/V stream.  The slices of one K/V head are neighbouring CTAs that read the
// same tiles at the same time (the repeats come from L2).
//
// Roles (256 threads):
//   warp 4 lane 0  TMA producer: K and V tiles (2 x 16 KB boxes each) into an
//                  NS-deep ring, one full/empty barrier pair per stage
//   warp 5 lane 0  tcgen05 issuer: S_j as soon as tile j has landed (and
//                  its S buffer is free), Oᵀ += V_jᵀ·P_jᵀ as soon as P_j is
//                  written, whichever comes first; warp 5 also owns the
//                  TMEM allocation
//   warps 0-3      row r of the tile = TMEM lane r = thread r: scores in
//                  log2 units, a running maximum per head shared by the CTA
//                  that moves only when a score exceeds it by more than 8
//                  (then Oᵀ and the partial sums are rescaled), P = 2^(s-m)
//                  written as 16-bit into shared memory, partial sums l per
//                  thread; at the end thread d reads row d of Oᵀ and the
//                  split record of every head is written
//   all            the last CTA of a (b, K/V head, slice) merges the split
//                  records of its heads at once, 32 records per L2 round trip
//
// The launch allows programmatic dependent launch: the first global access
// of every CTA follows grid_dep_wait, so the CTAs may be placed on SMs as
// the previous kernel's CTAs leave, and the barriers, TMEM and the first
// ring of K/V loads are set up before the queries arrive.
//
// TMEM (64 columns): S_0 [0,16), S_1 [16,32), Oᵀ [32,48).  e4m3 caches (256
// columns): S_0 [0,48) and S_1 [48,96), each the scores of the three query
// parts side by side, and Oᵀ of P part k at [96 + 16 k, 112 + 16 k); the
// products run with N = 48 over the three parts stacked in shared memory
// (one instruction where three N = 16 ones would cost three times the issue).
// Rows past the chunk's end inside the last tile are masked to -inf; their V
// rows are zeroed in shared memory before the P·V product (so stale cache
// contents cannot reach the output).  Every wait is bounded; the softmax
// warps run the same barrier sequence whatever a wait returns, so a timeout
// ends the kernel with PU_ERR_DEVICE_TIMEOUT (detail 305) instead of a hang.
#pragma once

#include <algorithm>
#include <type_traits>

#include "gqa.cuh"

namespace pu {
namespace decode {
namespace tc {

constexpr int BT = 128;                    // cache rows per tile (MMA M)
constexpr int kDim = 128;                  // head size
constexpr int NS = 3;                      // K/V ring depth
constexpr int kTileBytes = BT * kDim * 2;  // one K or V tile
constexpr float kRescaleLog2 = 8.f;
constexpr int kMergeBatch = 32;            // split records per L2 round trip of the merge
static_assert(kThreads == 256, "the softmax warps are 0-3, producer 4, issuer 5");

// Cache tiles of one element type: 16-bit tiles are two 64-column swizzle
// blocks (32 KB), e4m3 tiles one 128-column block (16 KB).  A 16-bit CTA
// takes an SM (192 KB ring).  e4m3 CTAs either take an SM with a 6-stage
// ring or, with kF8CtasPerSm = 2, share one with 2-stage rings (two CTAs of
// 3 stages would need 2 x 115 KB) so their per-tile chains (products,
// softmax, products) interleave.
constexpr int kF8CtasPerSm = 1;

template <typename KVT>
struct Ring {
  static constexpr int kTileBytes = BT * kDim * (int)sizeof(KVT);
  static constexpr int NS = sizeof(KVT) == 1 ? (kF8CtasPerSm == 1 ? 6 : 2) : 3;
};

// Shared memory.  16-bit: the query group [NP x 128] and each Pᵀ buffer
// [NP x 128 rows] are two 64-column blocks.  fp8: kParts e4m3 parts (one
// 128-column block each) of the scaled queries and of each Pᵀ, whose sum
// carries about 12 significant bits, the precision of f16.
constexpr int kParts = 3;

template <int NP, typename KVT = __half>
struct Cfg {
  static constexpr int NS = Ring<KVT>::NS;
  static constexpr int kBlock = NP * 128;                  // bytes of one swizzle block of NP rows
  static constexpr int kQBytes = (sizeof(KVT) == 1 ? kParts : 2) * kBlock;
  static constexpr int kPBytes = (sizeof(KVT) == 1 ? kParts : 2) * kBlock;
  static constexpr int kOffQ = 0;
  static constexpr int kOffP = kOffQ + kQBytes;            // two buffers
  static constexpr int kOffKV = kOffP + 2 * kPBytes;       // stage s: K, then V
  static constexpr int kOffBar = kOffKV + NS * 2 * Ring<KVT>::kTileBytes;
  // full[NS], empty[NS], s_full[2], p_full[2], p_free[2], drain
  static constexpr int kNumBars = 2 * NS + 7;
  static constexpr int kOffMisc = kOffBar + kNumBars * 8;  // tmem base, abort flag, last-CTA flag
  static constexpr int kOffRed = kOffMisc + 16;            // [4][NP] floats
  static constexpr int kOffQinv = kOffRed + 4 * NP * 4;    // fp8: [NP] per-head factor undoing the query scale
  static constexpr int kSmemBytes = kOffQinv + NP * 4;
  // S_0, S_1, then one O^T accumulator (16-bit) or kParts of them (e4m3: one
  // per P part, combined with weights kPartScale^-part at the end).  e4m3:
  // each S buffer holds the scores of the kParts query parts side by side
  // (kParts x NP columns, summed by the softmax warps), and the products run
  // with N = kParts x NP over the parts stacked in shared memory.
  static constexpr int kSCols = (sizeof(KVT) == 1 ? kParts : 1) * NP;
  static constexpr uint32_t kColO = 2 * kSCols;
  static constexpr uint32_t kTmemCols = sizeof(KVT) == 1 ? 256 : (NP <= 16 ? 64 : 128);
  static_assert(kColO + (sizeof(KVT) == 1 ? kParts : 1) * NP <= kTmemCols, "TMEM columns");
  static_assert(kOffP % 1024 == 0 && kPBytes % 1024 == 0 && kOffKV % 1024 == 0,
                "swizzled operands start on 1024-byte boundaries");
};

template <int NP>
__device__ __forceinline__ void tmem_ld_np(uint32_t taddr, uint32_t (&r)[NP]) {
  if constexpr (NP == 16) tmem_ld16(taddr, r);
  else tmem_ld32(taddr, r);
}

template <int NP>
__device__ __forceinline__ void tmem_st_np(uint32_t taddr, const uint32_t (&r)[NP]) {
  if constexpr (NP == 16) tmem_st16(taddr, r);
  else tmem_st32(taddr, r);
}

// (a, b) as kParts e4m3 pairs: part i is the e4m3 rounding (saturating) of
// what the previous parts left, multiplied by kPartScale^i when `scaled` (so
// a remainder stays in e4m3's normal range instead of its 2^-9-step
// subnormals), so (a, b) ~ sum_i part_i / kPartScale^i (scaled) or
// sum_i part_i.
constexpr float kPartScale = 16.f;

template <bool scaled>
__device__ __forceinline__ void split_e4m3(float a, float b, uint16_t (&part)[kParts]) {
#pragma unroll
  for (int i = 0; i < kParts; ++i) {
    const __nv_fp8x2_storage_t h2 = __nv_cvt_float2_to_fp8x2(make_float2(a, b), __NV_SATFINITE, __NV_E4M3);
    part[i] = (uint16_t)h2;
    if (i + 1 < kParts) {
      const float2 hf = __half22float2(__half2(__nv_cvt_fp8x2_to_halfraw2(h2, __NV_E4M3)));
      a -= hf.x;
      b -= hf.y;
      if (scaled) {
        a *= kPartScale;
        b *= kPartScale;
      }
    }
  }
}

template <typename T>
__device__ __forceinline__ uint16_t to16(float x);
template <>
__device__ __forceinline__ uint16_t to16<__half>(float x) { return __half_as_ushort(__float2half_rn(x)); }
template <>
__device__ __forceinline__ uint16_t to16<__nv_bfloat16>(float x) {
  return __bfloat16_as_ushort(__float2bfloat16_rn(x));
}

// A group of more than NP query heads is cut into ceil(G / NP) slices of at
// most NP heads, one CTA per slice; the CTAs of one (split, b, K/V head) are
// neighbours in the grid and read the same K/V tiles at the same time, so
// all but the first read come from L2.  The per-head loops run over NP with
// the heads past the slice skipped.
template <typename T, typename KVT, int NP>
__global__ void __launch_bounds__(kThreads, 1)
    gqa_tc_kernel(const __grid_constant__ CUtensorMap tmK, const __grid_constant__ CUtensorMap tmV,
                  const Params p) {
  using C = Cfg<NP, KVT>;
  constexpr int NS = C::NS;
  constexpr int kTileBytes = Ring<KVT>::kTileBytes;
  constexpr bool kF8 = sizeof(KVT) == 1;
  static_assert(!kF8 || NP == 16, "fp8 caches use 16-head slices");
  static_assert(NP == 16 || NP == 32, "padded group size");
  const int Gt = p.group;                       // query heads per K/V head
  const int n_slices = (Gt + NP - 1) / NP;
  const int slice = (int)blockIdx.x % n_slices;
  const int G = min(NP, Gt - slice * NP);       // this CTA's query heads
  extern __shared__ __align__(1024) uint8_t smem[];
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  if (smem_u32(smem) & 1023u) {
    if (tid == 0) record_device_error(PU_ERR_UNSUPPORTED, kSiteDecodeTc);
    return;
  }
  uint8_t* sQ = smem + C::kOffQ;
  uint8_t* sP = smem + C::kOffP;
  uint8_t* sKV = smem + C::kOffKV;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + C::kOffBar);
  uint64_t* bFull = bars;
  uint64_t* bEmpty = bFull + NS;
  uint64_t* bSf = bEmpty + NS;     // [2] S_j in TMEM
  uint64_t* bPf = bSf + 2;         // [2] P_j in shared memory (128 arrivals)
  uint64_t* bPfree = bPf + 2;      // [2] P_j·V_j done (P buffer free, Oᵀ settled)
  uint64_t* bDrain = bPfree + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + C::kOffMisc);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + C::kOffMisc + 4);
  int* sm_last = reinterpret_cast<int*>(smem + C::kOffMisc + 8);
  float* sm_red4 = reinterpret_cast<float*>(smem + C::kOffRed);

  const int split = (int)blockIdx.x / n_slices;
  const int bkv = blockIdx.y;                   // b * H_kv + K/V head
  const int H_kv = p.H / Gt;
  const int b = bkv / H_kv;
  const int bh0 = b * p.H + (bkv % H_kv) * Gt + slice * NP;   // this CTA's first query head
  int len = p.n_local;
  if (p.lens != nullptr) {
    const long long g = (long long)p.lens[b];
    len = g < 0 ? 0 : (g > p.n_local ? p.n_local : (int)g);
  }
  const int t_begin = split * p.chunk;
  const int t_end = min(t_begin + p.chunk, len);
  const int n_tiles = t_end > t_begin ? (t_end - t_begin + BT - 1) / BT : 0;

  // The producer sets up the barriers and puts the first ring of K/V loads
  // in flight before anything else, so the first tiles travel while the
  // queries are staged.  Nothing in global memory (q, the cache, the lengths
  // or the workspace) is touched before grid_dep_wait: the launch may begin
  // while the previous kernel of the stream is still finishing.
  constexpr int kProducer = 4 * 32;
  if (tid == kProducer) {
    for (int s = 0; s < NS; ++s) {
      mbar_init(bFull + s, 1);
      mbar_init(bEmpty + s, 1);
    }
    for (int t = 0; t < 2; ++t) {
      mbar_init(bSf + t, 1);
      mbar_init(bPf + t, 128);
      mbar_init(bPfree + t, 1);
    }
    mbar_init(bDrain, 1);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 5) {
    tmem_alloc(tmem_slot, C::kTmemCols);
    tmem_relinquish();
  }
  grid_dep_wait();
  grid_dep_launch_dependents();
  const int n_first = min(NS, n_tiles);
  auto issue_tile = [&](int i) {
    const int s = i % NS;
    uint8_t* dK = sKV + s * 2 * kTileBytes;
    uint8_t* dV = dK + kTileBytes;
    const int row = t_begin + i * BT;
    mbar_arrive_expect_tx(bFull + s, 2 * kTileBytes);
    if constexpr (kF8) {
      tma_load_3d(dK, &tmK, bFull + s, 0, row, bkv);
      tma_load_3d(dV, &tmV, bFull + s, 0, row, bkv);
    } else {
      for (int cb = 0; cb < 2; ++cb) tma_load_3d(dK + cb * BT * 128, &tmK, bFull + s, cb * 64, row, bkv);
      for (int cb = 0; cb < 2; ++cb) tma_load_3d(dV + cb * BT * 128, &tmV, bFull + s, cb * 64, row, bkv);
    }
  };
  if (tid == kProducer) {
    tma_prefetch_desc(&tmK);
    tma_prefetch_desc(&tmV);
    for (int i = 0; i < n_first; ++i) issue_tile(i);
  }

  // query group -> sQ (K-major, 128-byte swizzle; rows G..NP-1 zero); both
  // Pᵀ buffers zeroed (rows G..NP-1 are never written afterwards)
  float* s_qinv = reinterpret_cast<float*>(smem + C::kOffQinv);
  if constexpr (kF8) {
    // head n = tid / 16, elements 8*cr .. 8*cr+7: scaled by a power of two so
    // the head's largest |q| lands in [128, 256), then split into kParts
    // e4m3 parts
    const int n = tid >> 4, cr = tid & 15;
    float x[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) x[i] = 0.f;
    if (n < G) {
      const uint4 w = *reinterpret_cast<const uint4*>(static_cast<const T*>(p.q) + (size_t)(bh0 + n) * kDim + cr * 8);
      unpack8<T>(w, x);
    }
    float mx = 0.f;
#pragma unroll
    for (int i = 0; i < 8; ++i) mx = fmaxf(mx, fabsf(x[i]));
#pragma unroll
    for (int off = 8; off > 0; off >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, off));
    const int e = (mx > 0.f && isfinite(mx)) ? ((__float_as_int(mx) >> 23) & 0xff) - 127 : 7;
    const int sh = max(-100, min(100, 7 - e));
    const float up = __int_as_float((127 + sh) << 23), down = __int_as_float((127 - sh) << 23);
    uint32_t w[kParts][2];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      uint16_t pr[kParts];
      split_e4m3<false>(x[2 * i] * up, x[2 * i + 1] * up, pr);
#pragma unroll
      for (int k = 0; k < kParts; ++k)
        w[k][i >> 1] = (i & 1) ? (w[k][i >> 1] | ((uint32_t)pr[k] << 16)) : (uint32_t)pr[k];
    }
    const int off = n * 128 + ((((cr >> 1) ^ (n & 7))) << 4) + (cr & 1) * 8;
#pragma unroll
    for (int k = 0; k < kParts; ++k) *reinterpret_cast<uint2*>(sQ + k * C::kBlock + off) = make_uint2(w[k][0], w[k][1]);
    if (cr == 0) s_qinv[n] = n < G ? down : 0.f;
  } else {
    for (int c = tid; c < NP * 16; c += kThreads) {
      const int n = c >> 4, cr = c & 15, cb = cr >> 3, ch = cr & 7;
      uint4 w = make_uint4(0u, 0u, 0u, 0u);
      if (n < G) w = *reinterpret_cast<const uint4*>(static_cast<const T*>(p.q) + (size_t)(bh0 + n) * kDim + cr * 8);
      *reinterpret_cast<uint4*>(sQ + cb * C::kBlock + n * 128 + ((ch ^ (n & 7)) << 4)) = w;
    }
  }
  for (int c = tid; c < 2 * C::kPBytes / 16; c += kThreads)
    reinterpret_cast<uint4*>(sP)[c] = make_uint4(0u, 0u, 0u, 0u);
  fence_proxy_async_smem();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const uint32_t col_o = C::kColO;

  if (warp == 4) {
    // ---------------- TMA producer ----------------
    if (lane == 0 && n_tiles > 0) {
      int issued = n_first;                     // the first ring went out in the prologue
      for (int i = n_first; i < n_tiles; ++i) {
        if (!mbar_wait(bEmpty + i % NS, (i / NS - 1) & 1, abort_flag, kSiteDecodeTc)) break;
        issue_tile(i);
        ++issued;
      }
      // copies still in flight land before the CTA may exit
      volatile int no_abort = 0;
      for (int i = max(0, issued - NS); i < issued; ++i)
        mbar_wait(bFull + i % NS, (i / NS) & 1, &no_abort, kSiteDecodeTc);
    }
  } else if (warp == 5) {
    // ---------------- tcgen05 issuer ----------------
    if (lane == 0) {
      constexpr bool kBf16 = std::is_same<T, __nv_bfloat16>::value;
      constexpr uint32_t idS = kF8 ? make_idesc_e4m3(BT, kParts * NP, 0, 0) : make_idesc_16(BT, NP, 0, 0, kBf16);
      constexpr uint32_t idO = kF8 ? make_idesc_e4m3(kDim, kParts * NP, 1, 0) : make_idesc_16(kDim, NP, 1, 0, kBf16);
      const uint64_t dQ = make_sdesc_sw128(smem_u32(sQ), 16, 1024);
      const uint64_t dP0 = make_sdesc_sw128(smem_u32(sP), 16, 1024);
      const uint64_t dK0 = make_sdesc_sw128(smem_u32(sKV), 16, 1024);
      const uint64_t dV0 = make_sdesc_sw128(smem_u32(sKV + kTileBytes), BT * 128, 1024);
      auto issue_S = [&](int j) {                // S_{j} into buffer j & 1 from stage j % NS
        const uint64_t dk = sdesc_add(dK0, (j % NS) * 2 * kTileBytes);
        if constexpr (kF8) {
          // [S_part0 | S_part1 | S_part2] = K (query parts stacked, N = kParts x NP)^T:
          // four K = 32 steps
#pragma unroll
          for (int kk = 0; kk < 4; ++kk)
            mma_ss_f8(tmem + (j & 1) * C::kSCols, sdesc_add(dk, kk * 32), sdesc_add(dQ, kk * 32), idS, kk > 0);
        } else {
#pragma unroll
          for (int kk = 0; kk < kDim / 16; ++kk) {
            const uint32_t offk = (kk >> 2) * (BT * 128) + (kk & 3) * 32;
            const uint32_t offq = (kk >> 2) * C::kBlock + (kk & 3) * 32;
            mma_ss(tmem + (j & 1) * C::kSCols, sdesc_add(dk, offk), sdesc_add(dQ, offq), idS, kk > 0);
          }
        }
        mma_commit(bSf + (j & 1));
      };
      // S_js and P_jp·V_jp are issued as soon as each is ready (polling both
      // barriers), so a tile still in flight never holds back the P·V product
      // that frees an earlier stage.  S_js overwrites S buffer js & 1, free
      // once P_{js-2} was written, i.e. once P_{js-2}·V was issued: js <= jp + 1.
      int js = 0, jp = 0;
      uint64_t t_last = global_timer_ns();
      while (jp < n_tiles) {
        bool progressed = false;
        if (js < n_tiles && js <= jp + 1 && mbar_try_wait(smem_u32(bFull + js % NS), (js / NS) & 1)) {
          tc_fence_after();
          issue_S(js);
          ++js;
          progressed = true;
        }
        if (jp < js && mbar_try_wait(smem_u32(bPf + (jp & 1)), (jp >> 1) & 1)) {
          tc_fence_after();
          const uint64_t dv = sdesc_add(dV0, (jp % NS) * 2 * kTileBytes);
          const uint64_t dp = sdesc_add(dP0, (jp & 1) * C::kPBytes);
          if constexpr (kF8) {
            // [O_part0 | O_part1 | O_part2]^T += V^T (P parts stacked, N = kParts x
            // NP)^T: the V tile read MN-major (d = M, one 128-byte block), 32
            // cache rows per step
#pragma unroll
            for (int kk = 0; kk < 4; ++kk)
              mma_ss_f8(tmem + col_o, sdesc_add(dv, kk * 32 * 128), sdesc_add(dp, kk * 32), idO, (jp > 0 || kk > 0));
          } else {
#pragma unroll
            for (int kk = 0; kk < BT / 16; ++kk) {
              const uint32_t offp = (kk >> 2) * C::kBlock + (kk & 3) * 32;
              mma_ss(tmem + col_o, sdesc_add(dv, kk * 16 * 128), sdesc_add(dp, offp), idO, (jp > 0 || kk > 0));
            }
          }
          mma_commit(bPfree + (jp & 1));
          mma_commit(bEmpty + jp % NS);
          ++jp;
          progressed = true;
        }
        if (progressed) {
          t_last = global_timer_ns();
        } else {
          if (*abort_flag) break;
          if (global_timer_ns() - t_last > kWaitTimeoutNs) {
            *abort_flag = 1;
            record_device_error(PU_ERR_DEVICE_TIMEOUT, kSiteDecodeTc);
            break;
          }
        }
      }
      // every issued product completes before TMEM and shared memory go away
      mma_commit(bDrain);
      volatile int no_abort = 0;
      mbar_wait(bDrain, 0, &no_abort, kSiteDecodeTc);
    }
  } else if (warp < 4) {
    // ---------------- rows / heads (warps 0-3) ----------------
    const uint32_t lane_base = static_cast<uint32_t>(warp * 32) << 16;
    float m_run[NP], l_part[NP];
#pragma unroll
    for (int h = 0; h < NP; ++h) {
      m_run[h] = -INFINITY;
      l_part[h] = 0.f;
    }
    const int kb = tid >> 6, kc = tid & 63;       // this row's place in a Pᵀ row
    const uint32_t p_off = kb * C::kBlock + (kc & 7) * 2;
    float qf[NP];                                 // fp8: undoes the per-head query scale
#pragma unroll
    for (int h = 0; h < NP; ++h) qf[h] = kF8 ? s_qinv[h] * p.scale_log2 : p.scale_log2;
    for (int j = 0; j < n_tiles; ++j) {
      const int buf = j & 1;
      mbar_wait(bSf + buf, (j >> 1) & 1, abort_flag, kSiteDecodeTc);
      __syncwarp();
      tc_fence_after();
      float raw[NP];
      if constexpr (kF8) {
        // the query parts' scores side by side: summed in part order
        uint32_t r0[NP], r1[NP], r2[NP];
        static_assert(kParts == 3, "three query parts");
        tmem_ld_np<NP>(tmem + lane_base + buf * C::kSCols, r0);
        tmem_ld_np<NP>(tmem + lane_base + buf * C::kSCols + NP, r1);
        tmem_ld_np<NP>(tmem + lane_base + buf * C::kSCols + 2 * NP, r2);
        tmem_wait_ld();
        reg_fence(r0);
        reg_fence(r1);
        reg_fence(r2);
#pragma unroll
        for (int h = 0; h < NP; ++h)
          raw[h] = (__uint_as_float(r0[h]) + __uint_as_float(r1[h])) + __uint_as_float(r2[h]);
      } else {
        uint32_t r[NP];
        tmem_ld_np<NP>(tmem + lane_base + buf * C::kSCols, r);
        tmem_wait_ld();
        reg_fence(r);
#pragma unroll
        for (int h = 0; h < NP; ++h) raw[h] = __uint_as_float(r[h]);
      }
      const int tile0 = t_begin + j * BT;
      const bool valid = tile0 + tid < t_end;
      float s[NP];
      bool up = false;
#pragma unroll
      for (int h = 0; h < NP; ++h) {
        s[h] = valid ? raw[h] * qf[h] : -INFINITY;
        if (h < G) up |= s[h] > m_run[h] + kRescaleLog2;
      }
      if (bar_any_named(1, 128, up)) {
        // the tile's maximum of each head over all 128 rows
#pragma unroll
        for (int h = 0; h < NP; ++h) {
          if (h >= G) break;
          float v = s[h];
#pragma unroll
          for (int off = 16; off > 0; off >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, off));
          if (lane == 0) sm_red4[warp * NP + h] = v;
        }
        bar_sync_named(1, 128);
        float alpha[NP];
#pragma unroll
        for (int h = 0; h < NP; ++h) {
          alpha[h] = 1.f;
          if (h >= G) continue;
          const float tm = fmaxf(fmaxf(sm_red4[h], sm_red4[NP + h]), fmaxf(sm_red4[2 * NP + h], sm_red4[3 * NP + h]));
          if (tm > m_run[h] + kRescaleLog2) {      // same decision in every thread
            alpha[h] = (m_run[h] == -INFINITY) ? 0.f : ex2(m_run[h] - tm);
            m_run[h] = tm;
          }
          l_part[h] *= alpha[h];
        }
        if (j > 0) {
          // Oᵀ holds tiles < j once P_{j-1}·V_{j-1} is done; row tid of Oᵀ is
          // this thread's TMEM lane
          mbar_wait(bPfree + ((j - 1) & 1), ((j - 1) >> 1) & 1, abort_flag, kSiteDecodeTc);
          __syncwarp();
          tc_fence_after();
#pragma unroll
          for (int part = 0; part < (kF8 ? kParts : 1); ++part) {
            uint32_t ov[NP];
            tmem_ld_np<NP>(tmem + lane_base + col_o + part * NP, ov);
            tmem_wait_ld();
            reg_fence(ov);
#pragma unroll
            for (int h = 0; h < NP; ++h) ov[h] = __float_as_uint(__uint_as_float(ov[h]) * alpha[h]);
            tmem_st_np<NP>(tmem + lane_base + col_o + part * NP, ov);
          }
          tmem_wait_st();
        }
      }
      // the last tile: rows past the chunk's end get zero V rows
      if (!valid) {
        mbar_wait(bFull + j % NS, (j / NS) & 1, abort_flag, kSiteDecodeTc);
        uint8_t* vrow = sKV + (j % NS) * 2 * kTileBytes + kTileBytes + tid * 128;
#pragma unroll
        for (int cb = 0; cb < (kF8 ? 1 : 2); ++cb)
#pragma unroll
          for (int c = 0; c < 8; ++c)
            reinterpret_cast<uint4*>(vrow + cb * BT * 128)[c] = make_uint4(0u, 0u, 0u, 0u);
      }
      // P_j into buffer `buf` once P_{j-2}·V_{j-2} has read it
      if (j >= 2) mbar_wait(bPfree + buf, ((j - 2) >> 1) & 1, abort_flag, kSiteDecodeTc);
      if constexpr (kF8) {
        // P (<= 2^8) as kParts e4m3 parts; row h of each part, byte `tid` of
        // that row (128-byte swizzle)
        uint8_t* pb = sP + buf * C::kPBytes + (tid & 15);
        const int chunk = tid >> 4;
#pragma unroll
        for (int h = 0; h < NP; h += 2) {
          if (h >= G) break;
          const float p0 = ex2(s[h] - m_run[h]);   // 0 for masked rows
          const float p1 = (h + 1 < G) ? ex2(s[h + 1] - m_run[h + 1]) : 0.f;
          l_part[h] += p0;
          if (h + 1 < G) l_part[h + 1] += p1;
          uint16_t pr[kParts];
          split_e4m3<true>(p0, p1, pr);
          const int o0 = h * 128 + ((chunk ^ (h & 7)) << 4), o1 = (h + 1) * 128 + ((chunk ^ ((h + 1) & 7)) << 4);
#pragma unroll
          for (int k = 0; k < kParts; ++k) {
            pb[k * C::kBlock + o0] = (uint8_t)(pr[k] & 0xff);
            pb[k * C::kBlock + o1] = (uint8_t)(pr[k] >> 8);
          }
        }
      } else {
        uint8_t* pb = sP + buf * C::kPBytes + p_off;
#pragma unroll
        for (int h = 0; h < NP; ++h) {
          if (h >= G) break;
          const float pr = ex2(s[h] - m_run[h]);     // 0 for masked rows
          l_part[h] += pr;
          *reinterpret_cast<uint16_t*>(pb + h * 128 + (((kc >> 3) ^ (h & 7)) << 4)) = to16<T>(pr);
        }
      }
      fence_proxy_async_smem();
      tc_fence_before();
      mbar_arrive(bPf + buf);
      __syncwarp();
    }

    // split record of every head: m (log2 units), l, o[d] (thread d)
    float o[NP];
#pragma unroll
    for (int h = 0; h < NP; ++h) o[h] = 0.f;
    if (n_tiles > 0) {
      mbar_wait(bPfree + ((n_tiles - 1) & 1), ((n_tiles - 1) >> 1) & 1, abort_flag, kSiteDecodeTc);
      __syncwarp();
      tc_fence_after();
      float w = 1.f;
#pragma unroll
      for (int part = 0; part < (kF8 ? kParts : 1); ++part, w *= 1.f / kPartScale) {
        uint32_t ov[NP];
        tmem_ld_np<NP>(tmem + lane_base + col_o + part * NP, ov);
        tmem_wait_ld();
        reg_fence(ov);
#pragma unroll
        for (int h = 0; h < NP; ++h) o[h] = fmaf(__uint_as_float(ov[h]), w, o[h]);
      }
    }
#pragma unroll
    for (int h = 0; h < NP; ++h) {
      if (h >= G) break;
      float v = l_part[h];
#pragma unroll
      for (int off = 16; off > 0; off >>= 1) v += __shfl_xor_sync(0xffffffffu, v, off);
      if (lane == 0) sm_red4[warp * NP + h] = v;
    }
    bar_sync_named(1, 128);
#pragma unroll
    for (int h = 0; h < NP; ++h) {
      if (h >= G) break;
      float* rec = p.ws_rec + ((size_t)(bh0 + h) * p.splits + split) * (kDim + 2);
      rec[2 + tid] = o[h] * p.o_scale;
      if (tid == 0) {
        rec[0] = m_run[h];
        rec[1] = (sm_red4[h] + sm_red4[NP + h]) + (sm_red4[2 * NP + h] + sm_red4[3 * NP + h]);
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 5) {
    tc_fence_after();
    tmem_dealloc(tmem, C::kTmemCols);
  }
  if (tid == 0) {
    // the barrier orders every thread's record stores before this fence, so
    // one device-scope fence publishes the CTA's records before its count
    __threadfence();
    const int prev = atomicAdd(p.ws_count + bkv * n_slices + slice, 1);
    *sm_last = (prev == p.splits - 1);
  }
  __syncthreads();
  if (!*sm_last) return;
  __threadfence();
  // last CTA of this (b, K/V head, slice): merge the split records of its G
  // query heads.  Thread i takes outputs (h, d) and (h, d + 64) of head h =
  // i / 64; it reads the records kMergeBatch at a time with every load of a
  // batch in flight together (one L2 round trip per batch) and folds them,
  // in record order, into a running maximum and running sums.
  const int S = p.splits;
  const float* recs = p.ws_rec + (size_t)bh0 * S * (kDim + 2);
  constexpr int kHalf = kDim / 2;
  for (int pi = tid; pi < G * kHalf; pi += kThreads) {
    const int h = pi / kHalf, d = pi % kHalf;
    const float* rh = recs + (size_t)h * S * (kDim + 2);
    float mx = -INFINITY, ls = 0.f, oa = 0.f, ob = 0.f;
    for (int s0 = 0; s0 < S; s0 += kMergeBatch) {
      float m[kMergeBatch], l[kMergeBatch], xa[kMergeBatch], xb[kMergeBatch];
#pragma unroll
      for (int u = 0; u < kMergeBatch; ++u) {
        const bool ok = s0 + u < S;
        const float* r = rh + (size_t)(s0 + u) * (kDim + 2);
        m[u] = ok ? __ldcg(r) : -INFINITY;
        l[u] = ok ? __ldcg(r + 1) : 0.f;
        xa[u] = ok ? __ldcg(r + 2 + d) : 0.f;
        xb[u] = ok ? __ldcg(r + 2 + d + kHalf) : 0.f;
      }
      float bm = mx;
#pragma unroll
      for (int u = 0; u < kMergeBatch; ++u) bm = fmaxf(bm, m[u]);
      if (bm == -INFINITY) continue;            // every record so far is empty
      const float a = (mx == -INFINITY) ? 0.f : ex2(mx - bm);
      ls *= a;
      oa *= a;
      ob *= a;
#pragma unroll
      for (int u = 0; u < kMergeBatch; ++u) {
        const float w = (m[u] == -INFINITY) ? 0.f : ex2(m[u] - bm);
        ls = fmaf(w, l[u], ls);
        oa = fmaf(w, xa[u], oa);
        ob = fmaf(w, xb[u], ob);
      }
      mx = bm;
    }
    __nv_bfloat16* out = p.o + (size_t)(bh0 + h) * kDim;
    out[d] = __float2bfloat16_rn(ls > 0.f ? oa / ls : 0.f);
    out[d + kHalf] = __float2bfloat16_rn(ls > 0.f ? ob / ls : 0.f);
    if (d == 0 && p.lse != nullptr) p.lse[bh0 + h] = (ls > 0.f) ? (mx + lg2(ls)) * kLn2 : -INFINITY;
  }
  if (tid == 0) p.ws_count[bkv * n_slices + slice] = 0;  // leave the workspace zeroed for the next call
}

// The tensor-core kernel takes D = 128 and either q and cache of the same
// 16-bit type with G >= 2, or an e4m3 cache (any G) with f16 / bf16 queries.
constexpr int kSliceHeads = 16;   // query heads per CTA (the MMA's N)

inline bool tc_eligible(long long H, long long H_kv, long long D, int q_dtype, int kv_dtype) {
  if (D != kDim) return false;
  if (kv_dtype == PU_DTYPE_FP8_E4M3) return q_dtype == PU_DTYPE_F16 || q_dtype == PU_DTYPE_BF16;
  return q_dtype == kv_dtype && (kv_dtype == PU_DTYPE_F16 || kv_dtype == PU_DTYPE_BF16) && H / H_kv >= 2;
}

inline long long n_slices(long long G) { return (G + kSliceHeads - 1) / kSliceHeads; }

// Split records one last CTA merges (heads x splits): more splits spread the
// stream over more SMs, but the merge runs on one SM (256 measured best of
// 64-1024 over G = 2-32, B = 1-8, with an earlier merge).
constexpr long long kMaxRecords = 256;

// One CTA per SM; chunks are whole tiles; at most kMaxRecords / (heads of a
// slice) splits.
inline Plan tc_plan(long long B, long long H, long long H_kv, long long n, int num_sms, bool ragged,
                    int ctas_per_sm = 1) {
  const long long G = H / H_kv;
  const int slots = num_sms * ctas_per_sm / kCtasPerSm;     // make_plan counts kCtasPerSm CTAs per SM
  Plan pl = make_plan(B * H_kv * n_slices(G), n, kDim, slots > 0 ? slots : 1, ragged, BT);
  const long long cap = std::max<long long>(1, kMaxRecords / std::min<long long>(G, kSliceHeads));
  if (pl.splits > cap) {
    const long long chunk = ((n + cap - 1) / cap + BT - 1) / BT * BT;
    pl.chunk = (int)chunk;
    pl.splits = (int)((n + chunk - 1) / chunk);
  }
  pl.total_bytes = pl.rec_off + round_up((size_t)B * H * pl.splits * (kDim + 2) * sizeof(float), 256);
  return pl;
}

template <typename T, typename KVT, int NP>
int launch_np(const CUtensorMap& tk, const CUtensorMap& tv, const Params& prm, dim3 grid, cudaStream_t st) {
  constexpr int smem = Cfg<NP, KVT>::kSmemBytes;
  const int rc = set_max_dynamic_smem(reinterpret_cast<const void*>(gqa_tc_kernel<T, KVT, NP>), smem,
                                      "grouped-head decode (tensor core) shared memory");
  if (rc) return rc;
  return check_cuda(launch_pdl(gqa_tc_kernel<T, KVT, NP>, grid, dim3(kThreads), smem, st, tk, tv, prm),
                    "grouped-head decode (tensor core) launch");
}

inline int launch(const Params& prm, int q_dtype, int kv_dtype, long long B, long long H_kv, cudaStream_t st) {
  const bool f8 = kv_dtype == PU_DTYPE_FP8_E4M3;
  CUtensorMap tk, tv;
  int rc = f8 ? make_tmap_u8_3d(&tk, prm.k, kDim, prm.n_local, B * H_kv, kDim, BT, true)
              : make_tmap_bf16_3d(&tk, prm.k, kDim, prm.n_local, B * H_kv, 64, BT, true);
  if (!rc)
    rc = f8 ? make_tmap_u8_3d(&tv, prm.v, kDim, prm.n_local, B * H_kv, kDim, BT, true)
            : make_tmap_bf16_3d(&tv, prm.v, kDim, prm.n_local, B * H_kv, 64, BT, true);
  if (rc) return rc;
  const dim3 grid((unsigned)(prm.splits * n_slices(prm.group)), (unsigned)(B * H_kv));
  if (f8)
    return q_dtype == PU_DTYPE_F16 ? launch_np<__half, __nv_fp8_e4m3, kSliceHeads>(tk, tv, prm, grid, st)
                                   : launch_np<__nv_bfloat16, __nv_fp8_e4m3, kSliceHeads>(tk, tv, prm, grid, st);
  return kv_dtype == PU_DTYPE_F16 ? launch_np<__half, __half, kSliceHeads>(tk, tv, prm, grid, st)
                                  : launch_np<__nv_bfloat16, __nv_bfloat16, kSliceHeads>(tk, tv, prm, grid, st);
}

}  // namespace tc
}  // namespace decode
}  // namespace pu

extern "C" {

// Serves every kernel pu_decode_gqa may pick for these sizes (with or
// without lengths, any dtypes).
size_t pu_decode_gqa_workspace_size(int64_t B, int64_t H, int64_t H_kv, int64_t n, int64_t D) {
  using namespace pu::decode;
  if (B <= 0 || H <= 0 || H_kv <= 0 || n <= 0 || D <= 0 || H % H_kv) return 0;
  const int sms = pu::sm_count();
  size_t bytes = workspace_bytes_any(B * H, n, D, sms);
  if (gqa_grouped(H, H_kv))
    bytes = std::max({bytes, gqa_plan(B, H, H_kv, n, D, sms, false).total_bytes,
                      gqa_plan(B, H, H_kv, n, D, sms, true).total_bytes});
  if (tc::tc_eligible(H, H_kv, D, PU_DTYPE_F16, PU_DTYPE_FP8_E4M3))
    bytes = std::max({bytes, tc::tc_plan(B, H, H_kv, n, sms, false, tc::kF8CtasPerSm).total_bytes,
                      tc::tc_plan(B, H, H_kv, n, sms, true, tc::kF8CtasPerSm).total_bytes});
  if (tc::tc_eligible(H, H_kv, D, PU_DTYPE_F16, PU_DTYPE_F16))
    bytes = std::max({bytes, tc::tc_plan(B, H, H_kv, n, sms, false).total_bytes,
                      tc::tc_plan(B, H, H_kv, n, sms, true).total_bytes});
  return bytes;
}

int pu_decode_gqa(const void* q, int q_dtype, const void* k_cache, const void* v_cache, int kv_dtype,
                  const int32_t* kv_lens, void* o, float* lse, void* workspace, size_t workspace_bytes,
                  int64_t B, int64_t H, int64_t H_kv, int64_t n, int64_t D, float sm_scale, float k_scale,
                  float v_scale, void* stream) {
  using namespace pu::decode;
  int rc = check_args(q, q_dtype, k_cache, v_cache, kv_dtype, B, H, n, D, true);
  if (rc) return rc;
  if (!o) return pu::set_error(PU_ERR_INVALID_ARGUMENT, "null output");
  if (H_kv <= 0 || H % H_kv != 0)
    return pu::set_error(PU_ERR_INVALID_ARGUMENT, "H = %lld is not a multiple of H_kv = %lld", (long long)H,
                         (long long)H_kv);
  if (!(k_scale > 0.f) || !(v_scale > 0.f) || !isfinite(k_scale) || !isfinite(v_scale))
    return pu::set_error(PU_ERR_INVALID_ARGUMENT, "k_scale and v_scale must be positive and finite");
  // tensor core for D = 128 with 16-bit caches and G >= 2 or e4m3 caches
  // and any G; the CUDA-core grouped kernel for D = 64 or mixed 16-bit
  // dtypes (G = 2, 4, 8); otherwise the query-head kernel reading K/V head h / G
  const bool on_tc = tc::tc_eligible(H, H_kv, D, q_dtype, kv_dtype);
  const bool grouped = !on_tc && gqa_grouped(H, H_kv);
  const bool ragged = kv_lens != nullptr;
  const Plan pl = on_tc ? tc::tc_plan(B, H, H_kv, n, pu::sm_count(), ragged,
                                      kv_dtype == PU_DTYPE_FP8_E4M3 ? tc::kF8CtasPerSm : 1)
                        : grouped ? gqa_plan(B, H, H_kv, n, D, pu::sm_count(), ragged)
                                  : make_plan(B * H, n, D, pu::sm_count(), ragged);
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
  prm.group = (int)(H / H_kv);
  prm.o_scale = v_scale;
  prm.splits = pl.splits;
  prm.chunk = pl.chunk;
  prm.scale_log2 = sm_scale * k_scale * kLog2e;
  prm.ws_rec = reinterpret_cast<float*>(static_cast<char*>(workspace) + pl.rec_off);
  prm.ws_count = static_cast<int*>(workspace);
  prm.o = static_cast<__nv_bfloat16*>(o);
  prm.lse = lse;
  if (on_tc) return tc::launch(prm, q_dtype, kv_dtype, B, H_kv, static_cast<cudaStream_t>(stream));
  if (grouped)
    return launch_gqa(prm, q_dtype, kv_dtype, (int)D, prm.group, (int)(B * H_kv), static_cast<cudaStream_t>(stream));
  return launch<true>(prm, q_dtype, kv_dtype, (int)D, (int)(B * H), static_cast<cudaStream_t>(stream));
}

}  // extern "C"
