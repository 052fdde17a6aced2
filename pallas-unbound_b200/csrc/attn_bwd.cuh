// attn_bwd.cuh — training-attention backward on tcgen05 tensor cores.
//
// The reference has no backward kernel (its Pallas kernel is forward-only and
// discards m, l; src/pallas_flash/kernels/attention.py:25).  This computes the
// gradients of the attention of benchmarks/baseline_mha.py:22-58 from the
// forward's saved LSE:
//   P = exp(scale*Q K^T - LSE),  dV = P^T dO,  dP = dO V^T,
//   Delta = rowsum(dO * O),      dS = P * (dP - Delta),
//   dQ = scale * dS K,           dK = scale * dS^T Q.
//
// Three kernels, no atomics (every gradient element is written once, so the
// backward is deterministic):
//   prep     Delta and LSE*log2(e) per query row (padded to 128-row tiles).
//   dkdv     one CTA per 128-row K/V tile of one (b, h).  K, V stay in shared
//            memory; Q / dO tiles with their row statistics stream through
//            2-deep TMA rings.  TMEM lanes = key rows:
//              S^T  = K Q^T   [0,128)      P^T  (bf16) over S^T's columns
//              dP^T = V dO^T  [128,256)    dS^T (bf16) over dP^T's columns
//              dV  += P^T dO  [256,384)    dK  += dS^T Q  [384,512)
//            Both products read their A operand from TMEM.  Tensor order per
//            query tile i: dV_i, S_{i+1}, dK_i, dP_{i+1}.
//   dq       one CTA per 128-row query tile: Q, dO resident, K / V streamed.
//            TMEM lanes = query rows:
//              S  = Q K^T  [0,128)   dP = dO V^T  [128,256)
//              dQ += dS K  [256,256+D)          dS (bf16) [384,448)
//            S_{j+1} is issued as soon as S_j has been read, dP_{j+1} as soon
//            as dP_j has been read, dQ_j once dS_j is in TMEM; dQ is written
//            once, in bf16, at the end.
// In both main kernels warps 0-7 form two warpgroups that split the 128
// columns of the score tile (64 each), warp 8 is the TMA producer and warp 9
// the tcgen05 issuer / TMEM owner.
#pragma once

#include <cuda_bf16.h>

#include "pu_host.cuh"
#include "pu_ptx.cuh"

namespace pu {
namespace bwd {

constexpr int BM = 128;   // query rows per tile
constexpr int BN = 128;   // key/value rows per tile
constexpr int kThreads = 320;
constexpr int HC = 64;    // score columns per compute warpgroup
constexpr float kLog2e = 1.4426950408889634f;
constexpr uint32_t kTmemCols = 512;

struct Params {
  int Nq, Nkv, H, BH;
  int n_q_tiles, n_kv_tiles;
  int causal;
  float scale_log2;
  float scale;
  int nq_pad;              // row pitch of the stats arrays (multiple of BM)
  const float* lse2;       // [BH][nq_pad] LSE * log2(e), +inf past Nq
  const float* delta;      // [BH][nq_pad], 0 past Nq
  __nv_bfloat16* dq;
  __nv_bfloat16* dk;
  __nv_bfloat16* dv;
};

// Load 64 consecutive TMEM columns of this warp's lanes (one wait).
__device__ __forceinline__ void tmem_ld64(uint32_t taddr, uint32_t (&r)[64]) {
  tmem_ld32(taddr, *reinterpret_cast<uint32_t(*)[32]>(r));
  tmem_ld32(taddr + 32, *reinterpret_cast<uint32_t(*)[32]>(r + 32));
  tmem_wait_ld();
  reg_fence(r);
}

// Store this thread's row of an accumulator (n32 chunks of 32 fp32 columns
// at TMEM column `col0`) as bf16 times `sc` to `rowp` (skipped if !store).
__device__ __forceinline__ void store_row_bf16(uint32_t taddr, int n32, float sc, __nv_bfloat16* rowp,
                                               bool store) {
#pragma unroll 1
  for (int c = 0; c < n32; ++c) {
    uint32_t rr[32];
    tmem_ld32(taddr + c * 32, rr);
    tmem_wait_ld();
    reg_fence(rr);
    uint32_t w[16];
#pragma unroll
    for (int i = 0; i < 16; ++i)
      w[i] = pack_bf16x2(__uint_as_float(rr[2 * i]) * sc, __uint_as_float(rr[2 * i + 1]) * sc);
    if (store) {
      uint4* dst = reinterpret_cast<uint4*>(rowp + c * 32);
#pragma unroll
      for (int i = 0; i < 4; ++i) dst[i] = make_uint4(w[4 * i], w[4 * i + 1], w[4 * i + 2], w[4 * i + 3]);
    }
  }
}

// ============================================================================
// dK / dV
// ============================================================================
template <int D>
struct CfgKV {
  static constexpr int NSQ = 2;                  // Q / dO ring depth
  static constexpr int kTileQ = BM * D * 2;
  static constexpr int kTileKV = BN * D * 2;
  static constexpr int kColBlocks = D / 64;
  static constexpr int kOffK = 0;
  static constexpr int kOffV = kOffK + kTileKV;
  static constexpr int kOffQ = kOffV + kTileKV;
  static constexpr int kOffDO = kOffQ + NSQ * kTileQ;
  static constexpr int kOffStats = kOffDO + NSQ * kTileQ;   // [NSQ][lse2[BM], delta[BM]]
  static constexpr int kStatBytes = 2 * BM * 4;
  static constexpr int kOffBar = kOffStats + NSQ * kStatBytes;
  // barriers: KV, Qf[NSQ], Qe[NSQ], dOf[NSQ], dOe[NSQ], S, dP, P, dS, final
  static constexpr int kNumBars = 1 + 4 * NSQ + 5;
  static constexpr int kSmemBytes = kOffBar + kNumBars * 8 + 16;
  static_assert(kSmemBytes <= 232448, "shared memory budget");
  static constexpr uint32_t kColS = 0, kColDP = 128, kColDV = 256, kColDK = 384;
};

template <int D>
__global__ void __launch_bounds__(kThreads, 1)
    attn_bwd_dkdv_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                         const __grid_constant__ CUtensorMap tmV, const __grid_constant__ CUtensorMap tmDO,
                         const Params p) {
  using C = CfgKV<D>;
  extern __shared__ __align__(1024) uint8_t smem[];
  const int tid = threadIdx.x;
  const int warp = tid >> 5;
  const int lane = tid & 31;
  if (smem_u32(smem) & 1023u) {  // the swizzled tiles need 1024-byte alignment
    if (tid == 0) record_device_error(PU_ERR_UNSUPPORTED, kSiteBwdKV);
    return;
  }
  uint8_t* sK = smem + C::kOffK;
  uint8_t* sV = smem + C::kOffV;
  uint8_t* sQ = smem + C::kOffQ;
  uint8_t* sDO = smem + C::kOffDO;
  float* s_stats = reinterpret_cast<float*>(smem + C::kOffStats);  // [NSQ][2][BM]
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + C::kOffBar);
  uint64_t* bKV = bars;
  uint64_t* bQf = bars + 1;
  uint64_t* bQe = bQf + C::NSQ;
  uint64_t* bDOf = bQe + C::NSQ;
  uint64_t* bDOe = bDOf + C::NSQ;
  uint64_t* bS = bDOe + C::NSQ;
  uint64_t* bDP = bS + 1;
  uint64_t* bP = bDP + 1;
  uint64_t* bDS = bP + 1;
  uint64_t* bFinal = bDS + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bFinal + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  // One linear grid, (b, h) fastest: all heads' heaviest (causal: first)
  // key tiles first (longest-first start order).
  const int kv_tile = (int)(blockIdx.x / (unsigned)p.BH);
  const int bh = (int)(blockIdx.x % (unsigned)p.BH);
  const int kv0 = kv_tile * BN;
  const int first_q = p.causal ? min(kv0 / BM, p.n_q_tiles) : 0;
  const int n_it = p.n_q_tiles - first_q;

  if (tid == 0) {
    mbar_init(bKV, 1);
    for (int s = 0; s < C::NSQ; ++s) {
      mbar_init(bQf + s, 1);
      mbar_init(bQe + s, 1);
      mbar_init(bDOf + s, 1);
      mbar_init(bDOe + s, 1);
    }
    mbar_init(bS, 1);
    mbar_init(bDP, 1);
    mbar_init(bP, 256);
    mbar_init(bDS, 256);
    mbar_init(bFinal, 1);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 9) {
    tmem_alloc(tmem_slot, kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 8) {
    // ---------------- TMA producer ----------------
    if (lane == 0 && n_it > 0) {
      tma_prefetch_desc(&tmQ);
      tma_prefetch_desc(&tmK);
      tma_prefetch_desc(&tmV);
      tma_prefetch_desc(&tmDO);
      mbar_arrive_expect_tx(bKV, 2 * C::kTileKV);
      for (int cb = 0; cb < C::kColBlocks; ++cb) {
        tma_load_3d(sK + cb * BN * 128, &tmK, bKV, cb * 64, kv0, bh);
        tma_load_3d(sV + cb * BN * 128, &tmV, bKV, cb * 64, kv0, bh);
      }
      for (int it = 0; it < n_it; ++it) {
        const int st = it % C::NSQ;
        const uint32_t u = it / C::NSQ;
        const int q0 = (first_q + it) * BM;
        if (u > 0 && !mbar_wait(bQe + st, (u - 1) & 1, abort_flag, kSiteBwdEmpty)) break;
        mbar_arrive_expect_tx(bQf + st, C::kTileQ + C::kStatBytes);
        for (int cb = 0; cb < C::kColBlocks; ++cb)
          tma_load_3d(sQ + st * C::kTileQ + cb * BM * 128, &tmQ, bQf + st, cb * 64, q0, bh);
        float* stat = s_stats + st * 2 * BM;
        bulk_load(stat, p.lse2 + (size_t)bh * p.nq_pad + q0, BM * 4, bQf + st);
        bulk_load(stat + BM, p.delta + (size_t)bh * p.nq_pad + q0, BM * 4, bQf + st);
        if (u > 0 && !mbar_wait(bDOe + st, (u - 1) & 1, abort_flag, kSiteBwdEmpty)) break;
        mbar_arrive_expect_tx(bDOf + st, C::kTileQ);
        for (int cb = 0; cb < C::kColBlocks; ++cb)
          tma_load_3d(sDO + st * C::kTileQ + cb * BM * 128, &tmDO, bDOf + st, cb * 64, q0, bh);
      }
    }
  } else if (warp == 9) {
    // ---------------- tcgen05 issuer ----------------
    if (lane == 0 && n_it > 0) {
      constexpr uint32_t idSS = make_idesc_bf16(BN, BM, 0, 0);   // S^T, dP^T: K-major A and B
      constexpr uint32_t idKMN = make_idesc_bf16(BN, D, 0, 1);   // dV, dK: A from TMEM, B MN-major
      const uint32_t aK = smem_u32(sK), aV = smem_u32(sV);
      // descriptors are built once per tile; per MMA only the start address moves
      // X^T = A_tile . B_tile^T over the head dimension (both K-major)
      auto issue_t = [&](uint32_t dcol, uint32_t aA, uint32_t aB) {
        const uint64_t da = make_sdesc_sw128(aA, 16, 1024), db = make_sdesc_sw128(aB, 16, 1024);
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
          const uint32_t off = (kk >> 2) * (BN * 128) + (kk & 3) * 32;
          const uint32_t offq = (kk >> 2) * (BM * 128) + (kk & 3) * 32;
          mma_ss(tmem + dcol, sdesc_add(da, off), sdesc_add(db, offq), idSS, kk > 0);
        }
      };
      // acc += A^T(TMEM, bf16 pairs at a_col: query cols [0,64) then [64,128)
      // at +64 columns) . B (MN-major [query][d] tile)
      auto issue_acc = [&](uint32_t dcol, uint32_t a_col, uint32_t aB, bool first) {
        const uint64_t db = make_sdesc_sw128(aB, BM * 128, 1024);
#pragma unroll
        for (int kk = 0; kk < BM / 16; ++kk) {
          mma_ts(tmem + dcol, tmem + a_col + (kk >> 2) * 64 + (kk & 3) * 8, sdesc_add(db, kk * 16 * 128),
                 idKMN, (!first || kk > 0));
        }
      };
      bool ok = mbar_wait(bKV, 0, abort_flag, kSiteBwdKV) && mbar_wait(bQf, 0, abort_flag, kSiteBwdLoad);
      if (ok) {
        tc_fence_after();
        issue_t(C::kColS, aK, smem_u32(sQ));
        mma_commit(bS);
        ok = mbar_wait(bDOf, 0, abort_flag, kSiteBwdLoad);
      }
      if (ok) {
        tc_fence_after();
        issue_t(C::kColDP, aV, smem_u32(sDO));
        mma_commit(bDP);
      }
      for (int it = 0; ok && it < n_it; ++it) {
        const int st = it % C::NSQ;
        const int nst = (it + 1) % C::NSQ;
        const uint32_t un = (it + 1) / C::NSQ;
        // dV += P^T dO
        if (!mbar_wait(bP, it & 1, abort_flag, kSiteBwdSoftmax)) break;
        tc_fence_after();
        issue_acc(C::kColDV, C::kColS, smem_u32(sDO + st * C::kTileQ), it == 0);
        mma_commit(bDOe + st);
        // S^T of the next query tile (after dV_it has read P^T: issue order)
        if (it + 1 < n_it) {
          if (!mbar_wait(bQf + nst, un & 1, abort_flag, kSiteBwdLoad)) break;
          tc_fence_after();
          issue_t(C::kColS, aK, smem_u32(sQ + nst * C::kTileQ));
          mma_commit(bS);
        }
        // dK += dS^T Q
        if (!mbar_wait(bDS, it & 1, abort_flag, kSiteBwdDs)) break;
        tc_fence_after();
        issue_acc(C::kColDK, C::kColDP, smem_u32(sQ + st * C::kTileQ), it == 0);
        mma_commit(bQe + st);
        // dP^T of the next query tile (after dK_it has read dS^T)
        if (it + 1 < n_it) {
          if (!mbar_wait(bDOf + nst, un & 1, abort_flag, kSiteBwdLoad)) break;
          tc_fence_after();
          issue_t(C::kColDP, aV, smem_u32(sDO + nst * C::kTileQ));
          mma_commit(bDP);
        } else {
          mma_commit(bFinal);
        }
      }
    }
  } else {
    // ---------------- compute warpgroups (warps 0-3: query cols 0-63, 4-7: 64-127) ----------------
    const int g = warp >> 2;
    const int r = tid & 127;                              // TMEM lane = key row
    const int kv_idx = kv0 + r;
    const uint32_t lane_base = static_cast<uint32_t>((warp & 3) * 32) << 16;
    const int cb = g * HC;                                // first query column of this warpgroup
    bool ok = true;
    for (int it = 0; it < n_it; ++it) {
      const int q0 = (first_q + it) * BM;
      const int st = it % C::NSQ;
      ok = mbar_wait(bQf + st, (it / C::NSQ) & 1, abort_flag, kSiteBwdLoad);
      ok = ok && mbar_wait(bS, it & 1, abort_flag, kSiteBwdMma);
      ok = __all_sync(0xffffffffu, ok);
      if (!ok) break;
      tc_fence_after();
      const float* lse_t = s_stats + st * 2 * BM + cb;
      const float* del_t = s_stats + st * 2 * BM + BM + cb;
      uint32_t pk[HC / 2];
      {
        uint32_t sr[HC];
        tmem_ld64(tmem + lane_base + C::kColS + cb, sr);
        const bool mask = p.causal && (q0 + cb < kv0 + BN - 1);
#pragma unroll
        for (int c4 = 0; c4 < HC; c4 += 4) {
          const float4 lv = *reinterpret_cast<const float4*>(lse_t + c4);
          float p0 = ex2(fmaf(__uint_as_float(sr[c4]), p.scale_log2, -lv.x));
          float p1 = ex2(fmaf(__uint_as_float(sr[c4 + 1]), p.scale_log2, -lv.y));
          float p2 = ex2(fmaf(__uint_as_float(sr[c4 + 2]), p.scale_log2, -lv.z));
          float p3 = ex2(fmaf(__uint_as_float(sr[c4 + 3]), p.scale_log2, -lv.w));
          if (mask) {                                     // query < key: invisible
            const int qa = q0 + cb + c4;
            if (qa < kv_idx) p0 = 0.f;
            if (qa + 1 < kv_idx) p1 = 0.f;
            if (qa + 2 < kv_idx) p2 = 0.f;
            if (qa + 3 < kv_idx) p3 = 0.f;
          }
          pk[c4 / 2] = pack_bf16x2(p0, p1);
          pk[c4 / 2 + 1] = pack_bf16x2(p2, p3);
        }
      }
      // P^T over this warpgroup's own (already read) S^T columns
      tmem_st32(tmem + lane_base + C::kColS + cb, pk);
      tmem_wait_st();
      tc_fence_before();
      mbar_arrive(bP);

      ok = mbar_wait(bDP, it & 1, abort_flag, kSiteBwdMma);
      ok = __all_sync(0xffffffffu, ok);
      if (!ok) break;
      tc_fence_after();
      {
        uint32_t dr[HC];
        tmem_ld64(tmem + lane_base + C::kColDP + cb, dr);
#pragma unroll
        for (int c4 = 0; c4 < HC; c4 += 4) {
          const float4 dl = *reinterpret_cast<const float4*>(del_t + c4);
          const uint32_t pa = pk[c4 / 2], pb = pk[c4 / 2 + 1];
          const float e0 = __uint_as_float(pa << 16) * (__uint_as_float(dr[c4]) - dl.x);
          const float e1 = __uint_as_float(pa & 0xFFFF0000u) * (__uint_as_float(dr[c4 + 1]) - dl.y);
          const float e2 = __uint_as_float(pb << 16) * (__uint_as_float(dr[c4 + 2]) - dl.z);
          const float e3 = __uint_as_float(pb & 0xFFFF0000u) * (__uint_as_float(dr[c4 + 3]) - dl.w);
          pk[c4 / 2] = pack_bf16x2(e0, e1);
          pk[c4 / 2 + 1] = pack_bf16x2(e2, e3);
        }
      }
      // dS^T over this warpgroup's own (already read) dP^T columns
      tmem_st32(tmem + lane_base + C::kColDP + cb, pk);
      tmem_wait_st();
      tc_fence_before();
      mbar_arrive(bDS);
    }
    // epilogue: this warpgroup's D/2 columns of dV, dK for its key rows
    if (ok && n_it > 0) {
      ok = mbar_wait(bFinal, 0, abort_flag, kSiteBwdMma);
      ok = __all_sync(0xffffffffu, ok);
    }
    if (ok) {
      const bool store = kv_idx < p.Nkv;
      constexpr int DC = D / 2;
      __nv_bfloat16* dvrow = p.dv + ((size_t)bh * p.Nkv + kv_idx) * D + g * DC;
      __nv_bfloat16* dkrow = p.dk + ((size_t)bh * p.Nkv + kv_idx) * D + g * DC;
      if (n_it > 0) {
        tc_fence_after();
        store_row_bf16(tmem + lane_base + C::kColDV + g * DC, DC / 32, 1.f, dvrow, store);
        store_row_bf16(tmem + lane_base + C::kColDK + g * DC, DC / 32, p.scale, dkrow, store);
      } else if (store) {
        // no query attends to these keys: zero gradients
        const uint4 z = make_uint4(0, 0, 0, 0);
#pragma unroll
        for (int i = 0; i < DC / 8; ++i) {
          reinterpret_cast<uint4*>(dvrow)[i] = z;
          reinterpret_cast<uint4*>(dkrow)[i] = z;
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 9) {
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
}

// ============================================================================
// dQ
// ============================================================================
template <int D>
struct CfgQ {
  // K_j is read twice (S_j early, dQ_j last), so its ring is one deeper than
  // V's: the load of K_{j+2} starts as soon as dQ_{j-1} has finished.
  static constexpr int NSK = 3;                  // K ring depth
  static constexpr int NSV = 2;                  // V ring depth
  static constexpr int kTileQ = BM * D * 2;
  static constexpr int kTileKV = BN * D * 2;
  static constexpr int kColBlocks = D / 64;
  static constexpr int kOffQ = 0;
  static constexpr int kOffDO = kOffQ + kTileQ;
  static constexpr int kOffK = kOffDO + kTileQ;
  static constexpr int kOffV = kOffK + NSK * kTileKV;
  static constexpr int kOffBar = kOffV + NSV * kTileKV;
  // barriers: QdO, Kf[NSK], Ke[NSK], Vf[NSV], Ve[NSV], S, dP, Sread, dPread, dS, dQdone
  static constexpr int kNumBars = 1 + 2 * NSK + 2 * NSV + 6;
  static constexpr int kSmemBytes = kOffBar + kNumBars * 8 + 16;
  static_assert(kSmemBytes <= 232448, "shared memory budget");
  static constexpr uint32_t kColS = 0, kColDP = 128, kColDQ = 256, kColDS = 384;
};

template <int D>
__global__ void __launch_bounds__(kThreads, 1)
    attn_bwd_dq_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                       const __grid_constant__ CUtensorMap tmV, const __grid_constant__ CUtensorMap tmDO,
                       const Params p) {
  using C = CfgQ<D>;
  extern __shared__ __align__(1024) uint8_t smem[];
  const int tid = threadIdx.x;
  const int warp = tid >> 5;
  const int lane = tid & 31;
  if (smem_u32(smem) & 1023u) {
    if (tid == 0) record_device_error(PU_ERR_UNSUPPORTED, kSiteBwdKV);
    return;
  }
  uint8_t* sQ = smem + C::kOffQ;
  uint8_t* sDO = smem + C::kOffDO;
  uint8_t* sK = smem + C::kOffK;
  uint8_t* sV = smem + C::kOffV;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + C::kOffBar);
  uint64_t* bQ = bars;
  uint64_t* bKf = bars + 1;
  uint64_t* bKe = bKf + C::NSK;
  uint64_t* bVf = bKe + C::NSK;
  uint64_t* bVe = bVf + C::NSV;
  uint64_t* bS = bVe + C::NSV;
  uint64_t* bDP = bS + 1;
  uint64_t* bSr = bDP + 1;      // S_j read by the compute warps
  uint64_t* bDPr = bSr + 1;     // dP_j read
  uint64_t* bDS = bDPr + 1;     // dS_j in TMEM
  uint64_t* bDQd = bDS + 1;     // dQ += dS_j K_j done (dS columns reusable)
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bDQd + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  // one linear grid, (b, h) fastest, heaviest (causal: last) query tiles first
  const int q_tile = p.n_q_tiles - 1 - (int)(blockIdx.x / (unsigned)p.BH);
  const int bh = (int)(blockIdx.x % (unsigned)p.BH);
  const int q0 = q_tile * BM;
  int n_blocks = p.n_kv_tiles;
  if (p.causal) n_blocks = max(1, min(n_blocks, (q0 + BM + BN - 1) / BN));

  if (tid == 0) {
    mbar_init(bQ, 1);
    for (int s = 0; s < C::NSK; ++s) {
      mbar_init(bKf + s, 1);
      mbar_init(bKe + s, 1);
    }
    for (int s = 0; s < C::NSV; ++s) {
      mbar_init(bVf + s, 1);
      mbar_init(bVe + s, 1);
    }
    mbar_init(bS, 1);
    mbar_init(bDP, 1);
    mbar_init(bSr, 256);
    mbar_init(bDPr, 256);
    mbar_init(bDS, 256);
    mbar_init(bDQd, 1);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 9) {
    tmem_alloc(tmem_slot, kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 8) {
    // ---------------- TMA producer ----------------
    if (lane == 0) {
      tma_prefetch_desc(&tmQ);
      tma_prefetch_desc(&tmK);
      tma_prefetch_desc(&tmV);
      tma_prefetch_desc(&tmDO);
      mbar_arrive_expect_tx(bQ, 2 * C::kTileQ);
      for (int cb = 0; cb < C::kColBlocks; ++cb) {
        tma_load_3d(sQ + cb * BM * 128, &tmQ, bQ, cb * 64, q0, bh);
        tma_load_3d(sDO + cb * BM * 128, &tmDO, bQ, cb * 64, q0, bh);
      }
      for (int j = 0; j < n_blocks; ++j) {
        const int sk = j % C::NSK, sv = j % C::NSV;
        const uint32_t uk = j / C::NSK, uv = j / C::NSV;
        if (uk > 0 && !mbar_wait(bKe + sk, (uk - 1) & 1, abort_flag, kSiteBwdEmpty)) break;
        mbar_arrive_expect_tx(bKf + sk, C::kTileKV);
        for (int cb = 0; cb < C::kColBlocks; ++cb)
          tma_load_3d(sK + sk * C::kTileKV + cb * BN * 128, &tmK, bKf + sk, cb * 64, j * BN, bh);
        if (uv > 0 && !mbar_wait(bVe + sv, (uv - 1) & 1, abort_flag, kSiteBwdEmpty)) break;
        mbar_arrive_expect_tx(bVf + sv, C::kTileKV);
        for (int cb = 0; cb < C::kColBlocks; ++cb)
          tma_load_3d(sV + sv * C::kTileKV + cb * BN * 128, &tmV, bVf + sv, cb * 64, j * BN, bh);
      }
    }
  } else if (warp == 9) {
    // ---------------- tcgen05 issuer ----------------
    if (lane == 0) {
      constexpr uint32_t idSS = make_idesc_bf16(BM, BN, 0, 0);   // S, dP: K-major A and B
      constexpr uint32_t idQ = make_idesc_bf16(BM, D, 0, 1);     // dQ: A = dS from TMEM, B = K MN-major
      const uint32_t aQ = smem_u32(sQ), aDO = smem_u32(sDO);
      auto issue_ss = [&](uint32_t dcol, uint32_t aA, uint32_t aB) {
        const uint64_t da = make_sdesc_sw128(aA, 16, 1024), db = make_sdesc_sw128(aB, 16, 1024);
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
          const uint32_t off = (kk >> 2) * (BM * 128) + (kk & 3) * 32;
          const uint32_t offk = (kk >> 2) * (BN * 128) + (kk & 3) * 32;
          mma_ss(tmem + dcol, sdesc_add(da, off), sdesc_add(db, offk), idSS, kk > 0);
        }
      };
      bool ok = mbar_wait(bQ, 0, abort_flag, kSiteBwdLoad) && mbar_wait(bKf, 0, abort_flag, kSiteBwdLoad);
      if (ok) {
        tc_fence_after();
        issue_ss(C::kColS, aQ, smem_u32(sK));
        mma_commit(bS);
        ok = mbar_wait(bVf, 0, abort_flag, kSiteBwdLoad);
      }
      if (ok) {
        tc_fence_after();
        issue_ss(C::kColDP, aDO, smem_u32(sV));
        mma_commit(bDP);
      }
      for (int j = 0; ok && j < n_blocks; ++j) {
        const int sk = j % C::NSK, sv = j % C::NSV;
        const int nsk = (j + 1) % C::NSK, nsv = (j + 1) % C::NSV;
        const uint32_t unk = (j + 1) / C::NSK, unv = (j + 1) / C::NSV;
        const bool more = j + 1 < n_blocks;
        // S_{j+1} once S_j has been read
        if (!mbar_wait(bSr, j & 1, abort_flag, kSiteBwdSoftmax)) break;
        if (more) {
          if (!mbar_wait(bKf + nsk, unk & 1, abort_flag, kSiteBwdLoad)) break;
          tc_fence_after();
          issue_ss(C::kColS, aQ, smem_u32(sK + nsk * C::kTileKV));
          mma_commit(bS);
        }
        // dP_{j+1} once dP_j has been read
        if (!mbar_wait(bDPr, j & 1, abort_flag, kSiteBwdSoftmax)) break;
        mma_commit(bVe + sv);                // V_j's only reader (dP_j) has completed
        if (more) {
          if (!mbar_wait(bVf + nsv, unv & 1, abort_flag, kSiteBwdLoad)) break;
          tc_fence_after();
          issue_ss(C::kColDP, aDO, smem_u32(sV + nsv * C::kTileKV));
          mma_commit(bDP);
        }
        // dQ += dS_j K_j
        if (!mbar_wait(bDS, j & 1, abort_flag, kSiteBwdDs)) break;
        tc_fence_after();
        const uint64_t dk = make_sdesc_sw128(smem_u32(sK + sk * C::kTileKV), BN * 128, 1024);
#pragma unroll
        for (int kk = 0; kk < BN / 16; ++kk) {
          mma_ts(tmem + C::kColDQ, tmem + C::kColDS + kk * 8, sdesc_add(dk, kk * 16 * 128), idQ,
                 (j > 0 || kk > 0));
        }
        mma_commit(bDQd);
        mma_commit(bKe + sk);
      }
    }
  } else {
    // ---------------- compute warpgroups (warps 0-3: key cols 0-63, 4-7: 64-127) ----------------
    const int g = warp >> 2;
    const int r = tid & 127;                              // TMEM lane = query row
    const int q_idx = q0 + r;
    const uint32_t lane_base = static_cast<uint32_t>((warp & 3) * 32) << 16;
    const int cb = g * HC;                                // first key column of this warpgroup
    const float lse2 = p.lse2[(size_t)bh * p.nq_pad + q_idx];   // +inf past Nq
    const float dlt = p.delta[(size_t)bh * p.nq_pad + q_idx];
    const float neg_lse2 = -lse2;
    bool ok = true;
    for (int j = 0; j < n_blocks; ++j) {
      const int kvb = j * BN + cb;                        // key index of this warpgroup's column 0
      ok = mbar_wait(bS, j & 1, abort_flag, kSiteBwdMma);
      ok = __all_sync(0xffffffffu, ok);
      if (!ok) break;
      tc_fence_after();
      uint32_t pk[HC / 2];
      {
        uint32_t sr[HC];
        tmem_ld64(tmem + lane_base + C::kColS + cb, sr);
        tc_fence_before();
        mbar_arrive(bSr);
        const bool mask = (p.causal && kvb + HC - 1 > q0) || (kvb + HC > p.Nkv);
        const int lim = p.causal ? min(q_idx + 1, p.Nkv) : p.Nkv;   // keys < lim are visible
#pragma unroll
        for (int c = 0; c < HC; c += 2) {
          float p0 = ex2(fmaf(__uint_as_float(sr[c]), p.scale_log2, neg_lse2));
          float p1 = ex2(fmaf(__uint_as_float(sr[c + 1]), p.scale_log2, neg_lse2));
          if (mask) {
            if (kvb + c >= lim) p0 = 0.f;
            if (kvb + c + 1 >= lim) p1 = 0.f;
          }
          pk[c / 2] = pack_bf16x2(p0, p1);
        }
      }
      ok = mbar_wait(bDP, j & 1, abort_flag, kSiteBwdMma);
      ok = __all_sync(0xffffffffu, ok);
      if (!ok) break;
      tc_fence_after();
      {
        uint32_t dr[HC];
        tmem_ld64(tmem + lane_base + C::kColDP + cb, dr);
        tc_fence_before();
        mbar_arrive(bDPr);
#pragma unroll
        for (int c = 0; c < HC; c += 2) {
          const uint32_t pp = pk[c / 2];
          const float e0 = __uint_as_float(pp << 16) * (__uint_as_float(dr[c]) - dlt);
          const float e1 = __uint_as_float(pp & 0xFFFF0000u) * (__uint_as_float(dr[c + 1]) - dlt);
          pk[c / 2] = pack_bf16x2(e0, e1);
        }
      }
      // dS columns are reusable once dQ += dS_{j-1} K_{j-1} has completed
      if (j > 0) {
        ok = mbar_wait(bDQd, (j - 1) & 1, abort_flag, kSiteBwdDq);
        ok = __all_sync(0xffffffffu, ok);
        if (!ok) break;
      }
      tmem_st32(tmem + lane_base + C::kColDS + g * (HC / 2), pk);
      tmem_wait_st();
      tc_fence_before();
      mbar_arrive(bDS);
    }
    if (ok) {
      ok = mbar_wait(bDQd, (n_blocks - 1) & 1, abort_flag, kSiteBwdDq);
      ok = __all_sync(0xffffffffu, ok);
    }
    if (ok) {
      tc_fence_after();
      constexpr int DC = D / 2;
      __nv_bfloat16* dqrow = p.dq + ((size_t)bh * p.Nq + q_idx) * D + g * DC;
      store_row_bf16(tmem + lane_base + C::kColDQ + g * DC, DC / 32, p.scale, dqrow, q_idx < p.Nq);
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 9) {
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
}

// ============================================================================
// Fused single-pass backward (D = 128)
// ============================================================================
// One CTA per 128-row K/V tile, as in dkdv, but the five products of a
// (key tile, query tile) pair are all done here, P is computed once, and dQ
// leaves through fp32 reductions into an L2-resident accumulator:
//   S^T  = K Q^T        [0,128)     P^T (bf16) over S^T's first columns
//   dP^T = V dO^T       [128,256)   dS^T (bf16) over dP^T's first columns
//   dV  += P^T dO       [256,384)   (A = P^T from TMEM)
//   dK  += dS^T Q       [384,512)   (A = dS^T from TMEM)
//   dQ^T = K^T dS^T     [128,256)   (A = the K tile read MN-major, B = dS^T
//                                    from shared memory; lanes = head dim)
// dQ^T reuses dP^T's columns once the compute warps have read dP^T and
// written dS^T; four drain warps (one per TMEM lane quarter, thread = one
// head-dim column d) add it to dq_acc[q][d] with coalesced
// `red.global.add.f32` (a warp covers 32 consecutive d of one query row, one
// 128-byte line per instruction): the first 64 query columns, then the other
// 64 read, the columns released for the next dP^T, and those 64 added.
// Tensor order per query tile i:
//   dV_i, S_{i+1}, dK_i, dQ_i, [dQ_i drained] dP_{i+1}.
// Measured limits of this arrangement (clock64 traces of one CTA, causal
// B4 H16 N4096): ~6k SM cycles per tile pair against 2.6k of tensor work.
// The 64 KB of dQ reductions per tile pair move at about 20 bytes per SM
// clock whether issued as per-thread reductions or as TMA bulk reduce-adds,
// and the per-thread form slows the compute warps' shared-memory traffic;
// 64-row query tiles (which would give dQ^T its own TMEM columns) need N = 64
// products, which cost as much per instruction as N = 128 ones.
// Warps: 0-7 compute (two warpgroups, 64 query columns each), 8-11 dQ drain,
// 12 TMA producer, 13 tcgen05 issuer / TMEM owner.
// CTAs walk groups of kHeadGroup heads (so one group's dq_acc, Q and dO stay
// in L2), longest key tile first inside a group, heads fastest.
constexpr int kFusedThreads = 448;
constexpr int kHeadGroup = 8;

struct CfgF {
  static constexpr int D = 128;
  static constexpr int NSQ = 2;                  // Q / dO ring depth
  static constexpr int kTile = BM * D * 2;       // 32 KB (BM == BN)
  static constexpr int kOffK = 0;
  static constexpr int kOffV = kOffK + kTile;
  static constexpr int kOffQ = kOffV + kTile;
  static constexpr int kOffDO = kOffQ + NSQ * kTile;
  static constexpr int kOffDS = kOffDO + NSQ * kTile;        // dS^T [kv][q], two 64-column blocks
  static constexpr int kOffStats = kOffDS + kTile;           // [NSQ][lse2[BM], delta[BM]]
  static constexpr int kStatBytes = 2 * BM * 4;
  static constexpr int kOffBar = kOffStats + NSQ * kStatBytes;
  // barriers: KV, Qf[NSQ], Qe[NSQ], dOf[NSQ], dOe[NSQ], S, dP, P, dS, dQ, dQd
  static constexpr int kNumBars = 1 + 4 * NSQ + 6;
  static constexpr int kSmemBytes = kOffBar + kNumBars * 8 + 16;
  static_assert(kSmemBytes <= 232448, "shared memory budget");
  static constexpr uint32_t kColS = 0, kColDP = 128, kColDV = 256, kColDK = 384;
};

struct ParamsF {
  Params base;
  float* dq_acc;           // [BH][nq_pad][D] fp32, zeroed by prep
};

__device__ __forceinline__ void red_add_f32(float* p, float v) {
  asm volatile("red.global.add.f32 [%0], %1;" ::"l"(p), "f"(v) : "memory");
}

__global__ void __launch_bounds__(kFusedThreads, 1)
    attn_bwd_fused_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                          const __grid_constant__ CUtensorMap tmV, const __grid_constant__ CUtensorMap tmDO,
                          const ParamsF pf) {
  using C = CfgF;
  constexpr int D = C::D;
  const Params& p = pf.base;
  extern __shared__ __align__(1024) uint8_t smem[];
  const int tid = threadIdx.x;
  const int warp = tid >> 5;
  const int lane = tid & 31;
  if (smem_u32(smem) & 1023u) {
    if (tid == 0) record_device_error(PU_ERR_UNSUPPORTED, kSiteBwdKV);
    return;
  }
  uint8_t* sK = smem + C::kOffK;
  uint8_t* sV = smem + C::kOffV;
  uint8_t* sQ = smem + C::kOffQ;
  uint8_t* sDO = smem + C::kOffDO;
  uint8_t* sDS = smem + C::kOffDS;
  float* s_stats = reinterpret_cast<float*>(smem + C::kOffStats);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + C::kOffBar);
  uint64_t* bKV = bars;
  uint64_t* bQf = bars + 1;
  uint64_t* bQe = bQf + C::NSQ;
  uint64_t* bDOf = bQe + C::NSQ;
  uint64_t* bDOe = bDOf + C::NSQ;
  uint64_t* bS = bDOe + C::NSQ;    // S^T_i complete
  uint64_t* bDP = bS + 1;          // dP^T_i complete
  uint64_t* bP = bDP + 1;          // P^T_i in TMEM (256 arrivals)
  uint64_t* bDS = bP + 1;          // dS^T_i in TMEM and shared memory (256 arrivals)
  uint64_t* bDQ = bDS + 1;         // dK_i and dQ^T_i complete (and every earlier product)
  uint64_t* bDQd = bDQ + 1;        // dQ^T_i read out of TMEM (128 arrivals)
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bDQd + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  // block -> (head group, key tile longest first, head)
  const int per_group = kHeadGroup * p.n_kv_tiles;
  const int grp = (int)(blockIdx.x / (unsigned)per_group);
  const int rem = (int)(blockIdx.x - (unsigned)grp * (unsigned)per_group);
  const int hg = min(kHeadGroup, p.BH - grp * kHeadGroup);
  const int kv_tile = rem / hg;
  const int bh = grp * kHeadGroup + rem % hg;
  const int kv0 = kv_tile * BN;
  const int first_q = p.causal ? min(kv0 / BM, p.n_q_tiles) : 0;
  const int n_it = p.n_q_tiles - first_q;

  if (tid == 0) {
    mbar_init(bKV, 1);
    for (int s = 0; s < C::NSQ; ++s) {
      mbar_init(bQf + s, 1);
      mbar_init(bQe + s, 1);
      mbar_init(bDOf + s, 1);
      mbar_init(bDOe + s, 1);
    }
    mbar_init(bS, 1);
    mbar_init(bDP, 1);
    mbar_init(bP, 256);
    mbar_init(bDS, 256);
    mbar_init(bDQ, 1);
    mbar_init(bDQd, 128);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 13) {
    tmem_alloc(tmem_slot, kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 12) {
    // ---------------- TMA producer ----------------
    if (lane == 0 && n_it > 0) {
      tma_prefetch_desc(&tmQ);
      tma_prefetch_desc(&tmK);
      tma_prefetch_desc(&tmV);
      tma_prefetch_desc(&tmDO);
      mbar_arrive_expect_tx(bKV, 2 * C::kTile);
      for (int cb = 0; cb < 2; ++cb) {
        tma_load_3d(sK + cb * BN * 128, &tmK, bKV, cb * 64, kv0, bh);
        tma_load_3d(sV + cb * BN * 128, &tmV, bKV, cb * 64, kv0, bh);
      }
      for (int it = 0; it < n_it; ++it) {
        const int st = it % C::NSQ;
        const uint32_t u = it / C::NSQ;
        const int q0 = (first_q + it) * BM;
        if (u > 0 && !mbar_wait(bQe + st, (u - 1) & 1, abort_flag, kSiteBwdEmpty)) break;
        mbar_arrive_expect_tx(bQf + st, C::kTile + C::kStatBytes);
        for (int cb = 0; cb < 2; ++cb)
          tma_load_3d(sQ + st * C::kTile + cb * BM * 128, &tmQ, bQf + st, cb * 64, q0, bh);
        float* stat = s_stats + st * 2 * BM;
        bulk_load(stat, p.lse2 + (size_t)bh * p.nq_pad + q0, BM * 4, bQf + st);
        bulk_load(stat + BM, p.delta + (size_t)bh * p.nq_pad + q0, BM * 4, bQf + st);
        if (u > 0 && !mbar_wait(bDOe + st, (u - 1) & 1, abort_flag, kSiteBwdEmpty)) break;
        mbar_arrive_expect_tx(bDOf + st, C::kTile);
        for (int cb = 0; cb < 2; ++cb)
          tma_load_3d(sDO + st * C::kTile + cb * BM * 128, &tmDO, bDOf + st, cb * 64, q0, bh);
      }
    }
  } else if (warp == 13) {
    // ---------------- tcgen05 issuer ----------------
    if (lane == 0 && n_it > 0) {
      constexpr uint32_t idSS = make_idesc_bf16(BN, BM, 0, 0);   // S^T, dP^T: K-major A and B
      constexpr uint32_t idKMN = make_idesc_bf16(BN, D, 0, 1);   // dV, dK: A from TMEM, B MN-major
      constexpr uint32_t idQT = make_idesc_bf16(D, BM, 1, 1);    // dQ^T: A = K^T, B = dS^T, both MN-major
      const uint32_t aK = smem_u32(sK), aV = smem_u32(sV);
      auto issue_t = [&](uint32_t dcol, uint32_t aA, uint32_t aB) {
        const uint64_t da = make_sdesc_sw128(aA, 16, 1024), db = make_sdesc_sw128(aB, 16, 1024);
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
          const uint32_t off = (kk >> 2) * (BN * 128) + (kk & 3) * 32;
          const uint32_t offq = (kk >> 2) * (BM * 128) + (kk & 3) * 32;
          mma_ss(tmem + dcol, sdesc_add(da, off), sdesc_add(db, offq), idSS, kk > 0);
        }
      };
      auto issue_acc = [&](uint32_t dcol, uint32_t a_col, uint32_t aB, bool first) {
        const uint64_t db = make_sdesc_sw128(aB, BM * 128, 1024);
#pragma unroll
        for (int kk = 0; kk < BM / 16; ++kk) {
          mma_ts(tmem + dcol, tmem + a_col + (kk >> 2) * 64 + (kk & 3) * 8, sdesc_add(db, kk * 16 * 128),
                 idKMN, (!first || kk > 0));
        }
      };
      // dQ^T[d][q] = sum over key rows of K[kv][d] dS^T[kv][q]; both operands are
      // [kv][64-column block] 128-byte-swizzle tiles read along their rows
      const uint64_t dKt = make_sdesc_sw128(aK, BN * 128, 1024);
      const uint64_t dDS = make_sdesc_sw128(smem_u32(sDS), BN * 128, 1024);
      bool ok = mbar_wait(bKV, 0, abort_flag, kSiteBwdKV) && mbar_wait(bQf, 0, abort_flag, kSiteBwdLoad);
      if (ok) {
        tc_fence_after();
        issue_t(C::kColS, aK, smem_u32(sQ));
        mma_commit(bS);
        ok = mbar_wait(bDOf, 0, abort_flag, kSiteBwdLoad);
      }
      if (ok) {
        tc_fence_after();
        issue_t(C::kColDP, aV, smem_u32(sDO));
        mma_commit(bDP);
      }
      for (int it = 0; ok && it < n_it; ++it) {
        const int st = it % C::NSQ;
        const int nst = (it + 1) % C::NSQ;
        const uint32_t un = (it + 1) / C::NSQ;
        // dV += P^T dO
        if (!mbar_wait(bP, it & 1, abort_flag, kSiteBwdSoftmax)) break;
        tc_fence_after();
        issue_acc(C::kColDV, C::kColS, smem_u32(sDO + st * C::kTile), it == 0);
        mma_commit(bDOe + st);
        // S^T of the next query tile (issue order keeps it after dV_it's read of P^T)
        if (it + 1 < n_it) {
          if (!mbar_wait(bQf + nst, un & 1, abort_flag, kSiteBwdLoad)) break;
          tc_fence_after();
          issue_t(C::kColS, aK, smem_u32(sQ + nst * C::kTile));
          mma_commit(bS);
        }
        // dK += dS^T Q, then dQ^T = K^T dS^T into dP^T's columns
        if (!mbar_wait(bDS, it & 1, abort_flag, kSiteBwdDs)) break;
        tc_fence_after();
        issue_acc(C::kColDK, C::kColDP, smem_u32(sQ + st * C::kTile), it == 0);
#pragma unroll
        for (int kk = 0; kk < BN / 16; ++kk)
          mma_ss(tmem + C::kColDP, sdesc_add(dKt, kk * 16 * 128), sdesc_add(dDS, kk * 16 * 128), idQT, kk > 0);
        mma_commit(bQe + st);
        mma_commit(bDQ);
        // dP^T of the next query tile once dQ^T_it has left TMEM
        if (it + 1 < n_it) {
          if (!mbar_wait(bDQd, it & 1, abort_flag, kSiteBwdDq)) break;
          if (!mbar_wait(bDOf + nst, un & 1, abort_flag, kSiteBwdLoad)) break;
          tc_fence_after();
          issue_t(C::kColDP, aV, smem_u32(sDO + nst * C::kTile));
          mma_commit(bDP);
        }
      }
    }
  } else if (warp >= 8) {
    // ---------------- dQ drain (warp 8 + s reads TMEM lanes [32s, 32s+32): d = 32s + lane) ----------------
    const int sp = warp - 8;
    const uint32_t lane_base = static_cast<uint32_t>(sp * 32) << 16;
    const int d = sp * 32 + lane;
    float* acc_bh = pf.dq_acc + (size_t)bh * p.nq_pad * D + d;
    for (int it = 0; it < n_it; ++it) {
      const int q0 = (first_q + it) * BM;
      bool ok = mbar_wait(bDQ, it & 1, abort_flag, kSiteBwdDq);
      ok = __all_sync(0xffffffffu, ok);
      if (!ok) break;
      tc_fence_after();
      float* rowp = acc_bh + (size_t)q0 * D;
      uint32_t v[64];
      tmem_ld64(tmem + lane_base + C::kColDP, v);
#pragma unroll
      for (int c = 0; c < 64; ++c) red_add_f32(rowp + (size_t)c * D, __uint_as_float(v[c]));
      tmem_ld64(tmem + lane_base + C::kColDP + 64, v);
      tc_fence_before();
      mbar_arrive(bDQd);
#pragma unroll
      for (int c = 0; c < 64; ++c) red_add_f32(rowp + (size_t)(64 + c) * D, __uint_as_float(v[c]));
    }
  } else {
    // ---------------- compute warpgroups (warps 0-3: query cols 0-63, 4-7: 64-127) ----------------
    const int g = warp >> 2;
    const int r = tid & 127;                              // TMEM lane = key row
    const int kv_idx = kv0 + r;
    const uint32_t lane_base = static_cast<uint32_t>((warp & 3) * 32) << 16;
    const int cb = g * HC;
    // this thread's row of its dS^T block (128-byte swizzle: 16-byte chunk c at c ^ (r & 7))
    uint8_t* ds_row = sDS + g * (BN * 128) + (r >> 3) * 1024 + (r & 7) * 128;
    bool ok = true;
    for (int it = 0; it < n_it; ++it) {
      const int q0 = (first_q + it) * BM;
      const int st = it % C::NSQ;
      ok = mbar_wait(bQf + st, (it / C::NSQ) & 1, abort_flag, kSiteBwdLoad);
      ok = ok && mbar_wait(bS, it & 1, abort_flag, kSiteBwdMma);
      ok = __all_sync(0xffffffffu, ok);
      if (!ok) break;
      tc_fence_after();
      const float* lse_t = s_stats + st * 2 * BM + cb;
      const float* del_t = s_stats + st * 2 * BM + BM + cb;
      uint32_t pk[HC / 2];
      {
        uint32_t sr[HC];
        tmem_ld64(tmem + lane_base + C::kColS + cb, sr);
        const bool mask = p.causal && (q0 + cb < kv0 + BN - 1);
#pragma unroll
        for (int c4 = 0; c4 < HC; c4 += 4) {
          const float4 lv = *reinterpret_cast<const float4*>(lse_t + c4);
          float p0 = ex2(fmaf(__uint_as_float(sr[c4]), p.scale_log2, -lv.x));
          float p1 = ex2(fmaf(__uint_as_float(sr[c4 + 1]), p.scale_log2, -lv.y));
          float p2 = ex2(fmaf(__uint_as_float(sr[c4 + 2]), p.scale_log2, -lv.z));
          float p3 = ex2(fmaf(__uint_as_float(sr[c4 + 3]), p.scale_log2, -lv.w));
          if (mask) {
            const int qa = q0 + cb + c4;
            if (qa < kv_idx) p0 = 0.f;
            if (qa + 1 < kv_idx) p1 = 0.f;
            if (qa + 2 < kv_idx) p2 = 0.f;
            if (qa + 3 < kv_idx) p3 = 0.f;
          }
          pk[c4 / 2] = pack_bf16x2(p0, p1);
          pk[c4 / 2 + 1] = pack_bf16x2(p2, p3);
        }
      }
      tmem_st32(tmem + lane_base + C::kColS + cb, pk);
      tmem_wait_st();
      tc_fence_before();
      mbar_arrive(bP);

      ok = mbar_wait(bDP, it & 1, abort_flag, kSiteBwdMma);
      // the dS^T buffer is free once dQ^T_{it-1} (its only reader) has completed
      if (it > 0) ok = ok && mbar_wait(bDQ, (it - 1) & 1, abort_flag, kSiteBwdDq);
      ok = __all_sync(0xffffffffu, ok);
      if (!ok) break;
      tc_fence_after();
      {
        uint32_t dr[HC];
        tmem_ld64(tmem + lane_base + C::kColDP + cb, dr);
#pragma unroll
        for (int c4 = 0; c4 < HC; c4 += 4) {
          const float4 dl = *reinterpret_cast<const float4*>(del_t + c4);
          const uint32_t pa = pk[c4 / 2], pb = pk[c4 / 2 + 1];
          const float e0 = __uint_as_float(pa << 16) * (__uint_as_float(dr[c4]) - dl.x);
          const float e1 = __uint_as_float(pa & 0xFFFF0000u) * (__uint_as_float(dr[c4 + 1]) - dl.y);
          const float e2 = __uint_as_float(pb << 16) * (__uint_as_float(dr[c4 + 2]) - dl.z);
          const float e3 = __uint_as_float(pb & 0xFFFF0000u) * (__uint_as_float(dr[c4 + 3]) - dl.w);
          pk[c4 / 2] = pack_bf16x2(e0, e1);
          pk[c4 / 2 + 1] = pack_bf16x2(e2, e3);
        }
      }
      tmem_st32(tmem + lane_base + C::kColDP + cb, pk);
#pragma unroll
      for (int c = 0; c < 8; ++c) {
        *reinterpret_cast<uint4*>(ds_row + ((c ^ (r & 7)) << 4)) =
            make_uint4(pk[4 * c], pk[4 * c + 1], pk[4 * c + 2], pk[4 * c + 3]);
      }
      tmem_wait_st();
      fence_proxy_async_smem();
      tc_fence_before();
      mbar_arrive(bDS);
    }
    // epilogue: this warpgroup's D/2 columns of dV, dK for its key rows
    if (ok && n_it > 0) {
      ok = mbar_wait(bDQ, (n_it - 1) & 1, abort_flag, kSiteBwdMma);
      ok = __all_sync(0xffffffffu, ok);
    }
    if (ok) {
      const bool store = kv_idx < p.Nkv;
      constexpr int DC = D / 2;
      __nv_bfloat16* dvrow = p.dv + ((size_t)bh * p.Nkv + kv_idx) * D + g * DC;
      __nv_bfloat16* dkrow = p.dk + ((size_t)bh * p.Nkv + kv_idx) * D + g * DC;
      if (n_it > 0) {
        tc_fence_after();
        store_row_bf16(tmem + lane_base + C::kColDV + g * DC, DC / 32, 1.f, dvrow, store);
        store_row_bf16(tmem + lane_base + C::kColDK + g * DC, DC / 32, p.scale, dkrow, store);
      } else if (store) {
        const uint4 z = make_uint4(0, 0, 0, 0);
#pragma unroll
        for (int i = 0; i < DC / 8; ++i) {
          reinterpret_cast<uint4*>(dvrow)[i] = z;
          reinterpret_cast<uint4*>(dkrow)[i] = z;
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 13) {
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
}

// dq[bh][i][:] = bf16(scale * dq_acc[bh][i][:]) for i < Nq; 8 elements per thread.
template <int D>
__global__ void __launch_bounds__(256) dq_convert_kernel(const float* __restrict__ dq_acc,
                                                         __nv_bfloat16* __restrict__ dq, long long BH,
                                                         int Nq, int nq_pad, float scale) {
  constexpr int G = D / 8;
  const long long gid = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  const long long row = gid / G;
  const int sub = (int)(gid % G);
  if (row >= BH * Nq) return;
  const long long bh = row / Nq;
  const long long i = row % Nq;
  const float4* src = reinterpret_cast<const float4*>(dq_acc + (bh * nq_pad + i) * D + sub * 8);
  const float4 a = src[0], b = src[1];
  uint4 w;
  w.x = pack_bf16x2(a.x * scale, a.y * scale);
  w.y = pack_bf16x2(a.z * scale, a.w * scale);
  w.z = pack_bf16x2(b.x * scale, b.y * scale);
  w.w = pack_bf16x2(b.z * scale, b.w * scale);
  *reinterpret_cast<uint4*>(dq + row * D + sub * 8) = w;
}

// Per padded row (b, h, i < nq_pad): delta = rowsum(dO * O) and
// lse2 = LSE * log2(e); rows past Nq get delta = 0, lse2 = +inf (P = 0).
// With a dq_acc, the row's fp32 dQ accumulator is zeroed too.
// D/8 lanes per row.
template <int D>
__global__ void __launch_bounds__(256) prep_kernel(const __nv_bfloat16* __restrict__ o,
                                                   const __nv_bfloat16* __restrict__ dout,
                                                   const float* __restrict__ lse,
                                                   float* __restrict__ lse2, float* __restrict__ delta,
                                                   float* __restrict__ dq_acc,
                                                   long long BH, int Nq, int nq_pad) {
  constexpr int LPR = D / 8;
  const long long gtid = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  const long long prow = gtid / LPR;                // padded row index
  const int sub = (int)(gtid % LPR);
  const long long bh = prow / nq_pad;
  const int i = (int)(prow % nq_pad);
  const bool valid = bh < BH && i < Nq;
  const long long row = bh * Nq + i;                // dense row index
  float acc = 0.f;
  if (valid) {
    const uint4 a = *reinterpret_cast<const uint4*>(o + row * D + sub * 8);
    const uint4 b = *reinterpret_cast<const uint4*>(dout + row * D + sub * 8);
    const uint32_t ua[4] = {a.x, a.y, a.z, a.w};
    const uint32_t ub[4] = {b.x, b.y, b.z, b.w};
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      acc = fmaf(__uint_as_float(ua[k] << 16), __uint_as_float(ub[k] << 16), acc);
      acc = fmaf(__uint_as_float(ua[k] & 0xFFFF0000u), __uint_as_float(ub[k] & 0xFFFF0000u), acc);
    }
  }
#pragma unroll
  for (int off = LPR / 2; off > 0; off >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, off);
  if (bh < BH && sub == 0) {
    delta[prow] = valid ? acc : 0.f;
    lse2[prow] = valid ? lse[row] * kLog2e : INFINITY;
  }
  if (dq_acc != nullptr && bh < BH) {
    float4* z = reinterpret_cast<float4*>(dq_acc + prow * D + sub * 8);
    z[0] = make_float4(0.f, 0.f, 0.f, 0.f);
    z[1] = make_float4(0.f, 0.f, 0.f, 0.f);
  }
}

inline size_t round256(size_t x) { return (x + 255) / 256 * 256; }

inline long long nq_padded(long long Nq) { return (Nq + BM - 1) / BM * BM; }

// [lse2 fp32 BH*nq_pad][delta fp32 BH*nq_pad], then for D = 128 (the fused
// backward) the fp32 dQ accumulator [BH][nq_pad][D].
inline size_t stats_bytes(long long BH, long long Nq) {
  return round256((size_t)BH * nq_padded(Nq) * sizeof(float));
}

inline size_t workspace_bytes_for(long long BH, long long Nq, long long D) {
  size_t b = 2 * stats_bytes(BH, Nq);
  if (D == 128) b += round256((size_t)BH * nq_padded(Nq) * D * sizeof(float));
  return b;
}

template <int D>
int launch_bwd(const void* q, const void* k, const void* v, const void* o, const float* lse,
               const void* dout, void* dq, void* dk, void* dv, void* ws, long long B, long long H,
               long long Nq, long long Nkv, float sm_scale, int causal, bool fused, cudaStream_t st) {
  const long long BH = B * H;
  const long long nq_pad = nq_padded(Nq);
  if (BH > 65535) return set_error(PU_ERR_UNSUPPORTED, "B*H = %lld exceeds 65535", BH);
  fused = fused && D == 128;
  float* lse2 = static_cast<float*>(ws);
  float* delta = reinterpret_cast<float*>(static_cast<char*>(ws) + stats_bytes(BH, Nq));
  float* dq_acc = fused ? reinterpret_cast<float*>(static_cast<char*>(ws) + 2 * stats_bytes(BH, Nq)) : nullptr;
  {
    const long long threads = BH * nq_pad * (D / 8);
    const unsigned blocks = (unsigned)((threads + 255) / 256);
    prep_kernel<D><<<blocks, 256, 0, st>>>(static_cast<const __nv_bfloat16*>(o),
                                           static_cast<const __nv_bfloat16*>(dout), lse, lse2, delta,
                                           dq_acc, BH, (int)Nq, (int)nq_pad);
    int rc = check_cuda(cudaGetLastError(), "backward prep launch");
    if (rc) return rc;
  }
  CUtensorMap tq, tk, tv, tdo;
  int rc = make_tmap_bf16_3d(&tq, q, D, Nq, BH, 64, BM, true);
  if (!rc) rc = make_tmap_bf16_3d(&tk, k, D, Nkv, BH, 64, BN, true);
  if (!rc) rc = make_tmap_bf16_3d(&tv, v, D, Nkv, BH, 64, BN, true);
  if (!rc) rc = make_tmap_bf16_3d(&tdo, dout, D, Nq, BH, 64, BM, true);
  if (rc) return rc;
  Params prm{};
  prm.Nq = (int)Nq;
  prm.Nkv = (int)Nkv;
  prm.H = (int)H;
  prm.BH = (int)BH;
  prm.n_q_tiles = (int)((Nq + BM - 1) / BM);
  prm.n_kv_tiles = (int)((Nkv + BN - 1) / BN);
  prm.causal = causal ? 1 : 0;
  prm.scale_log2 = sm_scale * kLog2e;
  prm.scale = sm_scale;
  prm.nq_pad = (int)nq_pad;
  prm.lse2 = lse2;
  prm.delta = delta;
  prm.dq = static_cast<__nv_bfloat16*>(dq);
  prm.dk = static_cast<__nv_bfloat16*>(dk);
  prm.dv = static_cast<__nv_bfloat16*>(dv);
  if (fused) {
    rc = set_max_dynamic_smem(reinterpret_cast<const void*>(attn_bwd_fused_kernel), CfgF::kSmemBytes,
                              "cudaFuncSetAttribute(fused bwd smem)");
    if (rc) return rc;
    ParamsF pfz{prm, dq_acc};
    attn_bwd_fused_kernel<<<dim3((unsigned)((long long)prm.n_kv_tiles * BH)), kFusedThreads, CfgF::kSmemBytes,
                            st>>>(tq, tk, tv, tdo, pfz);
    rc = check_cuda(cudaGetLastError(), "fused backward launch");
    if (rc) return rc;
    const long long threads = BH * Nq * (D / 8);
    dq_convert_kernel<D><<<(unsigned)((threads + 255) / 256), 256, 0, st>>>(
        dq_acc, static_cast<__nv_bfloat16*>(dq), BH, (int)Nq, (int)nq_pad, sm_scale);
    return check_cuda(cudaGetLastError(), "dQ convert launch");
  }
  rc = set_max_dynamic_smem(reinterpret_cast<const void*>(attn_bwd_dkdv_kernel<D>), CfgKV<D>::kSmemBytes,
                            "cudaFuncSetAttribute(dkdv smem)");
  if (!rc)
    rc = set_max_dynamic_smem(reinterpret_cast<const void*>(attn_bwd_dq_kernel<D>), CfgQ<D>::kSmemBytes,
                              "cudaFuncSetAttribute(dq smem)");
  if (rc) return rc;
  attn_bwd_dkdv_kernel<D><<<dim3((unsigned)((long long)prm.n_kv_tiles * BH)), kThreads, CfgKV<D>::kSmemBytes, st>>>(
      tq, tk, tv, tdo, prm);
  rc = check_cuda(cudaGetLastError(), "backward dK/dV launch");
  if (rc) return rc;
  attn_bwd_dq_kernel<D><<<dim3((unsigned)((long long)prm.n_q_tiles * BH)), kThreads, CfgQ<D>::kSmemBytes, st>>>(
      tq, tk, tv, tdo, prm);
  return check_cuda(cudaGetLastError(), "backward dQ launch");
}

}  // namespace bwd
}  // namespace pu

extern "C" size_t pu_attn_bwd_workspace_size(int64_t B, int64_t H, int64_t Nq, int64_t D) {
  if (B <= 0 || H <= 0 || Nq <= 0 || D <= 0) return 0;
  return pu::bwd::workspace_bytes_for(B * H, Nq, D);
}

namespace pu {
namespace bwd {

inline int bwd_entry(const void* q, const void* k, const void* v, const void* o, const float* lse,
                     const void* dout, void* dq, void* dk, void* dv, void* workspace,
                     size_t workspace_bytes, int64_t B, int64_t H, int64_t Nq, int64_t Nkv, int64_t D,
                     float sm_scale, int causal, bool fused, void* stream) {
  int rc = pu::fwd::check_common(q, k, v, B, H, Nq, Nkv, D, sm_scale);
  if (rc) return rc;
  if (!o || !lse || !dout || !dq || !dk || !dv)
    return set_error(PU_ERR_INVALID_ARGUMENT, "null o/lse/dout/dq/dk/dv pointer");
  if (!aligned16(o) || !aligned16(dout) || !aligned16(dq) || !aligned16(dk) || !aligned16(dv))
    return set_error(PU_ERR_INVALID_ARGUMENT, "tensors must be 16-byte aligned");
  const size_t need = workspace_bytes_for(B * H, Nq, D);
  if (!workspace || workspace_bytes < need || (reinterpret_cast<uintptr_t>(workspace) & 255))
    return set_error(PU_ERR_WORKSPACE, "backward workspace needs %zu bytes (256-aligned), got %zu", need,
                     workspace_bytes);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (D == 128)
    return launch_bwd<128>(q, k, v, o, lse, dout, dq, dk, dv, workspace, B, H, Nq, Nkv, sm_scale, causal,
                           fused, st);
  return launch_bwd<64>(q, k, v, o, lse, dout, dq, dk, dv, workspace, B, H, Nq, Nkv, sm_scale, causal,
                        fused, st);
}

}  // namespace bwd
}  // namespace pu

extern "C" int pu_attn_bwd(const void* q, const void* k, const void* v, const void* o,
                           const float* lse, const void* dout, void* dq, void* dk, void* dv,
                           void* workspace, size_t workspace_bytes, int64_t B, int64_t H,
                           int64_t Nq, int64_t Nkv, int64_t D, float sm_scale, int causal,
                           void* stream) {
  return pu::bwd::bwd_entry(q, k, v, o, lse, dout, dq, dk, dv, workspace, workspace_bytes, B, H, Nq, Nkv,
                            D, sm_scale, causal, true, stream);
}

extern "C" int pu_attn_bwd_deterministic(const void* q, const void* k, const void* v, const void* o,
                                         const float* lse, const void* dout, void* dq, void* dk,
                                         void* dv, void* workspace, size_t workspace_bytes, int64_t B,
                                         int64_t H, int64_t Nq, int64_t Nkv, int64_t D, float sm_scale,
                                         int causal, void* stream) {
  return pu::bwd::bwd_entry(q, k, v, o, lse, dout, dq, dk, dv, workspace, workspace_bytes, B, H, Nq, Nkv,
                            D, sm_scale, causal, false, stream);
}
