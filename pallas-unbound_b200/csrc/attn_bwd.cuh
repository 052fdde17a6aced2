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
// Three kernels:
//   prep   : Delta (fp32), LSE in log2 units, zeroed fp32 dQ accumulator.
//   main   : one CTA per 128-row K/V tile of one (b, h); K and V stay in
//            shared memory while 128-row Q / dO tiles (with their LSE/Delta)
//            stream through 2-deep TMA rings.  Per query tile, with TMEM
//            lanes = key rows:
//              S^T  = K Q^T      -> TMEM [0,128)
//              dP^T = V dO^T     -> TMEM [128,256)
//              P^T  = exp2(S^T*scale*log2e - LSE*log2e)  (bf16, shared memory)
//              dV  += P^T dO     -> TMEM [256,256+D)
//              dS^T = P^T (dP^T - Delta)                  (bf16, over P^T)
//              dK  += dS^T Q     -> TMEM [384,384+D)
//              dQ_i = dS K       -> TMEM [128,128+D) (dP^T's columns)
//   post   : dQ = bf16(scale * dQ accumulator).
// Warp roles of the main kernel:
//   warps 0-7  two warpgroups, each owning 64 of the 128 query columns: P^T
//              and dS^T for every key row (thread = TMEM lane = key row), the
//              drain of dQ_i (thread = lane = query row): 32x32 fp32 chunks
//              staged with 128-byte swizzle in dO_i's consumed slot and added
//              into the fp32 accumulator with TMA bulk tensor reductions; and
//              their half of the dK/dV epilogue.
//   warp 8     TMA producer.   warp 9  tcgen05 issuer + TMEM owner.
// Tensor-core order per query tile i: dP_i, dV_i, S_{i+1}, dK_i, dQ_i — so
// S_{i+1} is ready when the warpgroups finish dS_i.
#pragma once

#include <cuda_bf16.h>

#include "pu_host.cuh"
#include "pu_ptx.cuh"

namespace pu {
namespace bwd {

constexpr int BM = 128;   // query rows per streamed tile
constexpr int BN = 128;   // key/value rows per CTA
constexpr int kThreads = 320;
constexpr float kLog2e = 1.4426950408889634f;
constexpr uint32_t kTmemCols = 512;
constexpr uint32_t kColS = 0, kColDP = 128, kColDV = 256, kColDK = 384;

template <int D>
struct Cfg {
  static constexpr int NSQ = 2;                  // Q / dO ring depth
  static constexpr int kTileQ = BM * D * 2;
  static constexpr int kTileKV = BN * D * 2;
  static constexpr int kTileP = BN * BM * 2;     // P^T / dS^T, bf16 [BN][BM]
  static constexpr int kStageBytes = 8 * 4096;   // dQ staging: 4 KB per compute warp
  // D = 128: the consumed dO slot (32 KB) stages dQ; D = 64: a dedicated buffer
  static constexpr bool kStageInDO = (kTileQ >= kStageBytes);
  static constexpr int kColBlocks = D / 64;
  static constexpr int kOffK = 0;
  static constexpr int kOffV = kOffK + kTileKV;
  static constexpr int kOffQ = kOffV + kTileKV;
  static constexpr int kOffDO = kOffQ + NSQ * kTileQ;
  static constexpr int kOffP = kOffDO + NSQ * kTileQ;
  static constexpr int kOffStage = kOffP + kTileP;
  static constexpr int kOffStats = kOffStage + (kStageInDO ? 0 : kStageBytes);  // [NSQ][lse2[BM], delta[BM]]
  static constexpr int kStatBytes = 2 * BM * 4;
  static constexpr int kOffBar = kOffStats + NSQ * kStatBytes;
  // barriers: KV, Qf[NSQ], Qe[NSQ], dOf[NSQ], dOe[NSQ], S, dP, P, dV, dS, dQf, dQfree, final
  static constexpr int kNumBars = 1 + 4 * NSQ + 8;
  static constexpr int kSmemBytes = kOffBar + kNumBars * 8 + 16;
  static_assert(kSmemBytes <= 232448, "shared memory budget");
};

struct Params {
  int Nq, Nkv, H;
  int n_q_tiles;
  int causal;
  float scale_log2;
  float scale;
  int nq_pad;              // row pitch of the stats arrays (multiple of BM)
  const float* lse2;       // [BH][nq_pad] LSE * log2(e), +inf past Nq
  const float* delta;      // [BH][nq_pad], 0 past Nq
  __nv_bfloat16* dk;
  __nv_bfloat16* dv;
};

// Byte offset of the 16-byte chunk `chunk` (8 bf16) of row `row` in a
// [rows][128] bf16 tile stored as two 64-column blocks with 128-byte swizzle
// (the layout a 64x`rows` TMA box with CU_TENSOR_MAP_SWIZZLE_128B produces).
__device__ __forceinline__ uint32_t sw128_offset(int row, int chunk, int rows) {
  const int cb = chunk >> 3;
  const int c = chunk & 7;
  return cb * rows * 128 + row * 128 + ((c ^ (row & 7)) << 4);
}

template <int D>
__global__ void __launch_bounds__(kThreads, 1)
    attn_bwd_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                    const __grid_constant__ CUtensorMap tmV, const __grid_constant__ CUtensorMap tmDO,
                    const __grid_constant__ CUtensorMap tmDQ, const Params p) {
  using C = Cfg<D>;
  constexpr int HC = BM / 2;               // query columns per compute warpgroup
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
  uint8_t* sP = smem + C::kOffP;
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
  uint64_t* bDV = bP + 1;
  uint64_t* bDS = bDV + 1;
  uint64_t* bDQf = bDS + 1;
  uint64_t* bDQfree = bDQf + 1;
  uint64_t* bFinal = bDQfree + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bFinal + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  // blockIdx.x walks the key tiles of one (b, h) — heaviest (causal: first)
  // first — and blockIdx.y the (b, h): CTAs resident together share a few
  // heads, so their Q/dO tiles and dQ accumulator rows stay in L2.
  const int kv_tile = blockIdx.x;
  const int bh = blockIdx.y;
  const int kv0 = kv_tile * BN;
  const int first_q = p.causal ? min(kv0 / BM, p.n_q_tiles) : 0;
  const int n_it = p.n_q_tiles - first_q;

  if (tid == 0) {
    mbar_init(bKV, 1);
    for (int s = 0; s < C::NSQ; ++s) {
      mbar_init(bQf + s, 1);
      mbar_init(bQe + s, 1);
      mbar_init(bDOf + s, 1);
      mbar_init(bDOe + s, 8);    // released by the 8 dQ-staging warps
    }
    mbar_init(bS, 1);
    mbar_init(bDP, 1);
    mbar_init(bP, 256);
    mbar_init(bDV, 1);
    mbar_init(bDS, 256);
    mbar_init(bDQf, 1);
    mbar_init(bDQfree, 256);
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
      constexpr uint32_t idKMN = make_idesc_bf16(BN, D, 0, 1);   // dV, dK: A K-major, B MN-major
      constexpr uint32_t idQ = make_idesc_bf16(BM, D, 1, 1);     // dQ: A (dS) MN-major, B (K) MN-major
      const uint32_t aK = smem_u32(sK), aV = smem_u32(sV), aP = smem_u32(sP);
      auto issue_S = [&](int it) {
        const uint32_t aQ = smem_u32(sQ + (it % C::NSQ) * C::kTileQ);
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
          const uint32_t off = (kk >> 2) * (BN * 128) + (kk & 3) * 32;
          const uint32_t offq = (kk >> 2) * (BM * 128) + (kk & 3) * 32;
          mma_ss(tmem + kColS, make_sdesc_sw128(aK + off, 16, 1024), make_sdesc_sw128(aQ + offq, 16, 1024),
                 idSS, kk > 0);
        }
        mma_commit(bS);
      };
      bool ok = mbar_wait(bKV, 0, abort_flag, kSiteBwdKV) && mbar_wait(bQf, 0, abort_flag, kSiteBwdLoad);
      if (ok) {
        tc_fence_after();
        issue_S(0);
      }
      for (int it = 0; ok && it < n_it; ++it) {
        const int st = it % C::NSQ;
        const uint32_t u = it / C::NSQ;
        const uint32_t aQ = smem_u32(sQ + st * C::kTileQ);
        const uint32_t aDO = smem_u32(sDO + st * C::kTileQ);
        // dP^T = V dO^T into dP's columns once dQ_{it-1} has been drained from them
        if (!mbar_wait(bDOf + st, u & 1, abort_flag, kSiteBwdLoad)) break;
        if (it > 0 && !mbar_wait(bDQfree, (it - 1) & 1, abort_flag, kSiteBwdDq)) break;
        tc_fence_after();
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
          const uint32_t off = (kk >> 2) * (BN * 128) + (kk & 3) * 32;
          const uint32_t offq = (kk >> 2) * (BM * 128) + (kk & 3) * 32;
          mma_ss(tmem + kColDP, make_sdesc_sw128(aV + off, 16, 1024),
                 make_sdesc_sw128(aDO + offq, 16, 1024), idSS, kk > 0);
        }
        mma_commit(bDP);
        // dV += P^T dO   (A = P^T [kv][q] K-major; B = dO [q][d] MN-major)
        if (!mbar_wait(bP, it & 1, abort_flag, kSiteBwdSoftmax)) break;
        tc_fence_after();
#pragma unroll
        for (int kk = 0; kk < BM / 16; ++kk) {
          const uint32_t offa = (kk >> 2) * (BN * 128) + (kk & 3) * 32;
          mma_ss(tmem + kColDV, make_sdesc_sw128(aP + offa, 16, 1024),
                 make_sdesc_sw128(aDO + kk * 16 * 128, BM * 128, 1024), idKMN, (it > 0 || kk > 0));
        }
        mma_commit(bDV);
        // next query tile's S^T: S's columns were read before P^T was published
        if (it + 1 < n_it) {
          if (!mbar_wait(bQf + (it + 1) % C::NSQ, ((it + 1) / C::NSQ) & 1, abort_flag, kSiteBwdLoad)) break;
          tc_fence_after();
          issue_S(it + 1);
        }
        // dK += dS^T Q ; dQ_it = dS K (into dP's columns)
        if (!mbar_wait(bDS, it & 1, abort_flag, kSiteBwdDs)) break;
        tc_fence_after();
#pragma unroll
        for (int kk = 0; kk < BM / 16; ++kk) {
          const uint32_t offa = (kk >> 2) * (BN * 128) + (kk & 3) * 32;
          mma_ss(tmem + kColDK, make_sdesc_sw128(aP + offa, 16, 1024),
                 make_sdesc_sw128(aQ + kk * 16 * 128, BM * 128, 1024), idKMN, (it > 0 || kk > 0));
        }
#pragma unroll
        for (int kk = 0; kk < BN / 16; ++kk) {
          mma_ss(tmem + kColDP, make_sdesc_sw128(aP + kk * 16 * 128, BN * 128, 1024),
                 make_sdesc_sw128(aK + kk * 16 * 128, BN * 128, 1024), idQ, kk > 0);
        }
        mma_commit(bDQf);
        mma_commit(bQe + st);
        if (it + 1 == n_it) mma_commit(bFinal);
      }
    }
  } else {
    // ---------------- compute warps 0-7 ----------------
    // Warpgroup g (warps 4g..4g+3) owns query columns [64g, 64g+64) of P^T,
    // dS^T and dQ; warp w reads TMEM lanes 32*(w%4).. (key rows for S^T/dP^T,
    // query rows for dQ).
    const int g = warp >> 2;
    const int r = tid & 127;                              // TMEM lane
    const int kv_idx = kv0 + r;
    const uint32_t lane_base = static_cast<uint32_t>((warp & 3) * 32) << 16;
    const int cbase = g * HC;                             // first query column of this warpgroup
    bool ok = true;

    // Drain dQ_j (this warpgroup's 64 columns of the rows in this warp's
    // lanes) into the fp32 accumulator: TMEM -> registers (then dP's columns
    // are released) -> 4 KB swizzled staging per 32x32 chunk -> TMA reduce-add.
    auto drain = [&](int j) -> bool {
      constexpr int DQC = D / 2;                      // dQ columns per warpgroup
      bool okd = mbar_wait(bDQf, j & 1, abort_flag, kSiteBwdDq);
      okd = __all_sync(0xffffffffu, okd);
      if (!okd) return false;
      tc_fence_after();
      uint32_t qh[DQC];
#pragma unroll
      for (int c = 0; c < DQC / 32; ++c)
        tmem_ld32(tmem + lane_base + kColDP + g * DQC + c * 32, *reinterpret_cast<uint32_t(*)[32]>(qh + c * 32));
      tmem_wait_ld();
      reg_fence(qh);
      tc_fence_before();
      mbar_arrive(bDQfree);
      const int q0j = (first_q + j) * BM;
      uint8_t* buf = (C::kStageInDO ? sDO + (j % C::NSQ) * C::kTileQ : smem + C::kOffStage) + warp * 4096;
#pragma unroll
      for (int c = 0; c < DQC / 32; ++c) {
        if (c > 0) {                    // single buffer: the previous reduction must have read it
          if (lane == 0) bulk_wait_group_read<0>();
          __syncwarp();
        }
#pragma unroll
        for (int k = 0; k < 8; ++k) {
          *reinterpret_cast<uint4*>(buf + lane * 128 + ((k ^ (lane & 7)) << 4)) =
              make_uint4(qh[c * 32 + 4 * k], qh[c * 32 + 4 * k + 1], qh[c * 32 + 4 * k + 2],
                         qh[c * 32 + 4 * k + 3]);
        }
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) {
          tma_reduce_add_3d(&tmDQ, buf, g * DQC + c * 32, q0j + (warp & 3) * 32, bh);
          bulk_commit_group();
        }
      }
      if (lane == 0) {
        bulk_wait_group_read<0>();
        mbar_arrive(bDOe + (j % C::NSQ));   // the staging (dO_j's slot) may be refilled
      }
      __syncwarp();
      return true;
    };

    for (int it = 0; it < n_it; ++it) {
      const int q0 = (first_q + it) * BM;
      const int st = it % C::NSQ;
      // the stage's row statistics (LSE*log2e, Delta) arrived with its Q tile
      ok = mbar_wait(bQf + st, (it / C::NSQ) & 1, abort_flag, kSiteBwdLoad);
      ok = __all_sync(0xffffffffu, ok);
      if (!ok) break;
      const float* lse_t = s_stats + st * 2 * BM + cbase;
      const float* del_t = s_stats + st * 2 * BM + BM + cbase;

      ok = mbar_wait(bS, it & 1, abort_flag, kSiteBwdMma);
      ok = __all_sync(0xffffffffu, ok);
      if (!ok) break;
      tc_fence_after();
      uint32_t pk[HC / 2];
      {
        uint32_t sr[HC];
        tmem_ld32(tmem + lane_base + kColS + cbase, *reinterpret_cast<uint32_t(*)[32]>(sr));
        tmem_ld32(tmem + lane_base + kColS + cbase + 32, *reinterpret_cast<uint32_t(*)[32]>(sr + 32));
        tmem_wait_ld();
        reg_fence(sr);
        const int qb = q0 + cbase;
        const bool need_mask = (p.causal && qb < kv0 + BN - 1) || (qb + HC > p.Nq) || (kv_idx >= p.Nkv);
        const int lo = p.causal ? kv_idx : 0;     // key kv_idx is visible to queries >= lo
        const bool kv_ok = kv_idx < p.Nkv;
#pragma unroll
        for (int c4 = 0; c4 < HC; c4 += 4) {
          const float4 lv = *reinterpret_cast<const float4*>(lse_t + c4);
          float p0 = ex2(fmaf(__uint_as_float(sr[c4]), p.scale_log2, -lv.x));
          float p1 = ex2(fmaf(__uint_as_float(sr[c4 + 1]), p.scale_log2, -lv.y));
          float p2 = ex2(fmaf(__uint_as_float(sr[c4 + 2]), p.scale_log2, -lv.z));
          float p3 = ex2(fmaf(__uint_as_float(sr[c4 + 3]), p.scale_log2, -lv.w));
          if (need_mask) {
            const int qa = qb + c4;
            if (!(kv_ok && qa >= lo && qa < p.Nq)) p0 = 0.f;
            if (!(kv_ok && qa + 1 >= lo && qa + 1 < p.Nq)) p1 = 0.f;
            if (!(kv_ok && qa + 2 >= lo && qa + 2 < p.Nq)) p2 = 0.f;
            if (!(kv_ok && qa + 3 >= lo && qa + 3 < p.Nq)) p3 = 0.f;
          }
          pk[c4 / 2] = pack_bf16x2(p0, p1);
          pk[c4 / 2 + 1] = pack_bf16x2(p2, p3);
        }
      }
      // dQ_{it-1}: its MMAs completing also frees the P^T/dS^T tile
      if (it > 0) {
        ok = drain(it - 1);
        if (!ok) break;
      }
#pragma unroll
      for (int ch = 0; ch < HC / 8; ++ch) {
        *reinterpret_cast<uint4*>(sP + sw128_offset(r, g * 8 + ch, BN)) =
            make_uint4(pk[ch * 4], pk[ch * 4 + 1], pk[ch * 4 + 2], pk[ch * 4 + 3]);
      }
      fence_proxy_async_smem();
      mbar_arrive(bP);

      // dS^T = P^T (dP^T - Delta)
      ok = mbar_wait(bDP, it & 1, abort_flag, kSiteBwdMma);
      ok = __all_sync(0xffffffffu, ok);
      if (!ok) break;
      tc_fence_after();
      {
        uint32_t dr[HC];
        tmem_ld32(tmem + lane_base + kColDP + cbase, *reinterpret_cast<uint32_t(*)[32]>(dr));
        tmem_ld32(tmem + lane_base + kColDP + cbase + 32, *reinterpret_cast<uint32_t(*)[32]>(dr + 32));
        tmem_wait_ld();
        reg_fence(dr);
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
      tc_fence_before();
      // dV has consumed P^T: overwrite the tile with dS^T
      ok = mbar_wait(bDV, it & 1, abort_flag, kSiteBwdMma);
      ok = __all_sync(0xffffffffu, ok);
      if (!ok) break;
#pragma unroll
      for (int ch = 0; ch < HC / 8; ++ch) {
        *reinterpret_cast<uint4*>(sP + sw128_offset(r, g * 8 + ch, BN)) =
            make_uint4(pk[ch * 4], pk[ch * 4 + 1], pk[ch * 4 + 2], pk[ch * 4 + 3]);
      }
      fence_proxy_async_smem();
      mbar_arrive(bDS);
    }
    if (ok && n_it > 0) ok = drain(n_it - 1);
    // epilogue: this warpgroup's 64 columns of dV, dK for the key rows in this
    // warp's lanes (TMEM loads are warp-wide; only rows inside the sequence
    // are stored)
    if (ok && n_it > 0) {
      ok = mbar_wait(bFinal, 0, abort_flag, kSiteBwdMma);
      ok = __all_sync(0xffffffffu, ok);
    }
    if (ok) {
      const bool store = kv_idx < p.Nkv;
      constexpr int DC = D / 2;                 // dV/dK columns per warpgroup
      __nv_bfloat16* dvrow = p.dv + ((size_t)bh * p.Nkv + kv_idx) * D + g * DC;
      __nv_bfloat16* dkrow = p.dk + ((size_t)bh * p.Nkv + kv_idx) * D + g * DC;
      if (n_it > 0) {
        tc_fence_after();
#pragma unroll 1
        for (int which = 0; which < 2; ++which) {
          const uint32_t col0 = (which ? kColDK : kColDV) + g * DC;
          const float sc = which ? p.scale : 1.f;
          __nv_bfloat16* rowp = which ? dkrow : dvrow;
#pragma unroll 1
          for (int c = 0; c < DC / 32; ++c) {
            uint32_t rr[32];
            tmem_ld32(tmem + lane_base + col0 + c * 32, rr);
            tmem_wait_ld();
            reg_fence(rr);
            uint32_t w[16];
#pragma unroll
            for (int i = 0; i < 16; ++i)
              w[i] = pack_bf16x2(__uint_as_float(rr[2 * i]) * sc, __uint_as_float(rr[2 * i + 1]) * sc);
            uint4* dst = reinterpret_cast<uint4*>(rowp + c * 32);
            if (store) {
#pragma unroll
              for (int i = 0; i < 4; ++i) dst[i] = make_uint4(w[4 * i], w[4 * i + 1], w[4 * i + 2], w[4 * i + 3]);
            }
          }
        }
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
    if (lane == 0) bulk_wait_group<0>();   // dQ reductions complete before exit
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 9) {
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
}

// Per row (b, h, i < nq_pad): delta = rowsum(dO * O), lse2 = LSE * log2(e)
// (rows past Nq: +inf and 0), and dQ accumulator row := 0.  D/8 lanes per row.
template <int D>
__global__ void __launch_bounds__(256) prep_kernel(const __nv_bfloat16* __restrict__ o,
                                                   const __nv_bfloat16* __restrict__ dout,
                                                   const float* __restrict__ lse,
                                                   float* __restrict__ lse2, float* __restrict__ delta,
                                                   float* __restrict__ dq_acc, long long BH, int Nq,
                                                   int nq_pad) {
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
    float4* z = reinterpret_cast<float4*>(dq_acc + row * D + sub * 8);
    z[0] = make_float4(0.f, 0.f, 0.f, 0.f);
    z[1] = make_float4(0.f, 0.f, 0.f, 0.f);
  }
#pragma unroll
  for (int off = LPR / 2; off > 0; off >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, off);
  if (bh < BH && sub == 0) {
    delta[prow] = valid ? acc : 0.f;
    lse2[prow] = valid ? lse[row] * kLog2e : INFINITY;
  }
}

// dQ (bf16) = scale * accumulator; 8 elements per thread.
__global__ void __launch_bounds__(256) post_kernel(const float* __restrict__ dq_acc,
                                                   __nv_bfloat16* __restrict__ dq, float scale,
                                                   long long n8) {
  const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n8) return;
  const float4 a = reinterpret_cast<const float4*>(dq_acc)[2 * i];
  const float4 b = reinterpret_cast<const float4*>(dq_acc)[2 * i + 1];
  uint4 w;
  w.x = pack_bf16x2(a.x * scale, a.y * scale);
  w.y = pack_bf16x2(a.z * scale, a.w * scale);
  w.z = pack_bf16x2(b.x * scale, b.y * scale);
  w.w = pack_bf16x2(b.z * scale, b.w * scale);
  reinterpret_cast<uint4*>(dq)[i] = w;
}

inline size_t round256(size_t x) { return (x + 255) / 256 * 256; }

inline long long nq_padded(long long Nq) { return (Nq + BM - 1) / BM * BM; }

// [dQ accumulator fp32 BH*Nq*D][lse2 fp32 BH*nq_pad][delta fp32 BH*nq_pad]
inline size_t workspace_bytes(long long BH, long long Nq, long long D) {
  return round256((size_t)BH * Nq * D * sizeof(float)) +
         2 * round256((size_t)BH * nq_padded(Nq) * sizeof(float));
}

template <int D>
int launch_bwd(const void* q, const void* k, const void* v, const void* o, const float* lse,
               const void* dout, void* dq, void* dk, void* dv, void* ws, long long B, long long H,
               long long Nq, long long Nkv, float sm_scale, int causal, cudaStream_t st) {
  using C = Cfg<D>;
  const long long BH = B * H;
  const long long nq_pad = nq_padded(Nq);
  float* dq_acc = static_cast<float*>(ws);
  float* lse2 = reinterpret_cast<float*>(static_cast<char*>(ws) + round256((size_t)BH * Nq * D * sizeof(float)));
  float* delta = reinterpret_cast<float*>(reinterpret_cast<char*>(lse2) + round256((size_t)BH * nq_pad * sizeof(float)));
  {
    const long long threads = BH * nq_pad * (D / 8);
    const unsigned blocks = (unsigned)((threads + 255) / 256);
    prep_kernel<D><<<blocks, 256, 0, st>>>(static_cast<const __nv_bfloat16*>(o),
                                           static_cast<const __nv_bfloat16*>(dout), lse, lse2, delta,
                                           dq_acc, BH, (int)Nq, (int)nq_pad);
    int rc = check_cuda(cudaGetLastError(), "backward prep launch");
    if (rc) return rc;
  }
  CUtensorMap tq, tk, tv, tdo, tdq;
  int rc = make_tmap_bf16_3d(&tq, q, D, Nq, BH, 64, BM, true);
  if (!rc) rc = make_tmap_bf16_3d(&tk, k, D, Nkv, BH, 64, BN, true);
  if (!rc) rc = make_tmap_bf16_3d(&tv, v, D, Nkv, BH, 64, BN, true);
  if (!rc) rc = make_tmap_bf16_3d(&tdo, dout, D, Nq, BH, 64, BM, true);
  if (!rc) rc = make_tmap_f32_3d(&tdq, dq_acc, D, Nq, BH, 32, 32, true);
  if (rc) return rc;
  static bool attr_done[64] = {false};
  const int dev = current_device();
  if (dev < 0) return PU_ERR_CUDA;
  if (dev >= 64 || !attr_done[dev]) {
    rc = check_cuda(cudaFuncSetAttribute(attn_bwd_kernel<D>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         C::kSmemBytes),
                    "cudaFuncSetAttribute(bwd smem)");
    if (rc) return rc;
    if (dev < 64) attr_done[dev] = true;
  }
  Params prm{};
  prm.Nq = (int)Nq;
  prm.Nkv = (int)Nkv;
  prm.H = (int)H;
  prm.n_q_tiles = (int)((Nq + BM - 1) / BM);
  prm.causal = causal ? 1 : 0;
  prm.scale_log2 = sm_scale * kLog2e;
  prm.scale = sm_scale;
  prm.nq_pad = (int)nq_pad;
  prm.lse2 = lse2;
  prm.delta = delta;
  prm.dk = static_cast<__nv_bfloat16*>(dk);
  prm.dv = static_cast<__nv_bfloat16*>(dv);
  const long long n_kv_tiles = (Nkv + BN - 1) / BN;
  if (BH > 65535) return set_error(PU_ERR_UNSUPPORTED, "B*H = %lld exceeds 65535", BH);
  dim3 grid((unsigned)n_kv_tiles, (unsigned)BH);
  attn_bwd_kernel<D><<<grid, kThreads, C::kSmemBytes, st>>>(tq, tk, tv, tdo, tdq, prm);
  rc = check_cuda(cudaGetLastError(), "backward main launch");
  if (rc) return rc;
  const long long n8 = BH * Nq * D / 8;
  post_kernel<<<(unsigned)((n8 + 255) / 256), 256, 0, st>>>(dq_acc, static_cast<__nv_bfloat16*>(dq),
                                                            sm_scale, n8);
  return check_cuda(cudaGetLastError(), "backward post launch");
}

}  // namespace bwd
}  // namespace pu

extern "C" size_t pu_attn_bwd_workspace_size(int64_t B, int64_t H, int64_t Nq, int64_t D) {
  if (B <= 0 || H <= 0 || Nq <= 0 || D <= 0) return 0;
  return pu::bwd::workspace_bytes(B * H, Nq, D);
}

extern "C" int pu_attn_bwd(const void* q, const void* k, const void* v, const void* o,
                           const float* lse, const void* dout, void* dq, void* dk, void* dv,
                           void* workspace, size_t workspace_bytes, int64_t B, int64_t H,
                           int64_t Nq, int64_t Nkv, int64_t D, float sm_scale, int causal,
                           void* stream) {
  using namespace pu::bwd;
  int rc = pu::fwd::check_common(q, k, v, B, H, Nq, Nkv, D, sm_scale);
  if (rc) return rc;
  if (!o || !lse || !dout || !dq || !dk || !dv)
    return pu::set_error(PU_ERR_INVALID_ARGUMENT, "null o/lse/dout/dq/dk/dv pointer");
  if (!pu::aligned16(o) || !pu::aligned16(dout) || !pu::aligned16(dq) || !pu::aligned16(dk) ||
      !pu::aligned16(dv))
    return pu::set_error(PU_ERR_INVALID_ARGUMENT, "tensors must be 16-byte aligned");
  const size_t need = pu::bwd::workspace_bytes(B * H, Nq, D);
  if (!workspace || workspace_bytes < need || (reinterpret_cast<uintptr_t>(workspace) & 255))
    return pu::set_error(PU_ERR_WORKSPACE, "backward workspace needs %zu bytes (256-aligned), got %zu",
                         need, workspace_bytes);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (D == 128)
    return launch_bwd<128>(q, k, v, o, lse, dout, dq, dk, dv, workspace, B, H, Nq, Nkv, sm_scale, causal, st);
  return launch_bwd<64>(q, k, v, o, lse, dout, dq, dk, dv, workspace, B, H, Nq, Nkv, sm_scale, causal, st);
}
