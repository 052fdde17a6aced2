// outproj.cuh — attention output projection fused with the tensor-parallel
// all-reduce, over NVLink peer memory.
//
// Reference: with heads sharded over the 'tp' mesh axis, each device computes
// its partial output projection Attention_local . W_O_local, and
// all_reduce_tp (src/pallas_flash/distributed/collectives.py:27-41, a psum)
// sums the partials so that every device holds the full activation.  Here,
// for G ranks (one process per GPU) holding O_g [T, K] and W_g [K, N] (bf16,
// row-major), every rank ends with Y = sum_g O_g W_g [T, N] (bf16):
//
//   outproj_gemm_kernel  persistent tcgen05 GEMM (one CTA per SM) over
//       128 x 256 output tiles: TMA loads of 128 x 64 O and 64 x 256 W tiles
//       through a 4-stage ring, fp32 accumulators double-buffered in TMEM so
//       a tile's epilogue overlaps the next tile's products.  The epilogue
//       rounds the tile to bf16 and stores it straight from registers into
//       the staging area of the tile's owner rank (t mod G) over NVLink, then
//       raises a flag there: the reduce-scatter's traffic leaves tile by tile
//       while the tensor cores keep multiplying.
//   outproj_gemm_pair_kernel  the same for T a multiple of 256 on CTA pairs
//       (clusters of two): 256 x 256 tiles, one tcgen05.mma.cta_group::2
//       product per K step with each CTA holding half of the O rows and half
//       of the W columns, which cuts the operand traffic per output by a
//       third; each CTA's epilogue handles its 128 x 256 half exactly as the
//       single-CTA kernel handles a tile.
//   reduce_bcast_kernel  each owner waits (bounded) for its tiles' G partials,
//       sums them in fp32 in rank order, rounds to bf16 and stores the result
//       tile into its own result area (local stores), raising its own flag.
//   receive_kernel       each rank waits (bounded) for every result tile's
//       flag in the owner's buffer and reads the tile from there (plain loads
//       over NVLink for the other owners) into the caller's Y.  Pulling the
//       results replaced owners storing every result tile into every rank's
//       buffer: per-thread 16-byte stores to peer memory moved ~390 GB/s.
// Every rank's Y is bitwise identical (each tile is reduced once, by its
// owner).  Partials travel as bf16, as an all-reduce of bf16 data would.
//
// Tiles in the exchange buffers are chunk-major: 16-byte chunk c (8 columns)
// of row r at chunk index c * 128 + r, so the 32 rows a warp holds after a
// TMEM load land in 512 contiguous bytes.
//
// Exchange buffer of one rank (pu_peer_alloc; zeroed once):
//   partials [2][G][n_owned][128*256] bf16   slot (epoch & 1)
//   results  [2][n_tiles][128*256] bf16
//   flags    partial [2][G][n_owned] u32, result [2][n_tiles] u32 (epochs)
// Double buffering by epoch parity is sufficient.  Partials: a rank's call
// e+2 starts after its receive of e+1, which needed every owner's reduce of
// e+1, which each owner ran after its reduce of e (stream order).  Results:
// an owner writes call e+2's results after every rank's partials of e+2
// arrived, and each rank stores those only after its receive of e+1, so
// after its receive of e.
#pragma once

#include <cuda_bf16.h>

#include <algorithm>
#include <cstdlib>
#include <mutex>

#include "pu_host.cuh"
#include "pu_ptx.cuh"

namespace pu {
namespace outproj {

constexpr int BM = 128;            // output rows (tokens) per tile
constexpr int BN = 256;            // output columns per tile (one tcgen05.mma N)
constexpr int BK = 64;             // K per pipeline stage (one 128-byte swizzle span)
constexpr int NS = 4;              // pipeline stages
constexpr int kThreads = 192;      // producer warp, MMA warp, 4 epilogue warps
constexpr int kTileA = BM * BK * 2;
constexpr int kTileB = BK * BN * 2;
constexpr int kStage = kTileA + kTileB;
constexpr int kOffBar = NS * kStage;
// barriers: full[NS], empty[NS], acc_full[2], acc_empty[2]
constexpr int kSmemBytes = kOffBar + 8 * (2 * NS + 4) + 16;
constexpr int kTileBytes = BM * BN * 2;   // one bf16 output tile (64 KB)
constexpr int kChunksPerRow = BN * 2 / 16;
constexpr int kMaxRanks = 8;
// CTA-pair kernel (T a multiple of 256): 256 x 256 tiles, one M = 256 product
// per K step over the pair; each CTA holds 128 rows of the O tile and 128
// columns of the W tile per stage (32 KB), so a pair reads 2 MB of operands
// per 256 x 256 tile where two single-CTA tiles read 3 MB.
constexpr int kPairRows = 2 * BM;
constexpr int kPairStages = 6;
constexpr int kTileBHalf = BK * (BN / 2) * 2;
constexpr int kPairStage = kTileA + kTileBHalf;
constexpr int kPairOffBar = kPairStages * kPairStage;
// barriers: full[S], empty[S], acc_full[2], acc_empty[2]
constexpr int kPairSmemBytes = kPairOffBar + 8 * (2 * kPairStages + 4) + 16;

struct Layout {
  int n_tiles, n_owned;
  size_t off_part, off_res, off_pflag, off_rflag, total;
};

inline Layout layout(long long T, long long N, long long G) {
  Layout l{};
  l.n_tiles = (int)((T / BM) * (N / BN));
  l.n_owned = (int)((l.n_tiles + G - 1) / G);
  l.off_part = 0;
  l.off_res = l.off_part + (size_t)2 * G * l.n_owned * kTileBytes;
  l.off_pflag = l.off_res + (size_t)2 * l.n_tiles * kTileBytes;
  l.off_rflag = l.off_pflag + ((size_t)2 * G * l.n_owned * 4 + 255) / 256 * 256;
  l.total = l.off_rflag + ((size_t)2 * l.n_tiles * 4 + 255) / 256 * 256;
  return l;
}

struct Params {
  unsigned char* exch[kMaxRanks];  // this process's pointer to each rank's exchange buffer
  int G, rank;
  unsigned epoch;
  int n_k;                         // K / BK
  int n_ntiles;                    // N / BN
  int n_tiles, n_owned;
  int n_pair_tiles;                // (T / 256) * (N / 256) for the CTA-pair kernel
  size_t off_part, off_res, off_pflag, off_rflag;
  uint64_t timeout_ns;
  __nv_bfloat16* y;                // caller's output [T, N]
  int N;
};

__device__ __forceinline__ size_t part_off(const Params& p, int src, int j) {
  return p.off_part + ((size_t)((p.epoch & 1u) * p.G + src) * p.n_owned + j) * kTileBytes;
}
__device__ __forceinline__ size_t res_off(const Params& p, int t) {
  return p.off_res + ((size_t)(p.epoch & 1u) * p.n_tiles + t) * kTileBytes;
}
__device__ __forceinline__ size_t pflag_off(const Params& p, int src, int j) {
  return p.off_pflag + ((size_t)((p.epoch & 1u) * p.G + src) * p.n_owned + j) * 4;
}
__device__ __forceinline__ size_t rflag_off(const Params& p, int t) {
  return p.off_rflag + ((size_t)(p.epoch & 1u) * p.n_tiles + t) * 4;
}

__device__ __forceinline__ unsigned ld_acquire_sys(const unsigned* f) {
  unsigned v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(f) : "memory");
  return v;
}
__device__ __forceinline__ void st_release_sys(unsigned* f, unsigned v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(f), "r"(v) : "memory");
}
// Bounded wait until *f == epoch.
__device__ __forceinline__ bool wait_flag(const unsigned* f, unsigned epoch, uint64_t timeout_ns) {
  if (ld_acquire_sys(f) == epoch) return true;
  const uint64_t t0 = global_timer_ns();
  while (ld_acquire_sys(f) != epoch) {
    if (global_timer_ns() - t0 > timeout_ns) return false;
    __nanosleep(128);
  }
  return true;
}
__device__ __forceinline__ void named_bar(int id, int n) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(n) : "memory");
}

// Epilogue of one 128 x 256 output tile `tile` (row-major tile index over
// T/128 x N/256) held in TMEM columns [acc, acc + 256) of lanes 0-127: warp
// quarter q = warp % 4 reads lanes 32q..32q+31 (thread = tile row r) and
// stores the bf16 row into Y (one rank) or chunk-major into the tile owner's
// partial slot (then raises the owner's flag once all 128 threads stored).
// Called by the four epilogue warps (128 threads, named barrier 1).
__device__ __forceinline__ void epilogue_tile(const Params& p, uint32_t tmem_acc, int tile, int tid) {
  const int warp = tid >> 5, lane = tid & 31;
  const int q = warp & 3;
  const int r = q * 32 + lane;                      // tile row
  const uint32_t lane_base = static_cast<uint32_t>(q * 32) << 16;
  const int owner = tile % p.G;
  uint4* dst = reinterpret_cast<uint4*>(p.exch[owner] + part_off(p, p.rank, tile / p.G));
  // one rank: nothing to reduce, the tile goes straight into Y (row-major)
  uint4* ydst = reinterpret_cast<uint4*>(p.y + (size_t)((tile / p.n_ntiles) * BM + r) * p.N +
                                         (tile % p.n_ntiles) * BN);
#pragma unroll 1
  for (int c = 0; c < BN / 32; ++c) {
    uint32_t v[32];
    tmem_ld32(tmem_acc + lane_base + c * 32, v);
    tmem_wait_ld();
    reg_fence(v);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const uint4 w = make_uint4(pack_bf16x2(__uint_as_float(v[8 * j]), __uint_as_float(v[8 * j + 1])),
                                 pack_bf16x2(__uint_as_float(v[8 * j + 2]), __uint_as_float(v[8 * j + 3])),
                                 pack_bf16x2(__uint_as_float(v[8 * j + 4]), __uint_as_float(v[8 * j + 5])),
                                 pack_bf16x2(__uint_as_float(v[8 * j + 6]), __uint_as_float(v[8 * j + 7])));
      if (p.G == 1)
        ydst[c * 4 + j] = w;
      else
        dst[(c * 4 + j) * BM + r] = w;              // chunk-major: a warp writes 512 bytes
    }
  }
}

__device__ __forceinline__ void epilogue_flag(const Params& p, int tile, int tid) {
  if (p.G == 1) return;
  named_bar(1, 128);
  if (tid == 64) {
    // the barrier orders the other threads' stores before this fence
    __threadfence_system();
    st_release_sys(reinterpret_cast<unsigned*>(p.exch[tile % p.G] + pflag_off(p, p.rank, tile / p.G)), p.epoch);
  }
}

// Persistent GEMM + bf16 partial tiles to their owner ranks.
__global__ void __launch_bounds__(kThreads, 1)
    outproj_gemm_kernel(const __grid_constant__ CUtensorMap tmO, const __grid_constant__ CUtensorMap tmW,
                        const Params p) {
  extern __shared__ __align__(1024) uint8_t smem[];
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  if (smem_u32(smem) & 1023u) {
    if (tid == 0) record_device_error(PU_ERR_UNSUPPORTED, kSiteOutProj);
    return;
  }
  uint64_t* bFull = reinterpret_cast<uint64_t*>(smem + kOffBar);
  uint64_t* bEmpty = bFull + NS;
  uint64_t* bAccFull = bEmpty + NS;   // [2] accumulator a complete
  uint64_t* bAccEmpty = bAccFull + 2; // [2] accumulator a read out by the epilogue
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bAccEmpty + 2);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  if (tid == 0) {
    for (int s = 0; s < NS; ++s) {
      mbar_init(bFull + s, 1);
      mbar_init(bEmpty + s, 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(bAccFull + a, 1);
      mbar_init(bAccEmpty + a, 128);
    }
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, 2 * BN);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) {
      tma_prefetch_desc(&tmO);
      tma_prefetch_desc(&tmW);
      int g = 0;                                      // stages loaded so far
      bool ok = true;
      for (int tile = blockIdx.x; ok && tile < p.n_tiles; tile += gridDim.x) {
        const int m0 = (tile / p.n_ntiles) * BM, n0 = (tile % p.n_ntiles) * BN;
        for (int s = 0; s < p.n_k; ++s, ++g) {
          const int st = g % NS;
          const uint32_t u = g / NS;
          if (u > 0 && !mbar_wait(bEmpty + st, (u - 1) & 1, abort_flag, kSiteOutProj)) { ok = false; break; }
          uint8_t* sa = smem + st * kStage;
          uint8_t* sb = sa + kTileA;
          mbar_arrive_expect_tx(bFull + st, kStage);
          tma_load_3d(sa, &tmO, bFull + st, s * BK, m0, 0);
          for (int b = 0; b < BN / 64; ++b)
            tma_load_3d(sb + b * (BK * 128), &tmW, bFull + st, n0 + b * 64, s * BK, 0);
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // A: O tile, K-major; B: W tile, MN-major (N contiguous), 64-column
      // blocks of BK rows each LBO = BK * 128 bytes apart
      constexpr uint32_t idesc = make_idesc_bf16(BM, BN, 0, 1);
      int g = 0, i = 0;
      bool ok = true;
      for (int tile = blockIdx.x; ok && tile < p.n_tiles; tile += gridDim.x, ++i) {
        const int a = i & 1;
        if (i >= 2 && !mbar_wait(bAccEmpty + a, ((i >> 1) - 1) & 1, abort_flag, kSiteOutProj)) break;
        tc_fence_after();
        for (int s = 0; s < p.n_k; ++s, ++g) {
          const int st = g % NS;
          if (!mbar_wait(bFull + st, (g / NS) & 1, abort_flag, kSiteOutProj)) { ok = false; break; }
          tc_fence_after();
          const uint64_t da = make_sdesc_sw128(smem_u32(smem + st * kStage), 16, 1024);
          const uint64_t db = make_sdesc_sw128(smem_u32(smem + st * kStage + kTileA), BK * 128, 1024);
#pragma unroll
          for (int kk = 0; kk < BK / 16; ++kk)
            mma_ss(tmem + a * BN, sdesc_add(da, kk * 32), sdesc_add(db, kk * 16 * 128), idesc, (s > 0 || kk > 0));
          mma_commit(bEmpty + st);
        }
        if (ok) mma_commit(bAccFull + a);
      }
    }
  } else {
    // epilogue: warps 2-5; TMEM lane quarter = warp % 4
    int i = 0;
    for (int tile = blockIdx.x; tile < p.n_tiles; tile += gridDim.x, ++i) {
      const int a = i & 1;
      bool ok = mbar_wait(bAccFull + a, (i >> 1) & 1, abort_flag, kSiteOutProj);
      ok = __all_sync(0xffffffffu, ok);
      if (!ok) break;
      tc_fence_after();
      epilogue_tile(p, tmem + a * BN, tile, tid);
      tc_fence_before();
      mbar_arrive(bAccEmpty + a);                     // TMEM accumulator a is free again
      epilogue_flag(p, tile, tid);
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 2 * BN);
  }
}

// The same GEMM over CTA pairs (clusters of two): the even CTA's thread
// issues tcgen05.mma.cta_group::2 products of 256 x 256 x 16, A = the pair's
// 256 O rows (128 in each CTA's shared memory), B = the tile's 256 W columns
// (128 in each CTA's shared memory); each CTA's TMEM holds its 128 rows of
// the fp32 accumulator (double-buffered, 2 x 256 columns).
//   warp 0   TMA producer of each CTA: its O rows and W columns; the loads of
//            both CTAs count on the even CTA's full barrier (armed by the
//            even CTA for the bytes of both)
//   warp 1   even CTA: the product issuer; it commits each stage's products to
//            both CTAs' empty barriers and each tile's to both CTAs'
//            accumulator barriers; both CTAs: TMEM allocation
//   warps 2-5 epilogue of each CTA: its 128-row half of the tile (one of the
//            128 x 256 tiles of the single-CTA kernel, so the exchange,
//            reduction and receive steps are shared), then an arrival on the
//            even CTA's accumulator-empty barrier
// Every wait is bounded; both CTAs always reach the closing cluster barrier,
// after which no CTA touches the other's shared memory.
__global__ void __launch_bounds__(kThreads, 1)
    outproj_gemm_pair_kernel(const __grid_constant__ CUtensorMap tmO, const __grid_constant__ CUtensorMap tmW,
                             const Params p) {
  extern __shared__ __align__(1024) uint8_t smem[];
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  if (smem_u32(smem) & 1023u) {                     // the same in both CTAs of a pair
    if (tid == 0) record_device_error(PU_ERR_UNSUPPORTED, kSiteOutProj);
    return;
  }
  const uint32_t rank = cluster_ctarank();
  const bool lead = rank == 0;
  const int pair = (int)blockIdx.x >> 1, n_pairs = (int)gridDim.x >> 1;
  uint64_t* bFull = reinterpret_cast<uint64_t*>(smem + kPairOffBar);
  uint64_t* bEmpty = bFull + kPairStages;
  uint64_t* bAccFull = bEmpty + kPairStages;  // [2] accumulator a complete
  uint64_t* bAccEmpty = bAccFull + 2;         // [2] (even CTA) accumulator a read out by both epilogues
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bAccEmpty + 2);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  if (tid == 0) {
    for (int s = 0; s < kPairStages; ++s) {
      mbar_init(bFull + s, 1);
      mbar_init(bEmpty + s, 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(bAccFull + a, 1);
      mbar_init(bAccEmpty + a, 8);                  // 4 epilogue warps x 2 CTAs
    }
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 1) {
    tmem_alloc_pair(tmem_slot, 2 * BN);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  cluster_sync();                                   // barriers of both CTAs initialised
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) {
      tma_prefetch_desc(&tmO);
      tma_prefetch_desc(&tmW);
      int g = 0;                                    // stages loaded so far
      bool ok = true;
      for (int tile = pair; ok && tile < p.n_pair_tiles; tile += n_pairs) {
        const int m0 = (tile / p.n_ntiles) * kPairRows + (int)rank * BM;
        const int n0 = (tile % p.n_ntiles) * BN + (int)rank * (BN / 2);
        for (int s = 0; s < p.n_k; ++s, ++g) {
          const int st = g % kPairStages;
          const uint32_t u = g / kPairStages;
          if (u > 0 && !mbar_wait(bEmpty + st, (u - 1) & 1, abort_flag, kSiteOutProj)) { ok = false; break; }
          uint8_t* sa = smem + st * kPairStage;
          uint8_t* sb = sa + kTileA;
          const uint32_t full_lead = mapa_shared(bFull + st, 0);
          if (lead) mbar_arrive_expect_tx(bFull + st, 2 * kPairStage);
          tma_load_3d_pair(sa, &tmO, full_lead, s * BK, m0, 0);
          for (int b = 0; b < BN / 2 / 64; ++b)
            tma_load_3d_pair(sb + b * (BK * 128), &tmW, full_lead, n0 + b * 64, s * BK, 0);
        }
      }
      if (lead) {
        // copies still in flight (the peer's included: they count on these
        // barriers) land before the pair may exit
        volatile int no_abort = 0;
        for (int h = max(0, g - kPairStages); h < g; ++h)
          mbar_wait(bFull + h % kPairStages, (h / kPairStages) & 1, &no_abort, kSiteOutProj);
      }
    }
  } else if (warp == 1) {
    if (lead && lane == 0) {
      // A: O rows, K-major; B: W columns, MN-major (N contiguous), 64-column
      // blocks of BK rows each LBO = BK * 128 bytes apart (two per CTA)
      constexpr uint32_t idesc = make_idesc_bf16(kPairRows, BN, 0, 1);
      int g = 0, i = 0;
      bool ok = true;
      for (int tile = pair; ok && tile < p.n_pair_tiles; tile += n_pairs, ++i) {
        const int a = i & 1;
        if (i >= 2 && !mbar_wait(bAccEmpty + a, ((i >> 1) - 1) & 1, abort_flag, kSiteOutProj)) break;
        tc_fence_after();
        for (int s = 0; s < p.n_k; ++s, ++g) {
          const int st = g % kPairStages;
          if (!mbar_wait(bFull + st, (g / kPairStages) & 1, abort_flag, kSiteOutProj)) { ok = false; break; }
          tc_fence_after();
          const uint64_t da = make_sdesc_sw128(smem_u32(smem + st * kPairStage), 16, 1024);
          const uint64_t db = make_sdesc_sw128(smem_u32(smem + st * kPairStage + kTileA), BK * 128, 1024);
#pragma unroll
          for (int kk = 0; kk < BK / 16; ++kk)
            mma_ss_pair(tmem + a * BN, sdesc_add(da, kk * 32), sdesc_add(db, kk * 16 * 128), idesc,
                        (s > 0 || kk > 0));
          mma_commit_pair(mapa_shared(bEmpty + st, 0));
          mma_commit_pair(mapa_shared(bEmpty + st, 1));
        }
        if (ok) {
          mma_commit_pair(mapa_shared(bAccFull + a, 0));
          mma_commit_pair(mapa_shared(bAccFull + a, 1));
        }
      }
    }
  } else {
    // epilogue: warps 2-5 of each CTA (TMEM lane quarter = warp % 4), its 128
    // rows of the pair tile
    int i = 0;
    for (int tile = pair; tile < p.n_pair_tiles; tile += n_pairs, ++i) {
      const int a = i & 1;
      bool ok = mbar_wait(bAccFull + a, (i >> 1) & 1, abort_flag, kSiteOutProj);
      ok = __all_sync(0xffffffffu, ok);
      if (!ok) break;
      tc_fence_after();
      // this half is tile t of the single-CTA numbering (128 x 256 tiles)
      const int t = ((tile / p.n_ntiles) * 2 + (int)rank) * p.n_ntiles + tile % p.n_ntiles;
      epilogue_tile(p, tmem + a * BN, t, tid);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_cluster(mapa_shared(bAccEmpty + a, 0));   // accumulator a read out here
      epilogue_flag(p, t, tid);
    }
  }
  tc_fence_before();
  cluster_sync();                                   // no remote arrival or product is still pending
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc_pair(tmem, 2 * BN);
  }
}

// Owner: sum the G partials of each owned tile in rank order, broadcast.
__global__ void __launch_bounds__(256) reduce_bcast_kernel(const Params p) {
  const int j = blockIdx.x;
  const int t = j * p.G + p.rank;
  if (t >= p.n_tiles) return;
  __shared__ int s_ok;
  if (threadIdx.x == 0) s_ok = 1;
  __syncthreads();
  unsigned char* mine = p.exch[p.rank];
  if ((int)threadIdx.x < p.G) {
    const unsigned* f = reinterpret_cast<const unsigned*>(mine + pflag_off(p, threadIdx.x, j));
    if (!wait_flag(f, p.epoch, p.timeout_ns)) {
      record_device_error(PU_ERR_DEVICE_TIMEOUT, kSiteOutProj);
      s_ok = 0;
    }
  }
  __syncthreads();
  if (!s_ok) return;
  // eight chunks per thread in flight: G partial chunks each, summed in rank
  // order in fp32 (the layout is the partials', so the result stays
  // chunk-major)
  constexpr int kChunks = kTileBytes / 16;
  constexpr int kU = 8;
  for (int c0 = threadIdx.x; c0 < kChunks; c0 += kU * blockDim.x) {
    float acc[kU][8];
#pragma unroll
    for (int u = 0; u < kU; ++u)
#pragma unroll
      for (int i = 0; i < 8; ++i) acc[u][i] = 0.f;
    for (int s = 0; s < p.G; ++s) {
      const uint4* src = reinterpret_cast<const uint4*>(mine + part_off(p, s, j));
      uint4 v[kU];
#pragma unroll
      for (int u = 0; u < kU; ++u) v[u] = __ldcv(src + c0 + u * blockDim.x);
#pragma unroll
      for (int u = 0; u < kU; ++u) {
        const uint32_t w[4] = {v[u].x, v[u].y, v[u].z, v[u].w};
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          acc[u][2 * i] += __uint_as_float(w[i] << 16);
          acc[u][2 * i + 1] += __uint_as_float(w[i] & 0xFFFF0000u);
        }
      }
    }
#pragma unroll
    for (int u = 0; u < kU; ++u) {
      const uint4 out = make_uint4(pack_bf16x2(acc[u][0], acc[u][1]), pack_bf16x2(acc[u][2], acc[u][3]),
                                   pack_bf16x2(acc[u][4], acc[u][5]), pack_bf16x2(acc[u][6], acc[u][7]));
      *(reinterpret_cast<uint4*>(mine + res_off(p, t)) + c0 + u * blockDim.x) = out;
    }
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    // the barrier orders the other threads' stores before this fence
    __threadfence_system();
    st_release_sys(reinterpret_cast<unsigned*>(mine + rflag_off(p, t)), p.epoch);
  }
}

// Every rank: wait for each result tile's flag in its owner's buffer, then
// read the tile from the owner's memory (over NVLink for the other ranks'
// tiles) and copy it into Y, 32 rows at a time through shared memory
// (chunk-major tile -> row-major Y, both sides coalesced).
__global__ void __launch_bounds__(256) receive_kernel(const Params p) {
  __shared__ int s_ok;
  __shared__ uint4 slab[32][kChunksPerRow + 1];      // +1: conflict-free transposed reads
  const int tid = threadIdx.x;
  for (int t = blockIdx.x; t < p.n_tiles; t += gridDim.x) {
    const unsigned char* owner = p.exch[t % p.G];
    if (tid == 0) {
      s_ok = wait_flag(reinterpret_cast<const unsigned*>(owner + rflag_off(p, t)), p.epoch, p.timeout_ns);
      if (!s_ok) record_device_error(PU_ERR_DEVICE_TIMEOUT, kSiteOutProj);
    }
    __syncthreads();
    const bool ok = s_ok;
    if (!ok) return;
    const int m0 = (t / p.n_ntiles) * BM, n0 = (t % p.n_ntiles) * BN;
    const uint4* src = reinterpret_cast<const uint4*>(owner + res_off(p, t));
    for (int r0 = 0; r0 < BM; r0 += 32) {
      // chunk c of rows r0..r0+31 is 512 contiguous bytes
      for (int e = tid; e < 32 * kChunksPerRow; e += blockDim.x) {
        const int c = e >> 5, rr = e & 31;
        slab[rr][c] = __ldcv(src + c * BM + r0 + rr);
      }
      __syncthreads();
      for (int e = tid; e < 32 * kChunksPerRow; e += blockDim.x) {
        const int rr = e / kChunksPerRow, c = e % kChunksPerRow;
        *reinterpret_cast<uint4*>(p.y + (size_t)(m0 + r0 + rr) * p.N + n0 + c * 8) = slab[rr][c];
      }
      __syncthreads();
    }
  }
}

// The CTA-pair kernel serves T % 256 == 0 unless PU_OUTPROJ_PAIR=0 (the
// single-CTA kernel then serves every shape; tests compare the two).
inline bool pair_kernel_enabled() {
  const char* e = getenv("PU_OUTPROJ_PAIR");
  return !(e && e[0] == '0');
}

// One persistent pair per cluster slot the device can hold at once
// (cudaOccupancyMaxActiveClusters, cached per device), so that no pair waits
// for a second wave.
inline int launch_pair(const CUtensorMap& tmO, const CUtensorMap& tmW, const Params& prm, cudaStream_t st) {
  int rc = set_max_dynamic_smem(reinterpret_cast<const void*>(outproj_gemm_pair_kernel), kPairSmemBytes,
                                "outproj pair smem attribute");
  if (rc) return rc;
  cudaLaunchConfig_t cfg{};
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = kPairSmemBytes;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  static std::mutex mu;
  static int slots[64] = {0};
  const int dev = current_device();
  if (dev < 0) return PU_ERR_CUDA;
  int n_slots = 0;
  {
    std::lock_guard<std::mutex> lock(mu);
    n_slots = dev < 64 ? slots[dev] : 0;
    if (n_slots <= 0) {
      cfg.gridDim = dim3(2 * (sm_count() / 2));
      rc = check_cuda(cudaOccupancyMaxActiveClusters(&n_slots, outproj_gemm_pair_kernel, &cfg),
                      "outproj pair occupancy");
      if (rc) return rc;
      if (n_slots <= 0) return set_error(PU_ERR_UNSUPPORTED, "no CTA pair of the out-projection fits an SM pair");
      if (dev < 64) slots[dev] = n_slots;
    }
  }
  cfg.gridDim = dim3(2 * std::min(prm.n_pair_tiles, n_slots));
  return check_cuda(cudaLaunchKernelEx(&cfg, outproj_gemm_pair_kernel, tmO, tmW, prm), "outproj pair GEMM launch");
}

}  // namespace outproj
}  // namespace pu

extern "C" {

size_t pu_outproj_exchange_bytes(int64_t T, int64_t N, int64_t G) {
  if (T <= 0 || N <= 0 || G <= 0 || T % pu::outproj::BM || N % pu::outproj::BN) return 0;
  return pu::outproj::layout(T, N, G).total;
}

int pu_outproj_allreduce(const void* o_local, const void* w_local, void* y, void* const* exchange, int64_t G,
                         int64_t rank, uint32_t epoch, int64_t T, int64_t K, int64_t N, uint64_t timeout_ns,
                         void* stream) {
  using namespace pu::outproj;
  if (!o_local || !w_local || !y || !exchange) return pu::set_error(PU_ERR_INVALID_ARGUMENT, "null pointer");
  if (T <= 0 || K <= 0 || N <= 0 || T % BM || N % BN || K % BK)
    return pu::set_error(PU_ERR_UNSUPPORTED, "T, K, N must be positive multiples of %d, %d, %d", BM, BK, BN);
  if (T > (1ll << 24) || K > (1ll << 20) || N > (1ll << 20))
    return pu::set_error(PU_ERR_UNSUPPORTED, "T, K or N too large");
  if (G < 1 || G > kMaxRanks) return pu::set_error(PU_ERR_UNSUPPORTED, "%lld ranks (1..%d)", (long long)G, kMaxRanks);
  if (rank < 0 || rank >= G) return pu::set_error(PU_ERR_INVALID_ARGUMENT, "rank %lld of %lld", (long long)rank, (long long)G);
  if (epoch == 0) return pu::set_error(PU_ERR_INVALID_ARGUMENT, "epochs start at 1");
  if (timeout_ns == 0 || timeout_ns > pu::kWaitTimeoutNs)
    return pu::set_error(PU_ERR_INVALID_ARGUMENT, "timeout must be in (0, 2 s]");
  if (!pu::aligned16(o_local) || !pu::aligned16(w_local) || !pu::aligned16(y))
    return pu::set_error(PU_ERR_INVALID_ARGUMENT, "o, w, y must be 16-byte aligned");
  const Layout l = layout(T, N, G);
  if ((long long)l.n_tiles > 0x7fffffffll) return pu::set_error(PU_ERR_UNSUPPORTED, "too many tiles");
  Params prm{};
  for (int g = 0; g < G; ++g) {
    if (!exchange[g] || !pu::aligned16(exchange[g]))
      return pu::set_error(PU_ERR_INVALID_ARGUMENT, "exchange buffer %d null or unaligned", g);
    prm.exch[g] = static_cast<unsigned char*>(exchange[g]);
  }
  prm.G = (int)G;
  prm.rank = (int)rank;
  prm.epoch = epoch;
  prm.n_k = (int)(K / BK);
  prm.n_ntiles = (int)(N / BN);
  prm.n_tiles = l.n_tiles;
  prm.n_owned = l.n_owned;
  prm.n_pair_tiles = (int)((T / kPairRows) * (N / BN));
  prm.off_part = l.off_part;
  prm.off_res = l.off_res;
  prm.off_pflag = l.off_pflag;
  prm.off_rflag = l.off_rflag;
  prm.timeout_ns = timeout_ns;
  prm.y = static_cast<__nv_bfloat16*>(y);
  prm.N = (int)N;
  CUtensorMap tmO, tmW;
  int rc = pu::make_tmap_bf16_3d(&tmO, o_local, (uint64_t)K, (uint64_t)T, 1, BK, BM, true);
  if (rc) return rc;
  rc = pu::make_tmap_bf16_3d(&tmW, w_local, (uint64_t)N, (uint64_t)K, 1, 64, BK, true);
  if (rc) return rc;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (T % kPairRows == 0 && pair_kernel_enabled()) {
    rc = launch_pair(tmO, tmW, prm, st);
  } else {
    rc = pu::set_max_dynamic_smem(reinterpret_cast<const void*>(outproj_gemm_kernel), kSmemBytes,
                                  "outproj smem attribute");
    if (rc) return rc;
    outproj_gemm_kernel<<<std::min(l.n_tiles, pu::sm_count()), kThreads, kSmemBytes, st>>>(tmO, tmW, prm);
    rc = pu::check_cuda(cudaGetLastError(), "outproj GEMM launch");
  }
  if (rc || G == 1) return rc;                        // one rank: the GEMM wrote y
  reduce_bcast_kernel<<<l.n_owned, 256, 0, st>>>(prm);
  rc = pu::check_cuda(cudaGetLastError(), "outproj reduce launch");
  if (rc) return rc;
  receive_kernel<<<std::min(l.n_tiles, 4 * pu::sm_count()), 256, 0, st>>>(prm);
  return pu::check_cuda(cudaGetLastError(), "outproj receive launch");
}

}  // extern "C"
