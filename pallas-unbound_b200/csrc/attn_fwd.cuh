// attn_fwd.cuh — training-attention forward on tcgen05 tensor cores.
//
// Reference: pallas_flash_attention (src/pallas_flash/ops/interface.py:20-85)
// launches flash_attention_kernel (kernels/attention.py:11-36) per
// (b, h, 1024-row query block); pipeline_kv_loop (kernels/pipeline.py:14-60)
// walks 128-row K/V blocks with an fp32 online softmax, P rounded to bf16
// (low_level/intrinsics.py:33-37) before the P.V product.
//
// B200 design: a persistent grid (one CTA per SM) walks work items of two
// 128-row query tiles (256 rows) of one (b, h); each item streams every K/V
// block once for both tiles.  Items are ordered longest first (causal: the
// last query blocks) with (b, h) fastest, and dealt to the CTAs in snake
// order (round r: CTA c takes item r*G + c, or r*G + G-1-c for odd r), which
// balances the causal work.  The rings, barriers and TMEM carry over from one
// item to the next, so item r+1's Q load and first QK^T products overlap
// item r's last products and epilogue.
//   warp 8      TMA producer: Q tiles once, then K_j / V_j through NS-deep
//               rings of 128-row tiles (128-byte swizzle).
//   warp 9      tcgen05 issuer (one thread) and TMEM owner.  Per K/V block j:
//                 O0 += P0_j V_j ; S0_{j+1} = Q0 K_{j+1}^T ;
//                 O1 += P1_j V_j ; S1_{j+1} = Q1 K_{j+1}^T
//               so the tensor core always has the other tile's work queued
//               while a softmax warpgroup is busy.  P.V reads P from tensor
//               memory (the `[d], [a], b_desc` form), V as an MN-major operand.
//   warps 0-3   softmax of tile 0, warps 4-7 softmax of tile 1: thread r owns
//               query row r (TMEM lane r).  Scores are scaled into log2
//               units; the running max only moves (O and l rescaled) when it
//               grows by more than kRescaleLog2, so P <= 2^8.  P is written
//               as bf16 over the first 64 columns of the tile's S columns.
//               Partial maxima in 8 independent accumulators and the row
//               sum in packed f32x2 pairs keep the reductions from
//               serialising on instruction latency.
// TMEM (512 columns): S0/P0 [0,128) S1/P1 [128,256) O0 [256,384) O1 [384,512).
// Ordering: the commit that signals S_t(j+1) also covers O_t += P_t(j) V_j
// (issued earlier by the same thread), so a softmax warpgroup that has seen
// S_t(j+1) may rescale O_t and overwrite P_t; S_t(j+1) itself is issued after
// P_t(j) V_j and the tensor pipe executes one thread's MMAs in issue order.
#pragma once

#include <cuda_bf16.h>

#include "pu_host.cuh"
#include "pu_ptx.cuh"

namespace pu {
namespace fwd {

constexpr int BM = 128;             // query rows per tile (two tiles per CTA)
constexpr int BN = 128;             // key/value rows per block
constexpr int kThreads = 320;       // 2 softmax warpgroups + producer + MMA
constexpr float kRescaleLog2 = 8.0f;
constexpr float kLn2 = 0.6931471805599453f;
constexpr float kLog2e = 1.4426950408889634f;
constexpr uint32_t kTmemCols = 512;
// TMEM column of tile t's S/P and O accumulators
__host__ __device__ constexpr uint32_t col_s(int t) { return 128u * t; }
__host__ __device__ constexpr uint32_t col_o(int t) { return 256u + 128u * t; }

template <int D>
struct Cfg {
  static constexpr int NS = (D == 128) ? 2 : 4;            // K/V ring depth
  static constexpr int kTileQ = BM * D * 2;                // bytes
  static constexpr int kTileKV = BN * D * 2;
  static constexpr int kColBlocks = D / 64;                // 128-byte swizzle column blocks
  static constexpr int kOffQ = 0;                          // two tiles
  static constexpr int kOffK = kOffQ + 2 * kTileQ;
  static constexpr int kOffV = kOffK + NS * kTileKV;
  static constexpr int kOffBar = kOffV + NS * kTileKV;
  // barriers: Q_full[2], K_full[NS], K_empty[NS], V_full[NS], V_empty[NS],
  //           S_full[2], P_full[2], O_final[2], Q_empty[2]; then tmem base +
  //           abort flag
  static constexpr int kNumBars = 2 + 4 * NS + 8;
  static constexpr int kSmemBytes = kOffBar + kNumBars * 8 + 16;
};

struct Params {
  int Nq, Nkv, H;
  int n_q_pairs;       // work items per (b, h): ceil(Nq / 256)
  int BH;
  int n_items;         // n_q_pairs * BH
  int causal;
  float scale_log2;
  __nv_bfloat16* o;
  float* lse;
};

template <int D>
__global__ void __launch_bounds__(kThreads, 1)
    attn_fwd_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                    const __grid_constant__ CUtensorMap tmV, const Params p) {
  using C = Cfg<D>;
  extern __shared__ __align__(1024) uint8_t smem[];
  const int tid = threadIdx.x;
  const int warp = tid >> 5;
  const int lane = tid & 31;
  if (smem_u32(smem) & 1023u) {  // the swizzled tiles need 1024-byte alignment
    if (tid == 0) record_device_error(PU_ERR_UNSUPPORTED, kSiteFwdQ);
    return;
  }
  uint8_t* sQ = smem + C::kOffQ;
  uint8_t* sK = smem + C::kOffK;
  uint8_t* sV = smem + C::kOffV;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + C::kOffBar);
  uint64_t* bQ = bars;              // [2]
  uint64_t* bKf = bars + 2;
  uint64_t* bKe = bKf + C::NS;
  uint64_t* bVf = bKe + C::NS;
  uint64_t* bVe = bVf + C::NS;
  uint64_t* bS = bVe + C::NS;       // [2]
  uint64_t* bP = bS + 2;            // [2]
  uint64_t* bOf = bP + 2;           // [2]
  uint64_t* bQe = bOf + 2;          // [2] Q tile t no longer read (last S_t done)
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bQe + 2);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  // Work item of round r for this CTA (snake order), or -1 when done; an
  // item is (b, h) = L % BH and query block n_q_pairs - 1 - L / BH.
  const int G = (int)gridDim.x;
  const int cta = (int)blockIdx.x;
  auto item_of = [&](int r) -> int {
    const long long L = (long long)r * G + ((r & 1) ? (G - 1 - cta) : cta);
    return L < p.n_items ? (int)L : -1;
  };
  const int n_kv_total = (p.Nkv + BN - 1) / BN;
  // K/V blocks each query tile of item L visits
  auto blocks_of = [&](int L, int (&n_t)[2]) {
    const int q0 = (p.n_q_pairs - 1 - L / p.BH) * (2 * BM);
#pragma unroll
    for (int t = 0; t < 2; ++t) {
      n_t[t] = n_kv_total;
      if (p.causal) n_t[t] = max(1, min(n_kv_total, (q0 + t * BM + BM + BN - 1) / BN));
    }
    return q0;
  };

  if (tid == 0) {
    for (int t = 0; t < 2; ++t) {
      mbar_init(bQ + t, 1);
      mbar_init(bS + t, 1);
      mbar_init(bP + t, 128);
      mbar_init(bOf + t, 1);
      mbar_init(bQe + t, 1);
    }
    for (int s = 0; s < C::NS; ++s) {
      mbar_init(bKf + s, 1);
      mbar_init(bKe + s, 1);
      mbar_init(bVf + s, 1);
      mbar_init(bVe + s, 1);
    }
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
      bool ok = true;
      int jg = 0;                                       // K/V blocks loaded so far
      for (int r = 0; ok; ++r) {
        const int L = item_of(r);
        if (L < 0) break;
        const int bh = L % p.BH;
        int n_t[2];
        const int q0 = blocks_of(L, n_t);
        const int n_max = max(n_t[0], n_t[1]);
        for (int t = 0; t < 2; ++t) {
          if (r > 0 && !mbar_wait(bQe + t, (r - 1) & 1, abort_flag, kSiteFwdQ)) { ok = false; break; }
          mbar_arrive_expect_tx(bQ + t, C::kTileQ);
          for (int cb = 0; cb < C::kColBlocks; ++cb)
            tma_load_3d(sQ + t * C::kTileQ + cb * BM * 128, &tmQ, bQ + t, cb * 64, q0 + t * BM, bh);
        }
        for (int j = 0; ok && j < n_max; ++j, ++jg) {
          const int st = jg % C::NS;
          const uint32_t u = jg / C::NS;
          if (u > 0 && !mbar_wait(bKe + st, (u - 1) & 1, abort_flag, kSiteFwdKEmpty)) { ok = false; break; }
          mbar_arrive_expect_tx(bKf + st, C::kTileKV);
          for (int cb = 0; cb < C::kColBlocks; ++cb)
            tma_load_3d(sK + st * C::kTileKV + cb * BN * 128, &tmK, bKf + st, cb * 64, j * BN, bh);
          if (u > 0 && !mbar_wait(bVe + st, (u - 1) & 1, abort_flag, kSiteFwdVEmpty)) { ok = false; break; }
          mbar_arrive_expect_tx(bVf + st, C::kTileKV);
          for (int cb = 0; cb < C::kColBlocks; ++cb)
            tma_load_3d(sV + st * C::kTileKV + cb * BN * 128, &tmV, bVf + st, cb * 64, j * BN, bh);
        }
      }
    }
  } else if (warp == 9) {
    // ---------------- tcgen05 issuer ----------------
    if (lane == 0) {
      constexpr uint32_t idS = make_idesc_bf16(BM, BN, 0, 0);
      constexpr uint32_t idO = make_idesc_bf16(BM, D, 0, 1);
      // descriptors are built once; per MMA only the start address moves
      const uint64_t dQ0 = make_sdesc_sw128(smem_u32(sQ), 16, 1024);
      const uint64_t dK0 = make_sdesc_sw128(smem_u32(sK), 16, 1024);
      const uint64_t dV0 = make_sdesc_sw128(smem_u32(sV), BN * 128, 1024);
      // S_t = Q_t K^T with K in ring slot `slot`
      auto issue_S = [&](int t, int slot) {
        const uint64_t dq = sdesc_add(dQ0, t * C::kTileQ);
        const uint64_t dk = sdesc_add(dK0, slot * C::kTileKV);
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
          const uint32_t off = (kk >> 2) * (BM * 128) + (kk & 3) * 32;
          const uint32_t offk = (kk >> 2) * (BN * 128) + (kk & 3) * 32;
          mma_ss(tmem + col_s(t), sdesc_add(dq, off), sdesc_add(dk, offk), idS, kk > 0);
        }
        mma_commit(bS + t);
      };
      // O_t (+)= P_t V with V in ring slot `slot`
      auto issue_PV = [&](int t, int slot, bool first) {
        const uint64_t dv = sdesc_add(dV0, slot * C::kTileKV);
#pragma unroll
        for (int kk = 0; kk < BN / 16; ++kk) {
          mma_ts(tmem + col_o(t), tmem + col_s(t) + kk * 8, sdesc_add(dv, kk * 16 * 128), idO,
                 (!first || kk > 0));
        }
      };
      bool ok = true;
      int jg = 0;                                       // K/V blocks consumed so far
      uint32_t jp[2] = {0, 0};                          // P_t blocks consumed so far
      for (int r = 0; ok; ++r) {
        const int L = item_of(r);
        if (L < 0) break;
        int n_t[2];
        blocks_of(L, n_t);
        const int n_max = max(n_t[0], n_t[1]);
        ok = mbar_wait(bKf + jg % C::NS, (jg / C::NS) & 1, abort_flag, kSiteFwdKFull);
        for (int t = 0; ok && t < 2; ++t) {
          ok = mbar_wait(bQ + t, r & 1, abort_flag, kSiteFwdQ);
          if (!ok) break;
          tc_fence_after();
          issue_S(t, jg % C::NS);
          if (n_t[t] == 1) mma_commit(bQe + t);         // Q_t's last reader
        }
        if (ok) mma_commit(bKe + jg % C::NS);
        for (int j = 0; ok && j < n_max; ++j) {
          const int st = (jg + j) % C::NS;
          const int nst = (jg + j + 1) % C::NS;
          if (!mbar_wait(bVf + st, ((jg + j) / C::NS) & 1, abort_flag, kSiteFwdVFull)) { ok = false; break; }
          const bool next_k = (j + 1 < n_max);
          bool k_ready = false;
          for (int t = 0; t < 2; ++t) {
            if (j >= n_t[t]) continue;
            if (!mbar_wait(bP + t, jp[t] & 1, abort_flag, kSiteFwdPFull)) { ok = false; break; }
            ++jp[t];
            tc_fence_after();
            issue_PV(t, st, j == 0);
            if (j + 1 < n_t[t]) {
              if (!k_ready) {
                if (!mbar_wait(bKf + nst, ((jg + j + 1) / C::NS) & 1, abort_flag, kSiteFwdKFull)) { ok = false; break; }
                tc_fence_after();
                k_ready = true;
              }
              issue_S(t, nst);
              if (j + 2 == n_t[t]) mma_commit(bQe + t);  // Q_t's last reader
            } else {
              mma_commit(bOf + t);
            }
          }
          if (!ok) break;
          mma_commit(bVe + st);
          if (next_k) mma_commit(bKe + nst);
        }
        jg += n_max;
      }
    }
  } else {
    // ---------------- softmax warpgroups (warps 0-3: tile 0, 4-7: tile 1) ----------------
    const int t = warp >> 2;
    const int row = tid & 127;                 // TMEM lane == query row in tile
    const uint32_t lane_base = static_cast<uint32_t>((warp & 3) * 32) << 16;
    const uint32_t tS = tmem + lane_base + col_s(t);
    const uint32_t tO = tmem + lane_base + col_o(t);
    bool ok = true;
    uint32_t js = 0;                           // S_t blocks consumed so far
    for (int r = 0; ok; ++r) {
    const int L = item_of(r);
    if (L < 0) break;
    const int bh = L % p.BH;
    int n_t[2];
    const int q0 = blocks_of(L, n_t);
    const int q_tile0 = q0 + t * BM;
    const int q_idx = q_tile0 + row;
    const int n_blocks = n_t[t];
    float m_ref = -INFINITY;                   // log2 domain
    float l = 0.f;
    for (int j = 0; j < n_blocks; ++j, ++js) {
      ok = mbar_wait(bS + t, js & 1, abort_flag, kSiteFwdSFull);
      ok = __all_sync(0xffffffffu, ok);
      if (!ok) break;
      tc_fence_after();
      uint32_t s[BN];
      {
        uint32_t (&s0)[32] = *reinterpret_cast<uint32_t(*)[32]>(s);
        uint32_t (&s1)[32] = *reinterpret_cast<uint32_t(*)[32]>(s + 32);
        uint32_t (&s2)[32] = *reinterpret_cast<uint32_t(*)[32]>(s + 64);
        uint32_t (&s3)[32] = *reinterpret_cast<uint32_t(*)[32]>(s + 96);
        tmem_ld32(tS, s0);
        tmem_ld32(tS + 32, s1);
        tmem_ld32(tS + 64, s2);
        tmem_ld32(tS + 96, s3);
        tmem_wait_ld();
        reg_fence(s);
      }
      const int kv0 = j * BN;
      if ((p.causal && kv0 + BN - 1 > q_tile0) || kv0 + BN > p.Nkv) {
        const int lim = p.causal ? min(q_idx + 1, p.Nkv) : p.Nkv;   // keys < lim are visible
#pragma unroll
        for (int c = 0; c < BN; ++c)
          if (kv0 + c >= lim) s[c] = __float_as_uint(-INFINITY);
      }
      float mx8[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) mx8[i] = __uint_as_float(s[i]);
#pragma unroll
      for (int c = 8; c < BN; ++c) mx8[c & 7] = fmaxf(mx8[c & 7], __uint_as_float(s[c]));
      const float mx = fmaxf(fmaxf(fmaxf(mx8[0], mx8[1]), fmaxf(mx8[2], mx8[3])),
                             fmaxf(fmaxf(mx8[4], mx8[5]), fmaxf(mx8[6], mx8[7])));
      const float m_blk = mx * p.scale_log2;
      float alpha = 1.f;
      if (j == 0) {
        m_ref = m_blk;
      } else if (m_blk > m_ref + kRescaleLog2) {
        alpha = ex2(m_ref - m_blk);
        m_ref = m_blk;
      }
      // O_t is quiescent: the commit behind S_t(j) covered O_t += P_t(j-1) V_{j-1}
      if (j > 0 && __any_sync(0xffffffffu, alpha != 1.f)) {
#pragma unroll 1
        for (int c = 0; c < D / 32; ++c) {
          uint32_t ov[32];
          tmem_ld32(tO + c * 32, ov);
          tmem_wait_ld();
          reg_fence(ov);
#pragma unroll
          for (int i = 0; i < 32; ++i) ov[i] = __float_as_uint(__uint_as_float(ov[i]) * alpha);
          tmem_st32(tO + c * 32, ov);
        }
      }
      // P = 2^(s*scale - m): scale-subtract and row sum on pairs of scores in
      // packed f32x2 arithmetic (half the instructions), exp2 on MUFU
      const uint64_t scale2 = f2_pack(p.scale_log2, p.scale_log2);
      const uint64_t negm2 = f2_pack(-m_ref, -m_ref);
      uint64_t rs2[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) rs2[i] = 0ull;
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        uint32_t pk[32];
#pragma unroll
        for (int i = 0; i < 32; ++i) {
          const int c = h * 64 + 2 * i;
          float x0, x1;
          f2_unpack(f2_fma(f2_pack(__uint_as_float(s[c]), __uint_as_float(s[c + 1])), scale2, negm2), x0, x1);
          const float p0 = ex2(x0);
          const float p1 = ex2(x1);
          rs2[i & 3] = f2_add(rs2[i & 3], f2_pack(p0, p1));
          pk[i] = pack_bf16x2(p0, p1);
        }
        tmem_st32(tS + h * 32, pk);
      }
      float ra, rb, rc, rd;
      f2_unpack(f2_add(rs2[0], rs2[1]), ra, rb);
      f2_unpack(f2_add(rs2[2], rs2[3]), rc, rd);
      const float rs = (ra + rb) + (rc + rd);
      l = l * alpha + rs;
      tmem_wait_st();
      tc_fence_before();
      mbar_arrive(bP + t);
    }
    if (ok) {
      ok = mbar_wait(bOf + t, r & 1, abort_flag, kSiteFwdODone);
      ok = __all_sync(0xffffffffu, ok);
    }
    if (ok) {
      tc_fence_after();
      const float inv_l = (l > 0.f) ? 1.f / l : 0.f;
      __nv_bfloat16* orow = p.o + ((size_t)bh * p.Nq + q_idx) * D;
#pragma unroll 1
      for (int c = 0; c < D / 32; ++c) {
        uint32_t ov[32];
        tmem_ld32(tO + c * 32, ov);
        tmem_wait_ld();
        reg_fence(ov);
        if (q_idx < p.Nq) {
          uint32_t w[16];
#pragma unroll
          for (int i = 0; i < 16; ++i)
            w[i] = pack_bf16x2(__uint_as_float(ov[2 * i]) * inv_l, __uint_as_float(ov[2 * i + 1]) * inv_l);
          uint4* dst = reinterpret_cast<uint4*>(orow + c * 32);
#pragma unroll
          for (int i = 0; i < 4; ++i) dst[i] = make_uint4(w[4 * i], w[4 * i + 1], w[4 * i + 2], w[4 * i + 3]);
        }
      }
      if (p.lse != nullptr && q_idx < p.Nq) {
        p.lse[(size_t)bh * p.Nq + q_idx] = (m_ref + lg2(l)) * kLn2;
      }
    }
    }  // items
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 9) {
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
}

inline int check_common(const void* q, const void* k, const void* v, long long B, long long H,
                        long long Nq, long long Nkv, long long D, float sm_scale) {
  if (!q || !k || !v) return set_error(PU_ERR_INVALID_ARGUMENT, "null q/k/v pointer");
  if (B <= 0 || H <= 0 || Nq <= 0 || Nkv <= 0)
    return set_error(PU_ERR_INVALID_ARGUMENT, "B, H, Nq, Nkv must be positive");
  if (D != 128 && D != 64)
    return set_error(PU_ERR_UNSUPPORTED, "head size %lld (supported: 64, 128; pad others)", D);
  if (!(sm_scale > 0.f)) return set_error(PU_ERR_INVALID_ARGUMENT, "sm_scale must be > 0");
  if (B * H > 65535) return set_error(PU_ERR_UNSUPPORTED, "B*H = %lld exceeds 65535", B * H);
  if (Nq > (1ll << 24) || Nkv > (1ll << 24))
    return set_error(PU_ERR_UNSUPPORTED, "sequence length above 2^24");
  if (((std::max(Nq, Nkv) + 127) / 128) * B * H > 0x7fffffffll)
    return set_error(PU_ERR_UNSUPPORTED, "B*H*ceil(N/128) above 2^31 - 1");
  return PU_OK;
}

template <int D>
int launch_fwd(const void* q, const void* k, const void* v, void* o, float* lse, long long B,
               long long H, long long Nq, long long Nkv, float sm_scale, int causal, cudaStream_t st) {
  using C = Cfg<D>;
  CUtensorMap tq, tk, tv;
  int rc = make_tmap_bf16_3d(&tq, q, D, Nq, B * H, 64, BM, true);
  if (!rc) rc = make_tmap_bf16_3d(&tk, k, D, Nkv, B * H, 64, BN, true);
  if (!rc) rc = make_tmap_bf16_3d(&tv, v, D, Nkv, B * H, 64, BN, true);
  if (rc) return rc;
  rc = set_max_dynamic_smem(reinterpret_cast<const void*>(attn_fwd_kernel<D>), C::kSmemBytes,
                            "cudaFuncSetAttribute(fwd smem)");
  if (rc) return rc;
  Params prm{};
  prm.Nq = (int)Nq;
  prm.Nkv = (int)Nkv;
  prm.H = (int)H;
  prm.n_q_pairs = (int)((Nq + 2 * BM - 1) / (2 * BM));
  prm.causal = causal ? 1 : 0;
  prm.scale_log2 = sm_scale * kLog2e;
  prm.o = static_cast<__nv_bfloat16*>(o);
  prm.lse = lse;
  prm.BH = (int)(B * H);
  prm.n_items = (int)((long long)prm.n_q_pairs * B * H);
  dim3 grid((unsigned)std::min<long long>(prm.n_items, sm_count()));
  attn_fwd_kernel<D><<<grid, kThreads, C::kSmemBytes, st>>>(tq, tk, tv, prm);
  return check_cuda(cudaGetLastError(), "attention forward launch");
}

}  // namespace fwd
}  // namespace pu

extern "C" int pu_attn_fwd(const void* q, const void* k, const void* v, void* o, float* lse,
                           int64_t B, int64_t H, int64_t Nq, int64_t Nkv, int64_t D, float sm_scale,
                           int causal, void* stream) {
  using namespace pu::fwd;
  int rc = check_common(q, k, v, B, H, Nq, Nkv, D, sm_scale);
  if (rc) return rc;
  if (!o) return pu::set_error(PU_ERR_INVALID_ARGUMENT, "null output pointer");
  if (!pu::aligned16(o) || (lse && (reinterpret_cast<uintptr_t>(lse) & 3)))
    return pu::set_error(PU_ERR_INVALID_ARGUMENT, "o must be 16-byte aligned, lse 4-byte aligned");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (D == 128) return launch_fwd<128>(q, k, v, o, lse, B, H, Nq, Nkv, sm_scale, causal, st);
  return launch_fwd<64>(q, k, v, o, lse, B, H, Nq, Nkv, sm_scale, causal, st);
}
