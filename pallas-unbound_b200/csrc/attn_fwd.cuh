// attn_fwd.cuh — training-attention forward on tcgen05 tensor cores.
//
// Reference: pallas_flash_attention (src/pallas_flash/ops/interface.py:20-85)
// launches flash_attention_kernel (kernels/attention.py:11-36) per
// (b, h, 1024-row query block); pipeline_kv_loop (kernels/pipeline.py:14-60)
// walks 128-row K/V blocks with an fp32 online softmax, P rounded to bf16
// (low_level/intrinsics.py:33-37) before the P.V product.
//
// B200 design (one CTA per 128-row query tile of one (b, h)):
//   warp 4      TMA producer: Q tile once, then K_j / V_j through an
//               NS-deep ring of 128-row tiles (128-byte swizzle).
//   warp 5      tcgen05 issuer (one thread) and TMEM owner:
//                 S_j  = Q . K_j^T     (A, B from shared memory, K-major)
//                 O   += P_j . V_j     (A = P from tensor memory, B = V
//                                       MN-major from shared memory)
//               S is double-buffered in TMEM so S_{j+1} runs on the tensor
//               core while the softmax warps work on S_j.
//   warps 0-3   softmax: thread r owns query row r (TMEM lane r), so row max
//               and row sum need no shuffles.  Scores are scaled into log2
//               units; the running max is only moved (and O, l rescaled)
//               when it grows by more than kRescaleLog2, which keeps P <= 2^8.
//               P goes to TMEM as bf16; the epilogue divides O by l, writes
//               bf16 O and the fp32 natural-log LSE.
// TMEM (512 columns): S0 [0,128) S1 [128,256) O [256,256+D) P [384,448).
#pragma once

#include <cuda_bf16.h>

#include "pu_host.cuh"
#include "pu_ptx.cuh"

namespace pu {
namespace fwd {

constexpr int BM = 128;             // query rows per CTA tile
constexpr int BN = 128;             // key/value rows per block
constexpr int kThreads = 192;       // 4 softmax warps + producer + MMA
constexpr float kRescaleLog2 = 8.0f;
constexpr float kLn2 = 0.6931471805599453f;
constexpr float kLog2e = 1.4426950408889634f;
constexpr uint32_t kTmemCols = 512;
constexpr uint32_t kColS0 = 0, kColS1 = 128, kColO = 256, kColP = 384;

template <int D>
struct Cfg {
  static constexpr int NS = (D == 128) ? 2 : 4;            // K/V ring depth
  static constexpr int kTileQ = BM * D * 2;                // bytes
  static constexpr int kTileKV = BN * D * 2;
  static constexpr int kColBlocks = D / 64;                // 128-byte swizzle column blocks
  static constexpr int kOffQ = 0;
  static constexpr int kOffK = kOffQ + kTileQ;
  static constexpr int kOffV = kOffK + NS * kTileKV;
  static constexpr int kOffBar = kOffV + NS * kTileKV;
  // barriers: Q_full, K_full[NS], K_empty[NS], V_full[NS], V_empty[NS],
  //           S_full[2], P_full, O_done; then tmem base + abort flag
  static constexpr int kNumBars = 1 + 4 * NS + 2 + 2;
  static constexpr int kSmemBytes = kOffBar + kNumBars * 8 + 16 + 1024;  // + alignment slack
};

struct Params {
  int Nq, Nkv, H;
  int n_q_tiles;
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
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sQ = smem + C::kOffQ;
  uint8_t* sK = smem + C::kOffK;
  uint8_t* sV = smem + C::kOffV;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + C::kOffBar);
  uint64_t* bQ = bars;
  uint64_t* bKf = bars + 1;
  uint64_t* bKe = bKf + C::NS;
  uint64_t* bVf = bKe + C::NS;
  uint64_t* bVe = bVf + C::NS;
  uint64_t* bS = bVe + C::NS;   // [2]
  uint64_t* bP = bS + 2;
  uint64_t* bO = bP + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bO + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int tid = threadIdx.x;
  const int warp = tid >> 5;
  const int lane = tid & 31;
  const int bh = blockIdx.x;
  // heaviest (causal: last) query tiles first
  const int q_tile = p.n_q_tiles - 1 - blockIdx.y;
  const int q0 = q_tile * BM;
  const int n_kv_blocks_total = (p.Nkv + BN - 1) / BN;
  int n_blocks = n_kv_blocks_total;
  if (p.causal) n_blocks = min(n_blocks, (q0 + BM + BN - 1) / BN);

  if (tid == 128) {
    mbar_init(bQ, 1);
    for (int s = 0; s < C::NS; ++s) {
      mbar_init(bKf + s, 1);
      mbar_init(bKe + s, 1);
      mbar_init(bVf + s, 1);
      mbar_init(bVe + s, 1);
    }
    mbar_init(bS, 1);
    mbar_init(bS + 1, 1);
    mbar_init(bP, 128);
    mbar_init(bO, 1);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 5) {
    tmem_alloc(tmem_slot, kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 4) {
    // ---------------- TMA producer ----------------
    if (lane == 0) {
      tma_prefetch_desc(&tmQ);
      tma_prefetch_desc(&tmK);
      tma_prefetch_desc(&tmV);
      mbar_arrive_expect_tx(bQ, C::kTileQ);
      for (int cb = 0; cb < C::kColBlocks; ++cb)
        tma_load_3d(sQ + cb * BM * 128, &tmQ, bQ, cb * 64, q0, bh);
      for (int j = 0; j < n_blocks; ++j) {
        const int st = j % C::NS;
        const uint32_t u = j / C::NS;
        if (u > 0 && !mbar_wait(bKe + st, (u - 1) & 1, abort_flag, kSiteFwdKEmpty)) break;
        mbar_arrive_expect_tx(bKf + st, C::kTileKV);
        for (int cb = 0; cb < C::kColBlocks; ++cb)
          tma_load_3d(sK + st * C::kTileKV + cb * BN * 128, &tmK, bKf + st, cb * 64, j * BN, bh);
        if (u > 0 && !mbar_wait(bVe + st, (u - 1) & 1, abort_flag, kSiteFwdVEmpty)) break;
        mbar_arrive_expect_tx(bVf + st, C::kTileKV);
        for (int cb = 0; cb < C::kColBlocks; ++cb)
          tma_load_3d(sV + st * C::kTileKV + cb * BN * 128, &tmV, bVf + st, cb * 64, j * BN, bh);
      }
    }
  } else if (warp == 5) {
    // ---------------- tcgen05 issuer ----------------
    if (lane == 0) {
      constexpr uint32_t idS = make_idesc_bf16(BM, BN, 0, 0);
      constexpr uint32_t idO = make_idesc_bf16(BM, D, 0, 1);
      const uint32_t aQ = smem_u32(sQ);
      bool ok = mbar_wait(bQ, 0, abort_flag, kSiteFwdQ);
      auto issue_S = [&](int j) -> bool {
        const int st = j % C::NS;
        if (!mbar_wait(bKf + st, (j / C::NS) & 1, abort_flag, kSiteFwdKFull)) return false;
        tc_fence_after();
        const uint32_t aK = smem_u32(sK + st * C::kTileKV);
        const uint32_t dS = tmem + ((j & 1) ? kColS1 : kColS0);
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
          const uint32_t off = (kk >> 2) * (BM * 128) + (kk & 3) * 32;
          const uint32_t offk = (kk >> 2) * (BN * 128) + (kk & 3) * 32;
          mma_ss(dS, make_sdesc_sw128(aQ + off, 16, 1024), make_sdesc_sw128(aK + offk, 16, 1024), idS,
                 kk > 0);
        }
        mma_commit(bS + (j & 1));
        mma_commit(bKe + st);
        return true;
      };
      if (ok) ok = issue_S(0);
      for (int j = 0; ok && j < n_blocks; ++j) {
        if (j + 1 < n_blocks && !issue_S(j + 1)) break;
        if (!mbar_wait(bP, j & 1, abort_flag, kSiteFwdPFull)) break;
        const int st = j % C::NS;
        if (!mbar_wait(bVf + st, (j / C::NS) & 1, abort_flag, kSiteFwdVFull)) break;
        tc_fence_after();
        const uint32_t aV = smem_u32(sV + st * C::kTileKV);
#pragma unroll
        for (int kk = 0; kk < BN / 16; ++kk) {
          mma_ts(tmem + kColO, tmem + kColP + kk * 8, make_sdesc_sw128(aV + kk * 16 * 128, BN * 128, 1024),
                 idO, (j > 0 || kk > 0));
        }
        mma_commit(bO);
        mma_commit(bVe + st);
      }
    }
  } else {
    // ---------------- softmax warps 0-3 ----------------
    const int row = tid;                       // TMEM lane == query row in tile
    const int q_idx = q0 + row;
    const uint32_t lane_base = static_cast<uint32_t>(warp * 32) << 16;
    float m_ref = -INFINITY;                   // log2 domain
    float l = 0.f;
    bool ok = true;
    for (int j = 0; j < n_blocks; ++j) {
      ok = mbar_wait(bS + (j & 1), (j >> 1) & 1, abort_flag, kSiteFwdSFull);
      ok = __all_sync(0xffffffffu, ok);
      if (!ok) break;
      tc_fence_after();
      const uint32_t tS = tmem + lane_base + ((j & 1) ? kColS1 : kColS0);
      float s[BN];
      {
        uint32_t r[32];
#pragma unroll
        for (int c = 0; c < BN / 32; ++c) {
          tmem_ld32(tS + c * 32, r);
          tmem_wait_ld();
#pragma unroll
          for (int i = 0; i < 32; ++i) s[c * 32 + i] = __uint_as_float(r[i]);
        }
      }
      const int kv0 = j * BN;
      if (p.causal && kv0 + BN - 1 > q0) {
#pragma unroll
        for (int c = 0; c < BN; ++c)
          if (kv0 + c > q_idx) s[c] = -INFINITY;
      }
      if (kv0 + BN > p.Nkv) {
#pragma unroll
        for (int c = 0; c < BN; ++c)
          if (kv0 + c >= p.Nkv) s[c] = -INFINITY;
      }
      float mx = s[0];
#pragma unroll
      for (int c = 1; c < BN; ++c) mx = fmaxf(mx, s[c]);
      const float m_blk = mx * p.scale_log2;
      float alpha = 1.f;
      if (j == 0) {
        m_ref = m_blk;
      } else if (m_blk > m_ref + kRescaleLog2) {
        alpha = ex2(m_ref - m_blk);
        m_ref = m_blk;
      }
      const float neg_m = -m_ref;
      float rs = 0.f;
      uint32_t pk[BN / 2];
#pragma unroll
      for (int c = 0; c < BN; c += 2) {
        const float p0 = ex2(fmaf(s[c], p.scale_log2, neg_m));
        const float p1 = ex2(fmaf(s[c + 1], p.scale_log2, neg_m));
        rs += p0 + p1;
        pk[c / 2] = pack_bf16x2(p0, p1);
      }
      // P_{j-1}.V_{j-1} must be done before O is rescaled or P overwritten
      if (j > 0) {
        ok = mbar_wait(bO, (j - 1) & 1, abort_flag, kSiteFwdODone);
        ok = __all_sync(0xffffffffu, ok);
        if (!ok) break;
        tc_fence_after();
        if (__any_sync(0xffffffffu, alpha != 1.f)) {
          uint32_t r[32];
#pragma unroll
          for (int c = 0; c < D / 32; ++c) {
            const uint32_t tO = tmem + lane_base + kColO + c * 32;
            tmem_ld32(tO, r);
            tmem_wait_ld();
#pragma unroll
            for (int i = 0; i < 32; ++i) r[i] = __float_as_uint(__uint_as_float(r[i]) * alpha);
            tmem_st32(tO, r);
          }
        }
      }
      l = l * alpha + rs;
      {
        uint32_t r[32];
#pragma unroll
        for (int c = 0; c < BN / 64; ++c) {
#pragma unroll
          for (int i = 0; i < 32; ++i) r[i] = pk[c * 32 + i];
          tmem_st32(tmem + lane_base + kColP + c * 32, r);
        }
      }
      tmem_wait_st();
      tc_fence_before();
      mbar_arrive(bP);
    }
    if (ok && n_blocks > 0) {
      ok = mbar_wait(bO, (n_blocks - 1) & 1, abort_flag, kSiteFwdODone);
      ok = __all_sync(0xffffffffu, ok);
    }
    if (ok) {
      tc_fence_after();
      const float inv_l = (l > 0.f) ? 1.f / l : 0.f;
      __nv_bfloat16* orow = p.o + ((size_t)bh * p.Nq + q_idx) * D;
      uint32_t r[32];
#pragma unroll
      for (int c = 0; c < D / 32; ++c) {
        tmem_ld32(tmem + lane_base + kColO + c * 32, r);
        tmem_wait_ld();
        if (q_idx < p.Nq) {
          uint32_t w[16];
#pragma unroll
          for (int i = 0; i < 16; ++i)
            w[i] = pack_bf16x2(__uint_as_float(r[2 * i]) * inv_l, __uint_as_float(r[2 * i + 1]) * inv_l);
          uint4* dst = reinterpret_cast<uint4*>(orow + c * 32);
#pragma unroll
          for (int i = 0; i < 4; ++i) dst[i] = make_uint4(w[4 * i], w[4 * i + 1], w[4 * i + 2], w[4 * i + 3]);
        }
      }
      if (p.lse != nullptr && q_idx < p.Nq) {
        p.lse[(size_t)bh * p.Nq + q_idx] = (m_ref + lg2(l)) * kLn2;
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 5) {
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
  if (B * H > 0x7fffffffll) return set_error(PU_ERR_UNSUPPORTED, "B*H too large");
  if (Nq > (1ll << 24) || Nkv > (1ll << 24))
    return set_error(PU_ERR_UNSUPPORTED, "sequence length above 2^24");
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
  static bool attr_done[64] = {false};
  const int dev = current_device();
  if (dev < 0) return PU_ERR_CUDA;
  if (dev >= 64 || !attr_done[dev]) {
    rc = check_cuda(cudaFuncSetAttribute(attn_fwd_kernel<D>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         C::kSmemBytes),
                    "cudaFuncSetAttribute(fwd smem)");
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
  prm.o = static_cast<__nv_bfloat16*>(o);
  prm.lse = lse;
  if (prm.n_q_tiles > 65535) return set_error(PU_ERR_UNSUPPORTED, "too many query tiles");
  dim3 grid((unsigned)(B * H), (unsigned)prm.n_q_tiles);
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
