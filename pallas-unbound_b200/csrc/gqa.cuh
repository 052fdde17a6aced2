// gqa.cuh — split-KV decode with grouped K/V heads: one CTA per (split, b,
// K/V head) computes all G query heads of the group from one read of each
// K/V row, so the cache is streamed from DRAM exactly once (the query-head
// kernel would read every K/V row once per query head, the repeats coming
// from L2 at best).
//
// No counterpart in the reference (one K/V head per query head, bf16 cache;
// src/pallas_flash/kernels/decoding.py:105-115).  Same split / record / merge
// scheme as split_kv_kernel: D/8 lanes per cache row, 128-bit (fp8: 64-bit)
// streaming loads; per lane the G query slices and output accumulators of its
// 8 columns live in registers.  Per iteration the scores of all its rows and
// heads are computed first (independent chains), then a lazy running maximum
// per head (it moves, with a rescale of o and l, only when the iteration's
// maximum exceeds it by more than 8 in log2 units, so every p <= 2^8) and the
// P.V updates.  Split records and the last-CTA merge are per query head.
#pragma once

#include "decode.cuh"

namespace pu {
namespace decode {

constexpr float kGqaRescaleLog2 = 8.f;

// rows in flight per lane group (registers: q and o take 16 G per lane, the
// scores G * kUnroll)
template <int G, typename KVT>
struct GqaShape {
  static constexpr int kUnroll = G >= 8 ? 4 : (sizeof(KVT) == 1 && G <= 2 ? 16 : 8);
};

template <typename QT, typename KVT, int D, int G>
__global__ void __launch_bounds__(kThreads, 1) gqa_kernel(const Params p) {
  using IO = KVIO<KVT>;
  constexpr int kU = GqaShape<G, KVT>::kUnroll;
  constexpr int LPR = D / 8;
  constexpr int RPW = 32 / LPR;
  constexpr int TW = RPW * kU;
  constexpr int ROWS_PER_ITER = kWarps * TW;
  constexpr int NGROUP = kWarps * RPW;
  static_assert(D == 64 || D == 128, "head size");

  __shared__ float sm_m[NGROUP];
  __shared__ float sm_l[NGROUP];
  __shared__ float sm_o[NGROUP][D];
  __shared__ int sm_last;

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int sub = lane % LPR, rw = lane / LPR;
  const int split = blockIdx.x;
  const int bkv = blockIdx.y;                           // b * H_kv + K/V head
  const int H_kv = p.H / G;
  const int b = bkv / H_kv;
  const int bh0 = b * p.H + (bkv % H_kv) * G;           // first query head of the group

  int len = p.n_local;
  if (p.lens != nullptr) {
    const long long g = (long long)p.lens[b];
    len = g < 0 ? 0 : (g > p.n_local ? p.n_local : (int)g);
  }
  const int t_begin = split * p.chunk;
  const int t_end = min(t_begin + p.chunk, len);

  float q[G][8];
#pragma unroll
  for (int g = 0; g < G; ++g) {
    const uint4 w = *reinterpret_cast<const uint4*>(static_cast<const QT*>(p.q) + (size_t)(bh0 + g) * D + sub * 8);
    unpack8<QT>(w, q[g]);
#pragma unroll
    for (int i = 0; i < 8; ++i) q[g][i] *= p.scale_log2;
  }
  const KVT* kb = static_cast<const KVT*>(p.k) + (size_t)bkv * p.n_local * D + sub * 8;
  const KVT* vb = static_cast<const KVT*>(p.v) + (size_t)bkv * p.n_local * D + sub * 8;

  float m[G], l[G], o[G][8];
#pragma unroll
  for (int g = 0; g < G; ++g) {
    m[g] = -INFINITY;
    l[g] = 0.f;
#pragma unroll
    for (int i = 0; i < 8; ++i) o[g][i] = 0.f;
  }

  for (int base = t_begin + warp * TW; base < t_end; base += ROWS_PER_ITER) {
    typename IO::W kw[kU], vw[kU];
    bool ok[kU];
#pragma unroll
    for (int u = 0; u < kU; ++u) {
      const int t = base + u * RPW + rw;
      ok[u] = t < t_end;
      kw[u] = IO::ld(kb + (size_t)t * D, ok[u]);
      vw[u] = IO::ld(vb + (size_t)t * D, ok[u]);
    }
    // scores of every row and head of the iteration (independent chains)
    float s[G][kU];
#pragma unroll
    for (int u = 0; u < kU; ++u) {
      float kf[8];
      IO::unpack(kw[u], kf);
#pragma unroll
      for (int g = 0; g < G; ++g) {
        uint64_t acc = f2_pack(0.f, 0.f);
#pragma unroll
        for (int i = 0; i < 8; i += 2)
          acc = f2_fma(f2_pack(q[g][i], q[g][i + 1]), f2_pack(kf[i], kf[i + 1]), acc);
        float a0, a1;
        f2_unpack(acc, a0, a1);
        s[g][u] = a0 + a1;
      }
    }
#pragma unroll
    for (int off = LPR / 2; off > 0; off >>= 1)
#pragma unroll
      for (int g = 0; g < G; ++g)
#pragma unroll
        for (int u = 0; u < kU; ++u) s[g][u] += __shfl_xor_sync(0xffffffffu, s[g][u], off);
    // per head: the maximum of the iteration's rows moves the running maximum
    // (with a rescale of o and l) only when it exceeds it by more than 8
#pragma unroll
    for (int g = 0; g < G; ++g) {
      float mx = -INFINITY;
#pragma unroll
      for (int u = 0; u < kU; ++u) {
        if (!ok[u]) s[g][u] = -INFINITY;
        mx = fmaxf(mx, s[g][u]);
      }
      if (mx > m[g] + kGqaRescaleLog2) {                 // same in all lanes of the row group
        const float alpha = ex2(m[g] - mx);              // 0 while m = -inf
        l[g] *= alpha;
#pragma unroll
        for (int i = 0; i < 8; ++i) o[g][i] *= alpha;
        m[g] = mx;
      }
    }
#pragma unroll
    for (int u = 0; u < kU; ++u) {
      float vf[8];
      IO::unpack(vw[u], vf);
#pragma unroll
      for (int g = 0; g < G; ++g) {
        // 0 for masked rows (s = -inf); nothing seen yet (m = -inf) adds nothing
        const float pr = (m[g] == -INFINITY) ? 0.f : ex2(s[g][u] - m[g]);
        l[g] += pr;
        const uint64_t p2 = f2_pack(pr, pr);
#pragma unroll
        for (int i = 0; i < 8; i += 2) {
          float o0, o1;
          f2_unpack(f2_fma(p2, f2_pack(vf[i], vf[i + 1]), f2_pack(o[g][i], o[g][i + 1])), o0, o1);
          o[g][i] = o0;
          o[g][i + 1] = o1;
        }
      }
    }
  }

  // per query head: merge the lane groups of this CTA into its split record
  const int grp = warp * RPW + rw;
#pragma unroll
  for (int g = 0; g < G; ++g) {
    if (sub == 0) {
      sm_m[grp] = m[g];
      sm_l[grp] = l[g];
    }
#pragma unroll
    for (int i = 0; i < 8; ++i) sm_o[grp][sub * 8 + i] = o[g][i];
    __syncthreads();
    float* rec = p.ws_rec + ((size_t)(bh0 + g) * p.splits + split) * (D + 2);
    if (tid < D) {
      float M = -INFINITY;
#pragma unroll
      for (int x = 0; x < NGROUP; ++x) M = fmaxf(M, sm_m[x]);
      float L = 0.f, O = 0.f;
      if (M != -INFINITY) {
#pragma unroll
        for (int x = 0; x < NGROUP; ++x) {
          const float w = (sm_m[x] == -INFINITY) ? 0.f : ex2(sm_m[x] - M);
          L += w * sm_l[x];
          O += w * sm_o[x][tid];
        }
      }
      rec[2 + tid] = O * p.o_scale;
      if (tid == 0) {
        rec[0] = M;
        rec[1] = L;
      }
    }
    __syncthreads();
  }
  __threadfence();
  __syncthreads();
  if (tid == 0) {
    const int prev = atomicAdd(p.ws_count + bkv, 1);
    sm_last = (prev == p.splits - 1);
  }
  __syncthreads();
  if (!sm_last) return;
  __threadfence();
  // last CTA of this (b, K/V head): merge every split record of each query head
  for (int g = 0; g < G; ++g) {
    const int bh = bh0 + g;
    float M, L, O;
    block_merge<D>(p.ws_rec + (size_t)bh * p.splits * (D + 2), p.splits, M, L, O);
    if (tid < D) {
      p.o[(size_t)bh * D + tid] = __float2bfloat16_rn(L > 0.f ? O / L : 0.f);
      if (tid == 0 && p.lse != nullptr) p.lse[bh] = (L > 0.f) ? (M + lg2(L)) * kLn2 : -INFINITY;
    }
    __syncthreads();
  }
  if (tid == 0) p.ws_count[bkv] = 0;  // leave the workspace zeroed for the next call
}

// Plan of the grouped kernel: splits sized on the B*H_kv streams, one CTA
// per SM; the records are per query head.
inline Plan gqa_plan(long long B, long long H, long long H_kv, long long n, long long D, int num_sms,
                     bool ragged) {
  Plan pl = make_plan(B * H_kv, n, D, num_sms / 2 > 0 ? num_sms / 2 : 1, ragged);  // make_plan counts 2 CTAs per SM
  pl.total_bytes = pl.rec_off + round_up((size_t)B * H * pl.splits * (D + 2) * sizeof(float), 256);
  return pl;
}

template <typename QT, typename KVT, int D>
int launch_gqa_g(const Params& prm, int G, dim3 grid, cudaStream_t st) {
  switch (G) {
    case 2: gqa_kernel<QT, KVT, D, 2><<<grid, kThreads, 0, st>>>(prm); break;
    case 4: gqa_kernel<QT, KVT, D, 4><<<grid, kThreads, 0, st>>>(prm); break;
    default: gqa_kernel<QT, KVT, D, 8><<<grid, kThreads, 0, st>>>(prm); break;
  }
  return check_cuda(cudaGetLastError(), "grouped-head decode launch");
}

template <typename QT, int D>
int launch_gqa_kv(const Params& prm, int kv_dtype, int G, dim3 grid, cudaStream_t st) {
  if (kv_dtype == PU_DTYPE_F16) return launch_gqa_g<QT, __half, D>(prm, G, grid, st);
  if (kv_dtype == PU_DTYPE_BF16) return launch_gqa_g<QT, __nv_bfloat16, D>(prm, G, grid, st);
  return launch_gqa_g<QT, __nv_fp8_e4m3, D>(prm, G, grid, st);
}

inline int launch_gqa(const Params& prm, int q_dtype, int kv_dtype, int D, int G, int BH_kv, cudaStream_t st) {
  const dim3 grid(prm.splits, BH_kv);
  const bool qh = (q_dtype == PU_DTYPE_F16);
  if (D == 128) return qh ? launch_gqa_kv<__half, 128>(prm, kv_dtype, G, grid, st)
                          : launch_gqa_kv<__nv_bfloat16, 128>(prm, kv_dtype, G, grid, st);
  return qh ? launch_gqa_kv<__half, 64>(prm, kv_dtype, G, grid, st)
            : launch_gqa_kv<__nv_bfloat16, 64>(prm, kv_dtype, G, grid, st);
}

inline bool gqa_grouped(long long H, long long H_kv) {
  const long long G = H / H_kv;
  return G == 2 || G == 4 || G == 8;
}

}  // namespace decode
}  // namespace pu
