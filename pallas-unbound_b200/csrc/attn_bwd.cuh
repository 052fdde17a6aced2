// attn_bwd.cuh — training-attention backward (placeholder until the tcgen05
// kernel lands).
#pragma once
#include "pu_host.cuh"

extern "C" size_t pu_attn_bwd_workspace_size(int64_t B, int64_t H, int64_t Nq, int64_t D) {
  return (size_t)(B * H * Nq * D * 4 + B * H * Nq * 4 + 4096);
}

extern "C" int pu_attn_bwd(const void*, const void*, const void*, const void*, const float*,
                           const void*, void*, void*, void*, void*, size_t, int64_t, int64_t,
                           int64_t, int64_t, int64_t, float, int, void*) {
  return pu::set_error(PU_ERR_UNSUPPORTED, "backward not built yet");
}
