// pu_host.cuh — host-side helpers: TMA tensor-map encoding through the
// driver entry point (so the library does not link libcuda directly), SM
// count cache, argument checks.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <cudaTypedefs.h>

#include <cstdint>

#include "pu_status.cuh"

namespace pu {

// Encode a 3-D bf16 tensor map over a dense [outer, rows, cols] array with a
// (box_cols x box_rows x 1) box and 128-byte swizzle.  Out-of-range rows read
// as zero.  Returns PU_OK or an error code (message set).
int make_tmap_bf16_3d(CUtensorMap* map, const void* base, uint64_t cols, uint64_t rows,
                      uint64_t outer, uint32_t box_cols, uint32_t box_rows, bool swizzle128);

// Same for 8-bit elements (fp8 caches).
int make_tmap_u8_3d(CUtensorMap* map, const void* base, uint64_t cols, uint64_t rows, uint64_t outer,
                    uint32_t box_cols, uint32_t box_rows, bool swizzle128);

// Same for fp32 elements (used for the dQ accumulator).
int make_tmap_f32_3d(CUtensorMap* map, const void* base, uint64_t cols, uint64_t rows,
                     uint64_t outer, uint32_t box_cols, uint32_t box_rows, bool swizzle128);

// Number of SMs of the current device (cached per device).
int sm_count();

// Current device ordinal (or -1 with the error set).
int current_device();

// Raise `func`'s dynamic shared-memory limit to `bytes` on the current device,
// once per (kernel, device); thread-safe.  Returns PU_OK or an error code.
int set_max_dynamic_smem(const void* func, int bytes, const char* what);

inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

}  // namespace pu
