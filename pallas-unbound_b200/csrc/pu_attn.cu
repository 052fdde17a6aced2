// pu_attn.cu — the single translation unit of libpu_attn.so.  The kernels
// share one per-device status word (a __device__ variable), so they are
// compiled together instead of with relocatable device code.
#include "capi.cuh"
#include "decode.cuh"
#include "attn_fwd.cuh"
#include "attn_bwd.cuh"
