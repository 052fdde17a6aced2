"""pallas_flash — B200 (sm_100a) implementation of Pallas-Unbound's attention
hot path, importable under the reference's own module paths:

    from pallas_flash.ops.interface import pallas_flash_attention
    from pallas_flash.kernels.decoding import pallas_flash_decoding

All compute runs in libpu_attn.so through its C ABI (include/pu_attn.h).
"""
from .ops.interface import pallas_flash_attention
from .kernels.decoding import pallas_flash_decoding

__all__ = ["pallas_flash_attention", "pallas_flash_decoding"]
