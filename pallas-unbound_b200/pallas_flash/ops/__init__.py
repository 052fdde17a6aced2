from .interface import pallas_flash_attention

__all__ = ["pallas_flash_attention"]
