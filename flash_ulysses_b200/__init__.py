"""B200 (sm_100a) fused QKV projection, Q/K RMSNorm, NeoX RoPE and Ulysses
exchange: a drop-in for joey-shao/flash_ulysses' ``FlashUlyssesContext``; with
``output_projection=True`` the context also runs the inverse exchange after
attention fused with the output projection."""

from .context import FlashUlyssesContext

__version__ = "0.1.0"
__all__ = ["FlashUlyssesContext"]
