"""B200 (sm_100a) fused QKV projection, Q/K RMSNorm, NeoX RoPE and Ulysses
exchange: a drop-in for joey-shao/flash_ulysses' ``FlashUlyssesContext``; with
``output_projection=True`` the context also runs the inverse exchange after
attention fused with the output projection.

``FlashUlyssesContext`` is resolved on first access, which loads the CUDA
library (and raises ``ImportError`` if it is not built: there is no CPU
fallback).  Importing a submodule that needs no GPU code, such as
``flash_ulysses_b200.workloads``, does not load the library.
"""

__version__ = "0.1.0"
__all__ = ["FlashUlyssesContext"]


def __getattr__(name):
    if name == "FlashUlyssesContext":
        from .context import FlashUlyssesContext

        return FlashUlyssesContext
    raise AttributeError(f"module {__name__!r} has no attribute {name!r}")
