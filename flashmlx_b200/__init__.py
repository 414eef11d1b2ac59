"""flashmlx_b200 -- B200-native MoE block for FlashMLX-style inference.

The product is libflashmoe (lib/libflashmoe.so, C ABI in include/flashmoe.h): router,
top-k, token/expert sort, 4-bit affine grouped SwiGLU experts, weighted combine and
the sigmoid-gated shared expert as sm_100a kernels.  `flashmlx_b200.ops` is the Python
mirror of the reference's operator calls on top of that ABI (torch only for device
buffers and streams); importing it without a built library raises ImportError.
"""
from . import synthetic  # noqa: F401  (numpy only)

__all__ = ["synthetic"]
