"""INT8 kernel tier on B200: GS128 W8A8 ops behind the ksdraft/kernels interface."""

from .quant import GROUP_SIZE, SCALE_DTYPE, quantize_last_dim, dequantize_last_dim
from .gemm import w8a8_gemm
from .linear import Int8Linear

__all__ = [
    "GROUP_SIZE", "SCALE_DTYPE",
    "quantize_last_dim", "dequantize_last_dim",
    "w8a8_gemm", "Int8Linear",
]
