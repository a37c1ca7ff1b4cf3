"""Training-side pieces of the hot path: PTQR dither and the data-parallel step."""

from .stages import quantize_last_dim_dithered, draw_seed

__all__ = ["quantize_last_dim_dithered", "draw_seed"]
