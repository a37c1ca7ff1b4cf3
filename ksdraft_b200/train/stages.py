"""PTQR dithered quantisation (drop-in for ksdraft/train/stages.py:27-50).

The reference adds uniform noise from `torch.rand` on a (by default global)
generator, which cannot be replayed across devices.  Here the noise comes
from a counter-based Philox4x32-10 stream evaluated inside the quantiser
kernel: element i of the padded (rows, Kp) grid gets
U = (philox(seed, offset + i) >> 8) * 2**-24 and the code is
clamp(round(x/scale + (U - 0.5) * 2*dither), -127, 127).  dither=0 is exactly
`quantize_last_dim`.  With `seed=None` the seed is drawn from `generator`
(or torch's default generator), so seeding torch makes runs reproducible.
"""

from __future__ import annotations

import torch

from ..kernels.quant import (GROUP_SIZE, SCALE_DTYPE, _check_group, _padded_length,
                             _rows_view, quantize_rows_into)


def draw_seed(generator: torch.Generator | None = None) -> int:
    """A 63-bit Philox key drawn from a torch generator (CPU default if None)."""
    return int(torch.randint(0, 2**63 - 1, (1,), generator=generator).item())


def quantize_last_dim_dithered(x: torch.Tensor, group: int, dither: float,
                               generator: torch.Generator | None = None, *,
                               seed: int | None = None, offset: int = 0):
    """GS quantisation with rounding dither in [-dither, dither] code steps."""
    if not torch.is_floating_point(x):
        raise TypeError("quantize expects floating-point input")
    _check_group(group)
    if dither > 0 and seed is None:
        seed = draw_seed(generator)
    K = x.shape[-1]
    G = _padded_length(K, group) // group
    lead = x.shape[:-1]
    if x.dtype == torch.float64:
        x = x.float()
    codes = torch.empty(*lead, K, dtype=torch.int8, device=x.device)
    scales = torch.empty(*lead, G, dtype=SCALE_DTYPE, device=x.device)
    if codes.numel() == 0 and scales.numel() == 0:
        return codes, scales
    quantize_rows_into(_rows_view(x), codes.view(-1, K), scales.view(-1, G),
                       dither=float(dither) if dither > 0 else 0.0, seed=seed or 0, offset=offset)
    return codes, scales


__all__ = ["quantize_last_dim_dithered", "draw_seed", "GROUP_SIZE"]
