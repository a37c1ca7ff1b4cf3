"""GS128 symmetric INT8 quantisation on the GPU (drop-in for ksdraft/kernels/quant.py).

Contract (ksdraft/kernels/quant.py:1-14, kept unchanged):
- symmetric per-group scales, group size 128 along the LAST dimension;
- scales stored fp16, rounded BEFORE encoding, bounded to [2**-24, 65504];
- codes saturate to [-127, 127], round half to even;
- a last dimension that is not a multiple of 128 is zero-padded to the next
  group; the returned codes keep the original length.

`quantize_last_dim` runs `ksd8_quantize_rows`: contiguous rows of whole
groups stream through shared memory by cp.async.bulk, anything else takes the
thread-load kernel (one warp per row-group); `quantize_cols` stages 128 x 128
tiles by TMA when the rows are 16-byte aligned.  `plain_loads=True` forces the
thread-load kernels (identical results; the tests compare the two).  There is
no CPU path: non-CUDA inputs raise.
"""

from __future__ import annotations

import torch

from .. import _lib

GROUP_SIZE = 128
SCALE_DTYPE = torch.float16
SCALE_MIN = 2.0**-24
SCALE_MAX = 65504.0


def _padded_length(n: int, group: int = GROUP_SIZE) -> int:
    return (n + group - 1) // group * group


def _check_group(group: int) -> None:
    """The GS128 grid is the one this build implements (the north-star layout);
    any other group is rejected as an invalid argument, as the reference rejects
    groups its kernels cannot tile (ks3_triton.py:185-186)."""
    if group != GROUP_SIZE:
        raise ValueError(f"ksdraft_b200 implements the GS128 grid only (group={group} requested)")


def _rows_view(x: torch.Tensor) -> torch.Tensor:
    """(..., K) -> (R, K) with unit stride along K (copies only if needed)."""
    x2 = x.reshape(-1, x.shape[-1]) if x.dim() != 2 else x
    if x2.shape[-1] > 0 and x2.stride(-1) != 1:
        x2 = x2.contiguous()
    if x2.shape[0] > 1 and x2.stride(0) < x2.shape[1]:
        x2 = x2.contiguous()
    return x2


def quantize_rows_into(x: torch.Tensor, codes: torch.Tensor, scales: torch.Tensor, *,
                       round_f16: bool = False, dither: float = 0.0, seed: int = 0,
                       offset: int = 0, plain_loads: bool = False) -> None:
    """Quantise the rows of a 2-D CUDA tensor into preallocated codes/scales."""
    _lib.require_cuda(x, codes, scales)
    R, K = x.shape
    flags = (_lib.Q_ROUND_F16 if round_f16 else 0) | (_lib.Q_DITHER if dither > 0 else 0) | \
        (_lib.Q_PLAIN_LOADS if plain_loads else 0)
    rc = _lib.lib().ksd8_quantize_rows(
        x.data_ptr(), _lib.dtype_code(x), R, K, x.stride(0) if R > 1 else K, GROUP_SIZE, flags,
        float(dither), seed & (2**64 - 1), offset & (2**64 - 1), codes.data_ptr(),
        codes.stride(0) if R > 1 else K, scales.data_ptr(), None, _lib.stream_ptr(x.device))
    _lib.check(rc, "quantize_last_dim")


def quantize_last_dim(x: torch.Tensor, group: int = GROUP_SIZE
                      ) -> tuple[torch.Tensor, torch.Tensor]:
    """x (..., K) float -> (codes int8 (..., K), scales fp16 (..., ceil(K/128))).

    Same results as ksdraft/kernels/quant.py:30-52 for fp32/bf16/fp16 inputs
    (bf16/fp16 are quantised from their exact fp32 values, as the reference's
    promotion does); fp64 inputs are rounded to fp32 first.
    """
    if not torch.is_floating_point(x):
        raise TypeError("quantize expects floating-point input")
    _check_group(group)
    _lib.require_cuda(x)
    if x.dtype == torch.float64:
        x = x.float()
    K = x.shape[-1]
    G = _padded_length(K, group) // group
    lead = x.shape[:-1]
    codes = torch.empty(*lead, K, dtype=torch.int8, device=x.device)
    scales = torch.empty(*lead, G, dtype=SCALE_DTYPE, device=x.device)
    if codes.numel() == 0 and scales.numel() == 0:
        return codes, scales
    x2 = _rows_view(x)
    quantize_rows_into(x2, codes.view(-1, K) if K else codes.reshape(-1, 0),
                       scales.view(-1, G))
    return codes, scales


def dequantize_last_dim(codes: torch.Tensor, scales: torch.Tensor,
                        group: int | None = None) -> torch.Tensor:
    """Inverse of quantize_last_dim (exact on the codes it produced), fp32.

    Elementwise code * scale as in ksdraft/kernels/quant.py:55-67; the W8A8
    paths of this package never materialise it (the transposed requantiser
    dequantises on the fly)."""
    K = codes.shape[-1]
    if group is None:
        group = _padded_length(K) // max(scales.shape[-1], 1)
    Kp = _padded_length(K, group)
    if Kp != K:
        codes = torch.nn.functional.pad(codes, (0, Kp - K))
    grouped = codes.reshape(*codes.shape[:-1], Kp // group, group)
    return (grouped.float() * scales.float()[..., None]).reshape(*codes.shape[:-1], Kp)[..., :K]


def quantize_cols(x: torch.Tensor, *, x_scales: torch.Tensor | None = None,
                  x_group: int = GROUP_SIZE, round_f16: bool = False,
                  plain_loads: bool = False) -> tuple[torch.Tensor, torch.Tensor]:
    """quantize_last_dim(x.t().contiguous()) in one pass, x 2-D (R, C).

    With int8 `x` and its `x_scales`, x is first dequantised (code * scale),
    i.e. quantize_last_dim(dequantize_last_dim(x, x_scales).t()) — the
    requantised transposes of ksdraft/kernels/ks3_int8.py:350, :407-424."""
    _lib.require_cuda(x)
    R, C = x.shape
    if x.stride(-1) != 1:
        x = x.contiguous()
    G = _padded_length(R) // GROUP_SIZE
    codes = torch.empty(C, R, dtype=torch.int8, device=x.device)
    scales = torch.empty(C, G, dtype=SCALE_DTYPE, device=x.device)
    rc = _lib.lib().ksd8_quantize_cols(
        x.data_ptr(), _lib.dtype_code(x), _lib.ptr(x_scales), x_group, R, C,
        x.stride(0) if R > 1 else C, GROUP_SIZE,
        (_lib.Q_ROUND_F16 if round_f16 else 0) | (_lib.Q_PLAIN_LOADS if plain_loads else 0),
        codes.data_ptr(), R, scales.data_ptr(), None, _lib.stream_ptr(x.device))
    _lib.check(rc, "quantize_cols")
    return codes, scales
