"""`project_fused` (interface of ksdraft/kernels/ks3_triton.py:159-195) on ksd8 kernels.

Input projection GEMM + spine + ReLU^2 + GS requantisation of the features,
returning (h codes (M, N) int8, h scales (M, ceil(N/group)) fp16) ready for
the output-projection GEMM.  `warp_scale` / `warp_shift` are the DEQUANTISED
fp16 per-chart scalars, as in the reference.  The spine follows the composed
semantics of ks3_int8.py:169-234 (the reference's parity oracle); the
reference's Triton epilogue differs from it in three documented places
(fp32 vs fp16 LUT index, fp32 vs fp16 Horner scaling, per-row vs
per-element pre-scale) and is only tolerance-comparable.
"""

from __future__ import annotations

import torch

from .gemm import _validate_and_pad, gemm_out
from .ks3_int8 import TANH_DOMAIN, spine_quant  # noqa: F401 (reference names)
from .quant import _check_group

FP16 = torch.float16


def project_fused(a_codes, a_scales, w_codes, w_scales, spine_codes, spine_scale,
                  warp_scale, warp_shift, tanh_lut, group: int, nonlinear: str):
    if group & (group - 1):
        raise ValueError("group must be a power of two (32 or 128)")
    _check_group(group)
    a_codes, w_codes = _validate_and_pad(a_codes, a_scales, w_codes, w_scales, group)
    coords = gemm_out(a_codes, a_scales, w_codes, w_scales, out_dtype=FP16, clamp_f16=True)
    ws = warp_scale.to(FP16).reshape(-1).contiguous()
    wh = warp_shift.to(FP16).reshape(-1).contiguous()
    return spine_quant(coords, spine_codes.reshape(-1, 6).contiguous(),
                       spine_scale.reshape(-1).contiguous(), None, ws, None, wh,
                       tanh_lut.contiguous(), nonlinear)
