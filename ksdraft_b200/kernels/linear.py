"""Int8Linear — W8A8 GS128 drop-in for nn.Linear (mirrors ksdraft/kernels/linear.py:23-97).

Same parameters, buffers and `_dither` attribute protocol as the reference:
fp32 master `weight` (+ optional `bias`), non-persistent `weight_codes` /
`weight_scales` re-derived from the master on every call.  Evaluation runs
the fused W8A8 path: per-token GS128 quantisation of the input, then the
tensor-core GEMM with the bias added in its epilogue and the output written
directly in the input's dtype.  Training keeps the reference's
straight-through `fake_quant_forward` (fp32 GEMM on quantise-dequantised
operands, linear.py:75-97) so gradients match the reference.
"""

from __future__ import annotations

import torch
from torch import nn

from .gemm import gemm_out, _validate_and_pad, w8a8_gemm  # noqa: F401 (reference names)
from .quant import GROUP_SIZE, dequantize_last_dim, quantize_last_dim


class Int8Linear(nn.Module):
    def __init__(self, in_features: int, out_features: int, bias: bool = True):
        super().__init__()
        self.in_features = in_features
        self.out_features = out_features
        self.weight = nn.Parameter(torch.zeros(out_features, in_features))
        self.bias = nn.Parameter(torch.zeros(out_features)) if bias else None
        self.register_buffer("weight_codes", None, persistent=False)
        self.register_buffer("weight_scales", None, persistent=False)

    @classmethod
    def from_float(cls, module: nn.Linear) -> "Int8Linear":
        lin = cls(module.in_features, module.out_features, bias=module.bias is not None)
        with torch.no_grad():
            lin.weight.copy_(module.weight)
            if module.bias is not None:
                lin.bias.copy_(module.bias)
        lin = lin.to(module.weight.device)
        if lin.weight.is_cuda:
            lin._quantize_weight()
        return lin

    @torch.no_grad()
    def _quantize_weight(self) -> None:
        dither = float(getattr(self, "_dither", 0.0))
        if dither > 0:
            from ..train.stages import quantize_last_dim_dithered
            codes, scales = quantize_last_dim_dithered(
                self.weight.detach().float(), GROUP_SIZE, dither,
                seed=getattr(self, "_dither_seed", None))
        else:
            codes, scales = quantize_last_dim(self.weight.detach().float())
        self.weight_codes = codes
        self.weight_scales = scales

    def _quantize_weight_dithered(self, dither: float) -> None:
        self._dither = dither
        self._quantize_weight()

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        if torch.is_grad_enabled() and self.weight.requires_grad:
            return self.fake_quant_forward(x)
        self._quantize_weight()
        x2 = x.reshape(-1, x.shape[-1])
        a_codes, a_scales = quantize_last_dim(x2)
        a_codes, w_codes = _validate_and_pad(a_codes, a_scales, self.weight_codes,
                                             self.weight_scales, GROUP_SIZE)
        out_dtype = x.dtype if x.dtype in (torch.float32, torch.bfloat16, torch.float16) \
            else torch.float32
        y = gemm_out(a_codes, a_scales, w_codes, self.weight_scales, out_dtype=out_dtype,
                     bias=self.bias.detach() if self.bias is not None else None)
        return y.reshape(*x.shape[:-1], self.out_features).to(x.dtype)

    def fake_quant_forward(self, x: torch.Tensor) -> torch.Tensor:
        """STE path (linear.py:75-97): fp32 GEMM on quantise-dequantised operands.

        The weight is quantised without grad (straight through); the input's
        quantisation carries the reference's scale gradient (ste_input_grad)."""
        self._quantize_weight()
        w = dequantize_last_dim(self.weight_codes.detach().float(), self.weight_scales.detach()) \
            + (self.weight - self.weight.detach())
        x2 = x.reshape(-1, x.shape[-1]).float()
        xq = _QuantSTE.apply(x2)
        y = xq @ w.reshape(self.out_features, self.in_features).T
        if self.bias is not None:
            y = y + self.bias.float()
        return y.reshape(*x.shape[:-1], self.out_features).to(x.dtype)


def ste_input_grad(x: torch.Tensor, codes: torch.Tensor, gx: torch.Tensor) -> torch.Tensor:
    """Input gradient of the reference's STE quantisation (linear.py:92-93).

    quantize_last_dim runs on the grad-carrying input there, so besides the
    straight-through gx the GS128 scale = fp16(clamp(amax / 127, 2^-24, 65504))
    (quant.py:47-49) passes a gradient: per group G = sum(gx * codes), rounded to
    fp16 where it crosses the fp16 scale tensor, / 127, only inside the clamp
    range, split evenly over the elements tied at amax, times their sign.
    x, codes, gx: (M, K) on the device; returns gx + that term (fp32)."""
    M, K = x.shape
    pad = -K % GROUP_SIZE
    xp = torch.nn.functional.pad(x.float(), (0, pad)).reshape(M, -1, GROUP_SIZE)
    cp = torch.nn.functional.pad(codes.float(), (0, pad)).reshape(M, -1, GROUP_SIZE)
    gp = torch.nn.functional.pad(gx.float(), (0, pad)).reshape(M, -1, GROUP_SIZE)
    a = xp.abs()
    amax = a.amax(-1, keepdim=True)
    tie = a == amax
    g16 = (gp * cp).sum(-1, keepdim=True).to(torch.float16).float()
    s32 = amax / 127.0
    inside = (s32 >= 2.0**-24) & (s32 <= 65504.0)
    share = torch.where(inside, g16 / 127.0 / tie.sum(-1, keepdim=True), 0.0)
    extra = torch.where(tie, torch.sign(xp) * share, 0.0)
    return gx.float() + extra.reshape(M, -1)[:, :K]


class _QuantSTE(torch.autograd.Function):
    """deq(q(x)) with the reference's STE gradient (ste_input_grad)."""

    @staticmethod
    def forward(ctx, x2):
        codes, scales = quantize_last_dim(x2.detach())
        ctx.save_for_backward(x2.detach(), codes)
        return dequantize_last_dim(codes, scales)

    @staticmethod
    def backward(ctx, g):
        x2, codes = ctx.saved_tensors
        return ste_input_grad(x2, codes, g)
