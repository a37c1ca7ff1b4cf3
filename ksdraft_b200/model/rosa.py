"""Rosa 1-bit hard-retrieval mixer on B200 (drop-in for ksdraft/model/rosa.py).

`_match_payload_sign` keeps the reference contract (rosa.py:40-98): bits
(..., T) in {0, 1} -> (..., T) fp32 in {+1, -1}; the longest suffix match is
capped at `max_match_len` = min(62, T-1) by default (the cap is part of the
semantics); among longest matches the latest endpoint j wins; the sign is the
key stream's successor value bit v[j+1].  It runs as two kernels: bit packing
(`ksd8_rosa_pack_bits`) and the per-stream match (`ksd8_rosa_match`), which
also exposes the match length and endpoint for parity checks.

`RosaMixer` mirrors rosa.py:101-165.  With Int8Linear projections (after
`to_int8`) its evaluation forward is the fused W8A8 pipeline: time-shift mix
fused with the per-token quantisation of the three projection inputs, three
GEMMs with bias writing fp32, bit packing straight from those outputs, the
match with the payload multiply fused into its token-major (B, T, S) store,
the per-token quantisation of that result and the output GEMM.  In training
mode it takes the reference's CUDA path: the hard core through HardRosaGPU
(kernels/rosa_credit_gpu.py), whose counterfactual credits give the q / k / v
projections their gradients.
"""

from __future__ import annotations

import torch
from torch import nn
from torch.nn import functional as F

from .. import _lib


def _default_max_len(t_len: int, max_match_len: int | None) -> int:
    if max_match_len is None:
        return max(1, min(62, t_len - 1)) if t_len > 1 else 0
    return min(max_match_len, t_len - 1)


def pack_bits(x: torch.Tensor, batch: int, t_len: int, streams: int, sb: int, st: int,
              ss: int) -> torch.Tensor:
    """Words (batch*streams, ceil(T/64)) uint64-as-int64 of bits x[b, t, s] > 0."""
    words = torch.empty(batch * streams, (t_len + 63) // 64, dtype=torch.int64, device=x.device)
    rc = _lib.lib().ksd8_rosa_pack_bits(x.data_ptr(), _lib.dtype_code(x), batch, t_len, streams,
                                        sb, st, ss, words.data_ptr(), None,
                                        _lib.stream_ptr(x.device))
    _lib.check(rc, "rosa_pack_bits")
    return words


def match_words(qw, kw, vw, batch: int, streams: int, t_len: int, max_len: int, *,
                payload: torch.Tensor | None = None, out: torch.Tensor,
                strides: tuple[int, int, int], with_indices: bool = False):
    dev = qw.device
    ml = me = None
    if with_indices:
        ml = torch.empty(batch * streams, t_len, dtype=torch.int32, device=dev)
        me = torch.empty(batch * streams, t_len, dtype=torch.int32, device=dev)
    pay = payload.detach().float().contiguous() if payload is not None else None
    # scratch of the adaptive matcher: [count, stream ids handed to the sorted kernel]
    scratch = torch.empty(1 + batch * streams, dtype=torch.int32, device=dev)
    rc = _lib.lib().ksd8_rosa_match_scratch(
        qw.data_ptr(), kw.data_ptr(), vw.data_ptr(), batch, streams, t_len, max(0, max_len),
        _lib.ptr(pay), out.data_ptr(), _lib.dtype_code(out), *strides, _lib.ptr(ml),
        _lib.ptr(me), scratch.data_ptr(), scratch.numel(), None, _lib.stream_ptr(dev))
    _lib.check(rc, "rosa_match")
    return ml, me


def match_payload_sign_with_indices(qbits, kbits, vbits, max_match_len=None):
    """(sign (..., T) fp32, match length (..., T) int32, endpoint j (..., T) int32 or -1)."""
    _lib.require_cuda(qbits, kbits, vbits)
    *lead, t_len = qbits.shape
    n = 1
    for d in lead:
        n *= d
    sign = torch.empty(*lead, t_len, dtype=torch.float32, device=qbits.device)
    if n == 0 or t_len == 0:
        z = torch.zeros(*lead, t_len, dtype=torch.int32, device=qbits.device)
        return sign.fill_(-1.0), z, z - 1
    words = []
    for b in (qbits, kbits, vbits):
        b2 = b.reshape(n, t_len)
        if b2.dtype == torch.bool:
            b2 = b2.to(torch.int8)
        if b2.dtype not in (torch.int8, torch.float32, torch.bfloat16, torch.float16):
            b2 = b2.to(torch.int8)
        words.append(pack_bits(b2, 1, t_len, n, 0, b2.stride(1), b2.stride(0)))
    ml, me = match_words(*words, 1, n, t_len, _default_max_len(t_len, max_match_len),
                         out=sign, strides=(0, 1, t_len), with_indices=True)
    return sign, ml.reshape(*lead, t_len), me.reshape(*lead, t_len)


def _match_payload_sign(qbits: torch.Tensor, kbits: torch.Tensor, vbits: torch.Tensor,
                        max_match_len: int | None = None) -> torch.Tensor:
    """Longest-suffix-match payload signs, (..., T) bits -> (..., T) fp32 +-1."""
    _lib.require_cuda(qbits, kbits, vbits)
    *lead, t_len = qbits.shape
    n = 1
    for d in lead:
        n *= d
    sign = torch.empty(*lead, t_len, dtype=torch.float32, device=qbits.device)
    if n == 0 or t_len == 0:
        return sign.fill_(-1.0)
    words = []
    for b in (qbits, kbits, vbits):
        b2 = b.reshape(n, t_len)
        if b2.dtype not in (torch.int8, torch.float32, torch.bfloat16, torch.float16):
            b2 = b2.to(torch.int8)
        words.append(pack_bits(b2, 1, t_len, n, 0, b2.stride(1), b2.stride(0)))
    match_words(*words, 1, n, t_len, _default_max_len(t_len, max_match_len), out=sign,
                strides=(0, 1, t_len))
    return sign


class RosaMixer(nn.Module):
    def __init__(self, d_model: int, streams: int = 512, bits: int = 1):
        super().__init__()
        if bits != 1:
            raise NotImplementedError(
                "reference implements 1-bit streams (the decided configuration); "
                "n-bit packed symbols arrive with the production kernel")
        self.d_model = d_model
        self.streams = streams
        self.bits = bits
        self.q_proj = nn.Linear(d_model, streams, bias=True)
        self.k_proj = nn.Linear(d_model, streams, bias=True)
        self.v_proj = nn.Linear(d_model, streams, bias=True)
        self.out_proj = nn.Linear(streams, d_model, bias=True)
        self.time_mix_q = nn.Parameter(torch.zeros(d_model))
        self.time_mix_k = nn.Parameter(torch.zeros(d_model))
        self.time_mix_v = nn.Parameter(torch.zeros(d_model))
        self.payload = nn.Parameter(torch.ones(streams))
        nn.init.zeros_(self.out_proj.weight)
        nn.init.zeros_(self.out_proj.bias)

    def _shifted(self, x: torch.Tensor):
        prev = F.pad(x, (0, 0, 1, 0))[:, :-1, :]
        q_in = prev + (x - prev) * torch.sigmoid(self.time_mix_q)
        k_in = prev + (x - prev) * torch.sigmoid(self.time_mix_k)
        v_in = prev + (x - prev) * torch.sigmoid(self.time_mix_v)
        return q_in, k_in, v_in

    def _fused_int8_eval(self) -> bool:
        from ..kernels.linear import Int8Linear
        return (not torch.is_grad_enabled() and all(
            isinstance(getattr(self, n), Int8Linear)
            for n in ("q_proj", "k_proj", "v_proj", "out_proj")))

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        """x (B, T, d) -> (B, T, d)."""
        _lib.require_cuda(x)
        if self._fused_int8_eval():
            return rosa_forward_int8(self, x)
        q_in, k_in, v_in = self._shifted(x)
        if self.training:
            # the reference's CUDA training path (rosa.py:141-145): the hard core
            # through HardRosaGPU, whose counterfactual credits give the q / k / v
            # projections gradients (ValueError beyond its window, as there)
            from ..kernels.rosa_credit_gpu import HardRosaGPU
            hard = HardRosaGPU.apply(self.q_proj(q_in), self.k_proj(k_in), self.v_proj(v_in),
                                     self.payload)
            return self.out_proj(hard.to(x.dtype))
        qbits = (self.q_proj(q_in) > 0).to(torch.int8)
        kbits = (self.k_proj(k_in) > 0).to(torch.int8)
        vbits = (self.v_proj(v_in) > 0).to(torch.int8)
        sign = _match_payload_sign(qbits.permute(0, 2, 1), kbits.permute(0, 2, 1),
                                   vbits.permute(0, 2, 1))
        out = self.payload[None, :, None] * sign
        return self.out_proj(out.permute(0, 2, 1).to(x.dtype))


@torch.no_grad()
def rosa_forward_int8(mixer: RosaMixer, x: torch.Tensor) -> torch.Tensor:
    """Fused W8A8 evaluation forward of a RosaMixer whose projections are Int8Linear."""
    from ..kernels.gemm import _validate_and_pad, gemm_out
    from ..kernels.quant import quantize_last_dim
    B, T, d = x.shape
    S = mixer.streams
    dev = x.device
    x = x.contiguous()
    G = (d + 127) // 128
    codes = [torch.empty(B * T, d, dtype=torch.int8, device=dev) for _ in range(3)]
    scales = [torch.empty(B * T, G, dtype=torch.float16, device=dev) for _ in range(3)]
    mixes = [torch.sigmoid(p.detach().float()).contiguous()
             for p in (mixer.time_mix_q, mixer.time_mix_k, mixer.time_mix_v)]
    rc = _lib.lib().ksd8_rosa_timemix_quantize(
        x.data_ptr(), _lib.dtype_code(x), B, T, d, *(m.data_ptr() for m in mixes),
        codes[0].data_ptr(), scales[0].data_ptr(), codes[1].data_ptr(), scales[1].data_ptr(),
        codes[2].data_ptr(), scales[2].data_ptr(), None, _lib.stream_ptr(dev))
    _lib.check(rc, "rosa_timemix_quantize")
    # _shifted promotes to fp32 (bf16 activations x fp32 sigmoid(time_mix)), so
    # the projections, and the bits taken from them, are fp32 (rosa.py:128-158).
    out_dtype = x.dtype if x.dtype in (torch.bfloat16, torch.float16, torch.float32) \
        else torch.float32
    words = []
    for i, name in enumerate(("q_proj", "k_proj", "v_proj")):
        lin = getattr(mixer, name)
        lin._quantize_weight()
        proj = gemm_out(codes[i], scales[i], lin.weight_codes, lin.weight_scales,
                        out_dtype=torch.float32,
                        bias=lin.bias.detach() if lin.bias is not None else None)
        words.append(pack_bits(proj, B, T, S, T * S, S, 1))
    # the match writes payload * sign token-major, (B, T, S): the out_proj input
    # rows (rosa.py:164-165) quantised along the streams with no transpose
    mixed = torch.empty(B, T, S, dtype=out_dtype, device=dev)
    match_words(*words, B, S, T, _default_max_len(T, None), payload=mixer.payload, out=mixed,
                strides=(T * S, S, 1))
    lin = mixer.out_proj
    lin._quantize_weight()
    oq, os_ = quantize_last_dim(mixed.reshape(B * T, S))
    oq, wq = _validate_and_pad(oq, os_, lin.weight_codes, lin.weight_scales, 128)
    y = gemm_out(oq, os_, wq, lin.weight_scales, out_dtype=out_dtype,
                 bias=lin.bias.detach() if lin.bias is not None else None)
    return y.reshape(B, T, d).to(x.dtype)
