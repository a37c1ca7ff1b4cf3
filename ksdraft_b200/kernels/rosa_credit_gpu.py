"""Rosa counterfactual credits on the GPU, the interface of
ksdraft/kernels/rosa_credit_gpu.py (HardRosaGPU, MAX_WINDOW).

HardRosaGPU's forward is the hard Rosa core (rosa.py:154-165): bits = proj > 0,
the longest-suffix match signs times the payload.  Its backward gives every
q / k / v projection the first-order single-bit counterfactual credit of its
bit -- flip it, re-match, project the change of the signs on dL/d sign -- through
the Bernoulli map sigmoid(x) (1 - sigmoid(x)) (rosa_credit_gpu.py:51-112).

The reference builds all 3T perturbed streams and re-matches each in full,
which it limits to T <= 63.  ksd8_rosa_credits recomputes only what a flip can
change, exactly (the v bit of a match's successor, the queries whose window
holds a flipped q bit within their match, the 64 keys whose windows hold a
flipped k bit), so windows up to MAX_WINDOW positions run; the work still grows
as T^2 per stream (about 64 key comparisons per (flip, later position)).
"""

from __future__ import annotations

import torch

from .. import _lib
from ..model.rosa import _default_max_len, pack_bits

MAX_WINDOW = 4096   # positions per stream; the C ABI accepts up to KSD8_ROSA_CREDITS_TMAX


def credits(qb: torch.Tensor, kb: torch.Tensor, vb: torch.Tensor, grad: torch.Tensor,
            max_len: int | None = None):
    """Credits of every bit: q / k / v bits (B, T, S) (nonzero = 1), grad (B, S, T)
    fp32 = dL/d sign.  Returns (cq, ck, cv), each (B, S, T) fp32: the change of
    sum_t sign(t) * grad(t) when that bit alone is flipped."""
    _lib.require_cuda(qb, kb, vb, grad)
    B, T, S = qb.shape
    if T > MAX_WINDOW:
        raise ValueError(f"credits support T <= {MAX_WINDOW}; got T={T}")
    words = [pack_bits(x.contiguous(), B, T, S, T * S, S, 1) for x in (qb, kb, vb)]
    g = grad.float().contiguous()
    out = [torch.empty(B, S, T, dtype=torch.float32, device=qb.device) for _ in range(3)]
    ml = _default_max_len(T, max_len)
    _lib.check(_lib.lib().ksd8_rosa_credits(
        words[0].data_ptr(), words[1].data_ptr(), words[2].data_ptr(), B * S, T, max(0, ml),
        g.data_ptr(), out[0].data_ptr(), out[1].data_ptr(), out[2].data_ptr(), None,
        _lib.stream_ptr(qb.device)), "rosa_credits")
    return tuple(out)


class HardRosaGPU(torch.autograd.Function):
    """q / k / v: (B, T, S) pre-bit projections; payload: (S,) -> hard (B, T, S).

    Forward: payload * sign of the longest-suffix match of the bits proj > 0
    (rosa.py:154-165).  Backward: exact single-bit counterfactual credits,
    delta = (1 - 2 bit) * credit, times sigmoid(x) (1 - sigmoid(x)); the
    payload gets sum over (B, T) of grad * sign (rosa_credit_gpu.py:79-112)."""

    @staticmethod
    def forward(ctx, q, k, v, payload):
        if q.shape[1] > MAX_WINDOW:
            raise ValueError(
                f"GPU exact credits support T <= {MAX_WINDOW}; got T={q.shape[1]}. "
                "Use the CPU engine or chunk the sequence.")
        _lib.require_cuda(q, k, v, payload)
        from ..model.rosa import _match_payload_sign
        qbits = (q > 0).to(torch.int8)
        kbits = (k > 0).to(torch.int8)
        vbits = (v > 0).to(torch.int8)
        sign = _match_payload_sign(qbits.permute(0, 2, 1), kbits.permute(0, 2, 1),
                                   vbits.permute(0, 2, 1))                # (B, S, T)
        ctx.save_for_backward(q, k, v, sign, payload)
        return (payload[None, :, None] * sign).permute(0, 2, 1)            # (B, T, S)

    @staticmethod
    def backward(ctx, grad_out):
        q, k, v, sign, payload = ctx.saved_tensors
        grad_hard = grad_out.permute(0, 2, 1).float()                      # (B, S, T)
        grad_sign = grad_hard * payload[None, :, None].float()
        bits = [(x > 0).to(torch.int8) for x in (q, k, v)]
        cr = credits(*bits, grad_sign)

        def bernoulli(pre):  # sigmoid(x)(1-sigmoid(x))/tau, tau = 1
            s = torch.sigmoid(pre)
            return (s * (1 - s)).to(pre.dtype)

        grads = []
        for c, b, pre in zip(cr, bits, (q, k, v)):
            delta = c * (1 - 2 * b.permute(0, 2, 1).float())                # (B, S, T)
            grads.append(delta.permute(0, 2, 1).to(pre.dtype) * bernoulli(pre))
        gp = (grad_hard * sign.float()).sum(dim=(0, 2))
        return grads[0], grads[1], grads[2], gp.to(payload.dtype)
