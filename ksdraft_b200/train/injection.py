"""DSpine adjacent injection + ln_ffn of one DraftBlock, forward and backward,
with the per-layer transfer-space loss rows (training step internals).

Reference: AdjacentInjection.forward (ksdraft/model/spine.py:56-69), the
block's `y = h + ffn(ln_ffn(h))` input (ksdraft/model/block.py:40-41) and the
transfer-space term of distillation_losses (ksdraft/train/__init__.py:80-85).

The low-rank projections are regrouped into five cuBLAS GEMMs in the
activation dtype (the reference runs them as eight nn.Linear calls):

    D1   = h @ [feature_down; gate_q.down]^T           (M, 64 + 32)
    p    = D1[:, :64] @ feature_up^T                    (M, d)
    P2   = p @ [gate_p.down; inject.down]^T             (M, 32 + 32)
    zsum = [D1[:, 64:], shift(P2[:, :32])] @ [gate_q.up, gate_p.up]^T
    inj  = shift(P2[:, 32:]) @ inject.up^T

where shift() moves every sequence's rows one position later and puts the
projections of the previous layer's p_0 (or zeros) at position 0 -- the
low-rank image of spine.py's p_prev, since a row-wise linear map commutes with
the shift.  ksd8_dspine_ln_fwd then forms h2 = h + sigmoid(zsum + gate_bias) *
inj and b = LayerNorm(h2) in one pass; ksd8_dspine_ln_bwd is its backward
(LayerNorm, gate, the three column sums), and ksd8_transfer_rows /
ksd8_transfer_bwd give the transfer term and its F.normalize backward.
"""

from __future__ import annotations

from types import SimpleNamespace

import torch

from .. import _lib

LN_EPS = 1e-5


def check_width(d: int) -> None:
    if d % 128 or d > 2048:
        raise ValueError(f"the fused injection + ln_ffn kernels need d_model % 128 == 0 and "
                         f"d_model <= 2048; got {d}")


def _stream(t: torch.Tensor):
    return _lib.stream_ptr(t.device)


def _shifted(low: torch.Tensor, first: torch.Tensor | None, B: int, T: int, out: torch.Tensor):
    """out (B, T, k) = low (M, k) one position later per sequence; row 0 = first (B, k) or 0."""
    o = out.view(B, T, -1)
    o[:, 1:].copy_(low.view(B, T, -1)[:, :-1])
    if first is None:
        o[:, 0].zero_()
    else:
        o[:, 0].copy_(first)


def _unshifted(g: torch.Tensor, B: int, T: int, out: torch.Tensor):
    """Adjoint of _shifted: out (M, k) row t = g row t + 1 (0 at the last position);
    returns g's rows at position 0 (the gradient of `first`)."""
    o = out.view(B, T, -1)
    gv = g.view(B, T, -1)
    o[:, :-1].copy_(gv[:, 1:])
    o[:, -1].zero_()
    return gv[:, 0]


class InjectionWeights:
    """The block's injection masters (fp32 flat views) regrouped for the five
    GEMMs, cast to the activation dtype once per step."""

    def __init__(self, W: dict, act: torch.dtype):
        self.fr = W["feature_down"].shape[0]
        self.r = W["gate_q.down"].shape[0]
        self.wd1 = torch.cat([W["feature_down"], W["gate_q.down"]], 0).to(act)   # (fr + r, d)
        self.wfu = W["feature_up"].to(act)                                        # (d, fr)
        self.wd2 = torch.cat([W["gate_p.down"], W["inject.down"]], 0).to(act)    # (2r, d)
        self.wu1 = torch.cat([W["gate_q.up"], W["gate_p.up"]], 1).to(act)        # (d, 2r)
        self.wiu = W["inject.up"].to(act)                                         # (d, r)
        self.gate_bias = W["gate_bias"].contiguous()


def forward(h: torch.Tensor, p_first: torch.Tensor | None, w: InjectionWeights,
            ln_w: torch.Tensor, ln_b: torch.Tensor, B: int, T: int):
    """h (M, d) activation dtype (the Rosa residual x + rosa(ln_attn(x))), p_first
    (B, d) the previous layer's p at position 0 or None.  Returns (b, h2, p,
    saved): b = ln_ffn(h2) for the KS3 cell, h2 the block's residual stream, p
    the predicted feature."""
    M, d = h.shape
    act = h.dtype
    r, fr = w.r, w.fr
    lib = _lib.lib()
    d1 = h @ w.wd1.t()
    p = d1[:, :fr] @ w.wfu.t()
    p2 = p @ w.wd2.t()
    f0 = None if p_first is None else p_first @ w.wd2.t()
    u1 = torch.empty(M, 2 * r, dtype=act, device=h.device)
    u1.view(B, T, 2 * r)[..., :r].copy_(d1.view(B, T, fr + r)[..., fr:])
    _shifted(p2[:, :r], None if f0 is None else f0[:, :r], B, T, u1[:, r:])
    u2 = torch.empty(M, r, dtype=act, device=h.device)
    _shifted(p2[:, r:], None if f0 is None else f0[:, r:], B, T, u2)
    zsum = u1 @ w.wu1.t()
    inj = u2 @ w.wiu.t()
    h2 = torch.empty_like(h)
    b = torch.empty_like(h)
    mean = torch.empty(M, dtype=torch.float32, device=h.device)
    rstd = torch.empty_like(mean)
    _lib.check(lib.ksd8_dspine_ln_fwd(h.data_ptr(), zsum.data_ptr(), inj.data_ptr(),
                                      _lib.dtype_code(h), M, d, w.gate_bias.data_ptr(),
                                      ln_w.data_ptr(), ln_b.data_ptr(), LN_EPS, h2.data_ptr(),
                                      b.data_ptr(), mean.data_ptr(), rstd.data_ptr(), None,
                                      _stream(h)), "dspine_ln_fwd")
    saved = SimpleNamespace(h=h, d1=d1, p=p, u1=u1, u2=u2, zsum=zsum, inj=inj, h2=h2,
                            mean=mean, rstd=rstd, p_first=p_first, w=w, ln_w=ln_w)
    return b, h2, p, saved


def transfer_rows(p: torch.Tensor, e: torch.Tensor):
    """Per-token transfer terms 1 - <normalize(p_t), e_t> (M,) and the (norm, dot)
    rows the backward reuses."""
    M, d = p.shape
    norm = torch.empty(M, dtype=torch.float32, device=p.device)
    dot = torch.empty_like(norm)
    term = torch.empty_like(norm)
    _lib.check(_lib.lib().ksd8_transfer_rows(p.data_ptr(), _lib.dtype_code(p), e.data_ptr(), M, d,
                                             norm.data_ptr(), dot.data_ptr(), term.data_ptr(),
                                             None, _stream(p)), "transfer_rows")
    return term, (norm, dot)


def backward(s: SimpleNamespace, db: torch.Tensor, dres: torch.Tensor, B: int, T: int,
             e: torch.Tensor, e_grad: torch.Tensor, rows, coef: float,
             dp_first_next: torch.Tensor | None, grads: dict, n_parts: int):
    """Backward of forward() and of coef * sum of this layer's transfer terms.

    db (M, d) activation dtype: gradient of b (from the KS3 cell); dres (M, d)
    fp32: gradient reaching h2 through the residual.  e / e_grad: normalised
    transfer targets and their fp32 gradient (accumulated); rows: (norm, dot)
    of transfer_rows(); dp_first_next (B, d) fp32: gradient of this layer's p at
    position 0 from the next layer, or None.  Writes the injection and ln_ffn
    master gradients into `grads` (name -> fp32 tensor).  Returns (dh, dp_first):
    dh (M, d) fp32 the gradient of h, dp_first (B, d) fp32 the gradient of
    p_first (None without one)."""
    M, d = db.shape
    act = db.dtype
    w, r, fr = s.w, s.w.r, s.w.fr
    lib = _lib.lib()
    st = _stream(db)
    dh2 = torch.empty(M, d, dtype=torch.float32, device=db.device)
    dz = torch.empty_like(db)
    dinj = torch.empty_like(db)
    parts = torch.empty(n_parts, 3, d, dtype=torch.float32, device=db.device)
    _lib.check(lib.ksd8_dspine_ln_bwd(s.h2.data_ptr(), s.mean.data_ptr(), s.rstd.data_ptr(),
                                      db.data_ptr(), dres.data_ptr(), s.zsum.data_ptr(),
                                      s.inj.data_ptr(), _lib.dtype_code(db), M, d,
                                      w.gate_bias.data_ptr(), s.ln_w.data_ptr(), dh2.data_ptr(),
                                      dz.data_ptr(), dinj.data_ptr(), parts.data_ptr(), n_parts,
                                      None, st), "dspine_ln_bwd")
    colsum = parts.sum(0)
    grads["ln_w"].copy_(colsum[0])
    grads["ln_b"].copy_(colsum[1])
    grads["gate_bias"].copy_(colsum[2])

    du1 = dz @ w.wu1                                   # (M, 2r): [d gate_q.down out | d shifted P2_p]
    du2 = dinj @ w.wiu                                 # (M, r):  d shifted P2_i
    wu1g = dz.t() @ s.u1                               # (d, 2r)
    grads["gate_q.up"].copy_(wu1g[:, :r])
    grads["gate_p.up"].copy_(wu1g[:, r:])
    grads["inject.up"].copy_(dinj.t() @ s.u2)
    dp2 = torch.empty(M, 2 * r, dtype=act, device=db.device)
    g0p = _unshifted(du1[:, r:], B, T, dp2[:, :r])
    g0i = _unshifted(du2, B, T, dp2[:, r:])
    pgrad = dp2 @ w.wd2                                # (M, d)
    wd2g = dp2.t() @ s.p                               # (2r, d)
    dp_first = None
    if s.p_first is not None:
        g0 = torch.cat([g0p, g0i], 1)                  # (B, 2r)
        dp_first = (g0 @ w.wd2).float()
        wd2g = wd2g + g0.t() @ s.p_first
    grads["gate_p.down"].copy_(wd2g[:r])
    grads["inject.down"].copy_(wd2g[r:])

    dp = torch.empty_like(db)
    norm, dot = rows
    first = None if dp_first_next is None else dp_first_next.contiguous()
    _lib.check(lib.ksd8_transfer_bwd(s.p.data_ptr(), _lib.dtype_code(s.p), e.data_ptr(),
                                     norm.data_ptr(), dot.data_ptr(), M, d, float(coef),
                                     pgrad.data_ptr(), None if first is None else first.data_ptr(),
                                     T, dp.data_ptr(), e_grad.data_ptr(), None, st),
               "transfer_bwd")
    dfd = dp @ w.wfu                                   # (M, fr)
    grads["feature_up"].copy_(dp.t() @ s.d1[:, :fr])
    dd1 = torch.cat([dfd, du1[:, :r]], 1)              # (M, fr + r)
    wd1g = dd1.t() @ s.h                               # (fr + r, d)
    grads["feature_down"].copy_(wd1g[:fr])
    grads["gate_q.down"].copy_(wd1g[fr:])
    dh2 += dd1 @ w.wd1
    return dh2, dp_first
