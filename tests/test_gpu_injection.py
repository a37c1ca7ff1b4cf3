"""GPU: the fused DSpine injection + ln_ffn kernels and the transfer-space rows
(ksdraft_b200/train/injection.py) against a plain PyTorch fp32 autograd
restatement of AdjacentInjection.forward (ksdraft/model/spine.py:56-69), the
block's ln_ffn (block.py:41) and the transfer term (train/__init__.py:80-85)."""

import pytest
import torch
import torch.nn.functional as F

pytestmark = pytest.mark.gpu

FR, R = 64, 32


def _params(d, gen):
    def rn(*shape, std=0.05):
        return (torch.randn(*shape, generator=gen) * std).cuda()
    W = {"feature_down": rn(FR, d), "feature_up": rn(d, FR), "gate_q.down": rn(R, d),
         "gate_q.up": rn(d, R), "gate_p.down": rn(R, d), "gate_p.up": rn(d, R),
         "gate_bias": rn(d, std=0.5), "inject.down": rn(R, d), "inject.up": rn(d, R)}
    ln_w = 1.0 + rn(d, std=0.2)
    ln_b = rn(d, std=0.2)
    return W, ln_w, ln_b


def _reference(h, p_first, W, ln_w, ln_b, e, B, T):
    """fp32 autograd: (b, h2, p, terms)."""
    d = h.shape[-1]
    hv = h.view(B, T, d)
    p = F.linear(F.linear(hv, W["feature_down"]), W["feature_up"])
    p_prev = F.pad(p, (0, 0, 1, 0))[:, :-1, :]
    if p_first is not None:
        p_prev = torch.cat([p_first[:, None, :], p_prev[:, 1:, :]], dim=1)
    gate = torch.sigmoid(F.linear(F.linear(hv, W["gate_q.down"]), W["gate_q.up"])
                         + F.linear(F.linear(p_prev, W["gate_p.down"]), W["gate_p.up"])
                         + W["gate_bias"])
    h2 = hv + gate * F.linear(F.linear(p_prev, W["inject.down"]), W["inject.up"])
    b = F.layer_norm(h2, (d,), ln_w, ln_b, 1e-5)
    fn = F.normalize(p.reshape(-1, d), dim=-1)
    terms = 1 - (fn * e).sum(-1)
    return b.reshape(-1, d), h2.reshape(-1, d), p.reshape(-1, d), terms


def _rel(a, b):
    return float((a.float() - b.float()).norm() / b.float().norm().clamp_min(1e-30))


@pytest.mark.parametrize("act,d,with_first", [(torch.float32, 256, True),
                                              (torch.float32, 128, False),
                                              (torch.bfloat16, 1536, True)])
def test_injection_ln_forward_backward_matches_autograd(act, d, with_first):
    from ksdraft_b200.train import injection
    gen = torch.Generator().manual_seed(d)
    B, T = 2, 96
    M = B * T
    W, ln_w, ln_b = _params(d, gen)
    h = torch.randn(M, d, generator=gen).cuda()
    p_first = torch.randn(B, d, generator=gen).cuda() * 0.1 if with_first else None
    e = F.normalize(torch.randn(M, d, generator=gen).cuda(), dim=-1)
    g_b = torch.randn(M, d, generator=gen).cuda()
    g_res = torch.randn(M, d, generator=gen).cuda()
    g_first = torch.randn(B, d, generator=gen).cuda() * 0.1
    coef = 0.37

    # fp32 autograd reference, on the values the fused path sees in `act`
    hq = h.to(act).float()
    Wq = {k: v.to(act).float() for k, v in W.items()}
    leaves = {k: v.clone().requires_grad_(True) for k, v in Wq.items()}
    lw, lb = ln_w.to(act).float().requires_grad_(True), ln_b.to(act).float().requires_grad_(True)
    hl = hq.clone().requires_grad_(True)
    pfl = None if p_first is None else p_first.to(act).float().requires_grad_(True)
    el = e.clone().requires_grad_(True)
    b_r, h2_r, p_r, t_r = _reference(hl, pfl, leaves, lw, lb, el, B, T)
    loss = ((b_r * g_b.to(act).float()).sum() + (h2_r * g_res).sum() + coef * t_r.sum()
            + (p_r.view(B, T, d)[:, 0] * g_first).sum())
    loss.backward()

    iw = injection.InjectionWeights(W, act)
    b, h2, p, saved = injection.forward(h.to(act), None if p_first is None else
                                        p_first.to(act), iw, ln_w, ln_b, B, T)
    terms, rows = injection.transfer_rows(p, e)
    grads = {n: torch.empty_like(v) for n, v in W.items()}
    grads["ln_w"] = torch.empty_like(ln_w)
    grads["ln_b"] = torch.empty_like(ln_b)
    e_grad = torch.zeros_like(e)
    dh, dpf = injection.backward(saved, g_b.to(act), g_res.clone(), B, T, e, e_grad, rows, coef,
                                 g_first, grads, n_parts=7)
    torch.cuda.synchronize()

    tol = 2e-5 if act == torch.float32 else 2e-2
    for name, got, ref in (("b", b, b_r), ("h2", h2, h2_r), ("p", p, p_r), ("terms", terms, t_r),
                           ("dh", dh, hl.grad), ("e_grad", e_grad, el.grad),
                           ("ln_w", grads["ln_w"], lw.grad), ("ln_b", grads["ln_b"], lb.grad)):
        r = _rel(got, ref.detach())
        print(f"{name}: rel-L2 {r:.2e}")
        assert r < tol, (name, r)
    for n in W:
        r = _rel(grads[n], leaves[n].grad)
        print(f"grad {n}: rel-L2 {r:.2e}")
        assert r < tol, (n, r)
    if p_first is None:
        assert dpf is None
    else:
        r = _rel(dpf, pfl.grad)
        print(f"dp_first: rel-L2 {r:.2e}")
        assert r < tol


def test_injection_rejects_unsupported_width():
    from ksdraft_b200.train import injection
    with pytest.raises(ValueError):
        injection.check_width(96)
    with pytest.raises(ValueError):
        injection.check_width(4096)
