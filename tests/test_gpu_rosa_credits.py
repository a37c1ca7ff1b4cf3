"""GPU: Rosa counterfactual credits (ksd8_rosa_credits, kernels/rosa_credit_gpu.py)
against the reference's HardRosaGPU (tests/golden/rosa_credits.npz, T <= 63)
and, beyond the reference's 63-position window, against the oracle's brute
force (every bit flipped and the whole stream re-matched)."""

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def _bits(kind, S, T, rng):
    if kind == "fair":
        return rng.integers(0, 2, (S, T)).astype(np.int8)
    if kind == "runs":          # long runs: long matches, the 62-bit cap, long chains
        return (np.cumsum(rng.random((S, T)) < 0.08, 1) % 2).astype(np.int8)
    base = (np.arange(T) % 3 == 0).astype(np.int8)        # periodic: many equal windows
    return (base[None, :] ^ (rng.random((S, T)) < 0.02)).astype(np.int8)


@pytest.mark.parametrize("kind", ["fair", "runs", "periodic"])
@pytest.mark.parametrize("T,max_len", [(1, None), (2, None), (70, None), (150, None),
                                       (300, None), (150, 5), (130, 64)])
def test_credits_match_oracle(oracle, kind, T, max_len):
    from ksdraft_b200.kernels.rosa_credit_gpu import credits
    rng = np.random.default_rng(T * 10 + len(kind) + (max_len or 0))
    S = 3
    q, k, v = (_bits(kind, S, T, rng) for _ in range(3))
    if kind != "fair":
        k[0] = q[0]          # a key stream equal to the query stream: matches at the cap
    grad = rng.standard_normal((S, T)).astype(np.float32)
    cq, ck, cv = oracle.rosa_credits(q, k, v, grad, max_match_len=max_len)
    to = lambda a: torch.from_numpy(a.T.copy()[None]).cuda()       # (1, T, S)  # noqa: E731
    got = credits(to(q), to(k), to(v), torch.from_numpy(grad[None]).cuda(), max_len)
    for g_, r, c in zip(got, (cq, ck, cv), "qkv"):
        g_ = g_[0].cpu().numpy().astype(np.float64)
        err = np.abs(g_ - r).max()
        assert err <= 1e-5 * max(1.0, np.abs(r).max()), (c, err)


@pytest.mark.parametrize("name", ["small", "runs", "mid"])
def test_hard_rosa_matches_reference(golden, name):
    """HardRosaGPU forward and backward against the reference's own (same
    inputs): the hard output bit for bit, the q / k / v / payload gradients
    within fp32 summation order."""
    from ksdraft_b200.kernels.rosa_credit_gpu import HardRosaGPU
    g = golden("rosa_credits")
    leaves = [torch.from_numpy(g[f"{name}_{c}"]).cuda().requires_grad_(True)
              for c in ("q", "k", "v", "payload")]
    y = HardRosaGPU.apply(*leaves)
    assert torch.equal(y.detach().cpu(), torch.from_numpy(g[f"{name}_y"]))
    y.backward(torch.from_numpy(g[f"{name}_gy"]).cuda())
    for leaf, c in zip(leaves, ("gq", "gk", "gv", "gp")):
        ref = torch.from_numpy(g[f"{name}_{c}"])
        got = leaf.grad.cpu()
        err = ((got - ref).abs().max() / ref.abs().max().clamp_min(1e-30)).item()
        assert err < 1e-5, (c, err)


def test_window_guard_and_arguments():
    from ksdraft_b200 import _lib
    from ksdraft_b200.kernels.rosa_credit_gpu import MAX_WINDOW, HardRosaGPU
    q = torch.randn(1, MAX_WINDOW + 1, 2, device="cuda")
    with pytest.raises(ValueError):
        HardRosaGPU.apply(q, q, q, torch.ones(2, device="cuda"))
    lib = _lib.lib()
    assert lib.ksd8_rosa_credits(None, None, None, 1, 4, 65, None, None, None, None, None,
                                 None) == _lib.ERR_ARG
    assert lib.ksd8_rosa_credits(None, None, None, 1, 20000, 62, None, None, None, None, None,
                                 None) == _lib.ERR_UNSUPPORTED
