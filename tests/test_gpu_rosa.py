"""GPU parity of the Rosa matcher: signs, match lengths and endpoints bit-exact."""

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def test_match_golden(golden):
    from ksdraft_b200.model.rosa import _match_payload_sign
    g = golden("rosa")
    keys = [k[:-5] for k in g if k.endswith("_sign") and not k.startswith("long")]
    for pre in keys:
        q, k, v = (torch.from_numpy(g[f"{pre}_{n}"]).cuda() for n in "qkv")
        s = _match_payload_sign(q, k, v).cpu().numpy()
        np.testing.assert_array_equal(s, g[f"{pre}_sign"], err_msg=pre)
    q, k, v = (torch.from_numpy(g[f"long_{n}"]).cuda() for n in "qkv")
    np.testing.assert_array_equal(_match_payload_sign(q, k, v).cpu().numpy(), g["long_sign"])
    np.testing.assert_array_equal(_match_payload_sign(q, k, v, max_match_len=5).cpu().numpy(),
                                  g["long_sign_ml5"])


def _streams(rng, S, T, repeat_frac=0.3):
    q = rng.integers(0, 2, (S, T), dtype=np.int8)
    k = q.copy()
    flip = rng.random((S, T)) > repeat_frac
    k[flip] = rng.integers(0, 2, int(flip.sum()), dtype=np.int8)
    # long repeated spans so that matches hit the 62 cap
    for s in range(S):
        if T > 200:
            a = int(rng.integers(0, T // 2))
            L = int(rng.integers(40, 120))
            b = int(rng.integers(a + 1, T - L)) if a + 1 < T - L else a
            k[s, a:a + L] = q[s, b:b + L]
    v = rng.integers(0, 2, (S, T), dtype=np.int8)
    return q, k, v


@pytest.mark.parametrize("S,T", [(8, 1), (8, 2), (16, 33), (16, 64), (16, 65), (12, 300),
                                 (6, 1000), (3, 4096), (64, 2048),
                                 (2, 8300)])   # T >= 8192: the brute-force kernel
def test_match_indices_vs_oracle(oracle, S, T):
    from ksdraft_b200.model.rosa import match_payload_sign_with_indices
    rng = np.random.default_rng(S * 1000 + T)
    q, k, v = _streams(rng, S, T)
    s, L, E = match_payload_sign_with_indices(*(torch.from_numpy(a).cuda() for a in (q, k, v)))
    so, Lo, Eo = oracle.rosa_match(q, k, v, method="dp")
    np.testing.assert_array_equal(s.cpu().numpy(), so)
    np.testing.assert_array_equal(L.cpu().numpy(), Lo)
    np.testing.assert_array_equal(E.cpu().numpy(), Eo)


def test_match_all_zero_and_no_match():
    from ksdraft_b200.model.rosa import _match_payload_sign
    q = torch.tensor([[1, 1, 1]], dtype=torch.int8).cuda()
    k = torch.tensor([[0, 0, 0]], dtype=torch.int8).cuda()
    v = torch.tensor([[1, 1, 1]], dtype=torch.int8).cuda()
    assert _match_payload_sign(q, k, v).cpu().tolist() == [[-1.0, -1.0, -1.0]]
    z = torch.zeros(2, 200, dtype=torch.int8).cuda()
    s = _match_payload_sign(z, z, z).cpu()
    assert s[:, 0].eq(-1).all() and s[:, 1:].eq(-1).all()   # v = 0 everywhere -> -1


def test_match_batched_layout_and_payload(oracle):
    """(B, T, S) projections packed by stride; payload fused into the store."""
    from ksdraft_b200.model.rosa import match_words, pack_bits, _default_max_len
    rng = np.random.default_rng(4)
    B, T, S = 2, 257, 48
    proj = [torch.from_numpy(rng.standard_normal((B, T, S)).astype(np.float32)).cuda()
            for _ in range(3)]
    words = [pack_bits(p, B, T, S, T * S, S, 1) for p in proj]
    pay = torch.from_numpy(rng.uniform(0.5, 2, S).astype(np.float32)).cuda()
    out = torch.empty(B, S, T, dtype=torch.bfloat16, device="cuda")
    match_words(*words, B, S, T, _default_max_len(T, None), payload=pay, out=out,
                strides=(S * T, 1, T))
    bits = [(p > 0).to(torch.int8).permute(0, 2, 1).reshape(B * S, T).cpu().numpy()
            for p in proj]
    so, _, _ = oracle.rosa_match(*bits, method="dp")
    want = (pay.cpu().numpy()[None, :, None] * so.reshape(B, S, T))
    assert torch.equal(out.cpu(), torch.from_numpy(want).to(torch.bfloat16))


def test_rosa_mixer_int8_eval_runs():
    from ksdraft_b200.kernels.linear import Int8Linear
    from ksdraft_b200.model.rosa import RosaMixer
    torch.manual_seed(0)
    m = RosaMixer(256, 128).cuda().eval()
    with torch.no_grad():
        m.out_proj.weight.normal_(0, 0.05)
    for n in ("q_proj", "k_proj", "v_proj", "out_proj"):
        setattr(m, n, Int8Linear.from_float(getattr(m, n)))
    x = torch.randn(2, 96, 256, device="cuda").to(torch.bfloat16)
    with torch.no_grad():
        y = m(x)
    assert y.shape == x.shape and y.dtype == torch.bfloat16 and torch.isfinite(y.float()).all()
