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
                                 (2, 8300)])   # T >= 8192: the bit-parallel kernel
def test_match_indices_vs_oracle(oracle, S, T):
    from ksdraft_b200.model.rosa import match_payload_sign_with_indices
    rng = np.random.default_rng(S * 1000 + T)
    q, k, v = _streams(rng, S, T)
    s, L, E = match_payload_sign_with_indices(*(torch.from_numpy(a).cuda() for a in (q, k, v)))
    so, Lo, Eo = oracle.rosa_match(q, k, v, method="dp")
    np.testing.assert_array_equal(s.cpu().numpy(), so)
    np.testing.assert_array_equal(L.cpu().numpy(), Lo)
    np.testing.assert_array_equal(E.cpu().numpy(), Eo)


@pytest.fixture
def rosa_algorithm():
    """Select a matcher kernel for one test, restoring the default after it."""
    from ksdraft_b200 import _lib

    def use(algo):
        _lib.check(_lib.lib().ksd8_rosa_set_algorithm(algo), "rosa_set_algorithm")
    yield use
    use(0)


@pytest.mark.parametrize("algo", [0, 1, 2, 3, 4])
@pytest.mark.parametrize("S,T,max_len", [(16, 31, None), (16, 32, None), (16, 97, None),
                                         (40, 700, None), (8, 2048, None), (8, 700, 5),
                                         (8, 700, 12), (8, 700, 13), (5, 3000, 40),
                                         (4, 4157, None), (6, 300, 64), (6, 200, 1)])
def test_match_kernels_agree_with_oracle(oracle, rosa_algorithm, algo, S, T, max_len):
    """Every matcher kernel (chunked prefix tables, per-position prefix tables,
    window scan, sorted keys, bit-parallel) gives the oracle's signs, lengths
    and endpoints, across chunk boundaries, around the 12-level table depth and
    with explicit caps; highly repetitive streams make many prefix collisions
    inside one 32-position chunk."""
    from ksdraft_b200.model.rosa import match_payload_sign_with_indices
    rosa_algorithm(algo)
    rng = np.random.default_rng(S * 7 + T)
    q, k, v = _streams(rng, S, T)
    q[: S // 2] = (np.arange(T) % 3 == 0).astype(np.int8)      # periodic: dense collisions
    k[: S // 2] = (np.arange(T) % 3 == 1).astype(np.int8)
    for i in range(S // 2, S // 2 + S // 4):                   # long runs: long matches below
        q[i] = (np.cumsum(rng.random(T) < 0.05) % 2).astype(np.int8)   # the cap, long chains
        k[i] = (np.cumsum(rng.random(T) < 0.05) % 2).astype(np.int8)
    args = (torch.from_numpy(a).cuda() for a in (q, k, v))
    s, L, E = match_payload_sign_with_indices(*args, max_match_len=max_len)
    so, Lo, Eo = oracle.rosa_match(q, k, v, max_match_len=max_len, method="dp")
    np.testing.assert_array_equal(L.cpu().numpy(), Lo)
    np.testing.assert_array_equal(E.cpu().numpy(), Eo)
    np.testing.assert_array_equal(s.cpu().numpy(), so)


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


def _mixer(d, S, seed):
    from ksdraft_b200.model.rosa import RosaMixer
    torch.manual_seed(seed)
    m = RosaMixer(d, S).cuda()
    with torch.no_grad():
        for n in ("q_proj", "k_proj", "v_proj"):
            getattr(m, n).weight.normal_(0, 0.02)
            getattr(m, n).bias.normal_(0, 0.02)
        m.out_proj.weight.normal_(0, 0.05)
        m.out_proj.bias.normal_(0, 0.05)
        for n in ("time_mix_q", "time_mix_k", "time_mix_v"):
            getattr(m, n).normal_(0, 1.0)
        m.payload.uniform_(0.5, 1.5)
    return m


def test_rosa_mixer_int8_eval_vs_oracle(oracle):
    """The fused W8A8 evaluation forward of RosaMixer after to_int8 (time-shift
    mix + per-token quantisation kernel, q/k/v GEMMs with bias, bit packing,
    match with the payload, out_proj) at B 2, T 1024, 512 streams, d 1536, on
    token-like inputs with repeated spans: bit-exact against the oracle."""
    from ksdraft_b200.kernels.linear import Int8Linear
    B, T, d, S = 2, 1024, 1536, 512
    m = _mixer(d, S, 0)
    for n in ("q_proj", "k_proj", "v_proj", "out_proj"):
        setattr(m, n, Int8Linear.from_float(getattr(m, n)))
    m.eval()
    g = torch.Generator().manual_seed(1)
    emb = torch.randn(4096, d, generator=g)
    ids = torch.randint(0, 4096, (B, T), generator=g)
    ids[:, 600:700] = ids[:, 100:200]                          # repeated spans -> long matches
    x = emb[ids].to(torch.bfloat16)
    with torch.no_grad():
        y = m(x.cuda())
    sig = [torch.sigmoid(getattr(m, f"time_mix_{c}").detach().float()).cpu().numpy()
           for c in "qkv"]
    w = {c: getattr(m, f"{c}_proj").weight.detach().cpu().numpy() for c in "qkv"}
    b = {c: getattr(m, f"{c}_proj").bias.detach().cpu().numpy() for c in "qkv"}
    y_o = oracle.rosa_mixer_int8_eval(x.float().numpy(), *sig, w, b,
                                      m.payload.detach().cpu().numpy(),
                                      m.out_proj.weight.detach().cpu().numpy(),
                                      m.out_proj.bias.detach().cpu().numpy())
    assert y.dtype == torch.bfloat16 and y.shape == (B, T, d)
    np.testing.assert_array_equal(y.float().cpu().numpy(), y_o)


def test_rosa_mixer_training_credits():
    """Training mode takes the reference's CUDA path (rosa.py:141-145): the hard
    core through HardRosaGPU, so the q / k / v projections receive the
    counterfactual credits; equal to autograd of the explicit composition."""
    import copy
    from ksdraft_b200.kernels.rosa_credit_gpu import HardRosaGPU
    B, T, d, S = 2, 200, 256, 128
    m = _mixer(d, S, 3).train()
    ref = copy.deepcopy(m)
    x = torch.randn(B, T, d, device="cuda")
    gy = torch.randn(B, T, d, device="cuda")
    y = m(x)
    y.backward(gy)
    q_in, k_in, v_in = ref._shifted(x)
    hard = HardRosaGPU.apply(ref.q_proj(q_in), ref.k_proj(k_in), ref.v_proj(v_in), ref.payload)
    yr = ref.out_proj(hard.to(x.dtype))
    yr.backward(gy)
    assert torch.equal(y, yr)
    for (n, p_), (_, pr) in zip(m.named_parameters(), ref.named_parameters()):
        assert p_.grad is not None and torch.isfinite(p_.grad).all(), n
        assert torch.equal(p_.grad, pr.grad), n
    assert m.q_proj.weight.grad.abs().sum() > 0          # the credits reach the projections


@pytest.mark.parametrize("dtype,B,T,d", [(torch.float32, 3, 37, 200), (torch.bfloat16, 2, 50, 256),
                                         (torch.bfloat16, 1, 20, 130), (torch.float16, 2, 33, 128)])
def test_timemix_quantize_vs_oracle(oracle, dtype, B, T, d):
    """ksd8_rosa_timemix_quantize (_shifted, rosa.py:128-133, then the GS128
    quantisation of each projection input) against the oracle's row quantiser
    of the same fp32 values: codes and scales bit-exact, across runs of tokens
    that straddle sequence starts and a partial last group."""
    from ksdraft_b200 import _lib
    g = torch.Generator().manual_seed(B * 100 + T + d)
    x = (torch.randn(B, T, d, generator=g) * 3).to(dtype)
    x[0, 5, :7] = 0
    mixes = [torch.sigmoid(torch.randn(d, generator=g)) for _ in range(3)]
    G = (d + 127) // 128
    xd = x.cuda().contiguous()
    codes = [torch.empty(B * T, d, dtype=torch.int8, device="cuda") for _ in range(3)]
    scales = [torch.empty(B * T, G, dtype=torch.float16, device="cuda") for _ in range(3)]
    mdev = [m.cuda().contiguous() for m in mixes]
    _lib.check(_lib.lib().ksd8_rosa_timemix_quantize(
        xd.data_ptr(), _lib.dtype_code(xd), B, T, d, *(m.data_ptr() for m in mdev),
        codes[0].data_ptr(), scales[0].data_ptr(), codes[1].data_ptr(), scales[1].data_ptr(),
        codes[2].data_ptr(), scales[2].data_ptr(), None, _lib.stream_ptr(xd.device)),
        "rosa_timemix_quantize")
    xf = x.float().numpy()
    prev = np.concatenate([np.zeros((B, 1, d), np.float32), xf[:, :-1]], 1)
    diff = torch.from_numpy(xf - prev).to(dtype).float().numpy()     # in x's dtype
    for p in range(3):
        xin = (prev + diff * mixes[p].numpy()).reshape(B * T, d).astype(np.float32)
        co, so = oracle.quantize_rows_c(xin)
        np.testing.assert_array_equal(codes[p].cpu().numpy(), co)
        np.testing.assert_array_equal(scales[p].float().cpu().numpy(), so)
