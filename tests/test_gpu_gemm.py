"""GPU parity of the tcgen05 W8A8 GS128 GEMM.

Per-group int32 partials and the canonical fp32 group sum are bit-exact
against the oracle; the output is within the reference test's tolerance
(rtol 1e-4, atol 1e-3, tests/test_int8.py:80) and 1e-3 relative L2 of the
reference's own CPU tier (golden fixtures).
"""

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def _q(oracle, x):
    c, s = oracle.quantize_last_dim(x)
    return torch.from_numpy(c).cuda(), torch.from_numpy(s).cuda()


def _rel(a, b):
    a, b = np.asarray(a, np.float64), np.asarray(b, np.float64)
    return np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30)


def test_gemm_golden_shapes(golden):
    from ksdraft_b200.kernels.gemm import w8a8_gemm
    g = golden("gemm")
    for i in range(5):
        args = [torch.from_numpy(g[f"s{i}_{k}"]).cuda() for k in ("ac", "as", "wc", "ws")]
        y = w8a8_gemm(*args).cpu().numpy()
        np.testing.assert_allclose(y, g[f"s{i}_y"], rtol=1e-4, atol=1e-3)
        assert _rel(y, g[f"s{i}_y"]) < 1e-3


def test_gemm_config1_vs_reference_and_oracle(golden, oracle):
    from ksdraft_b200.kernels.gemm import w8a8_gemm, w8a8_group_partials
    g = golden("gemm")
    torch.manual_seed(0)
    A = torch.randn(256, 1536).numpy()
    W = (torch.randn(1536, 1536) * 0.02).numpy()
    ac, as_ = oracle.quantize_last_dim(A)
    wc, ws = oracle.quantize_last_dim(W)
    dev = [torch.from_numpy(t).cuda() for t in (ac, as_, wc, ws)]
    y = w8a8_gemm(*dev).cpu().numpy()
    np.testing.assert_allclose(y[:64], g["cfg1_y64"], rtol=1e-4, atol=1e-3)
    y_can, parts = oracle.w8a8_gemm_canonical(ac, as_, wc, ws, with_partials=True)
    np.testing.assert_array_equal(y, y_can)                         # bit-exact
    p = w8a8_group_partials(dev[0], dev[2]).cpu().numpy()
    np.testing.assert_array_equal(p, parts)                          # int32 partials


@pytest.mark.parametrize("M,N,K", [(1, 16, 128), (33, 24, 384), (300, 520, 256),
                                   (128, 256, 1536), (257, 384, 5888), (64, 1536, 512),
                                   (512, 200, 4096)])
def test_gemm_bit_exact_vs_oracle(oracle, M, N, K):
    from ksdraft_b200.kernels.gemm import gemm_out, w8a8_group_partials
    rng = np.random.default_rng(M * 7 + N * 3 + K)
    a = rng.standard_normal((M, K)).astype(np.float32)
    w = (rng.standard_normal((N, K)) * 0.05).astype(np.float32)
    ac, as_ = _q(oracle, a)
    wc, ws = _q(oracle, w)
    y = gemm_out(ac, as_, wc, ws).cpu().numpy()
    y_can, parts = oracle.w8a8_gemm_canonical(ac.cpu().numpy(), as_.cpu().numpy(),
                                              wc.cpu().numpy(), ws.cpu().numpy(),
                                              with_partials=True)
    np.testing.assert_array_equal(y, y_can)
    p = w8a8_group_partials(ac, wc).cpu().numpy()
    np.testing.assert_array_equal(p, parts)
    y_ref = oracle.w8a8_gemm_reference_tier(ac.cpu().numpy(), as_.cpu().numpy(),
                                            wc.cpu().numpy(), ws.cpu().numpy())
    np.testing.assert_allclose(y, y_ref, rtol=1e-4, atol=1e-3)


def test_gemm_extreme_codes(oracle):
    """Full-scale +-127 / -128 codes: int32 dots up to 2^21, exact conversion."""
    from ksdraft_b200.kernels.gemm import gemm_out, w8a8_group_partials
    M, N, K = 128, 128, 512
    a = np.full((M, K), 127, np.int8)
    a[::2] = -128
    w = np.full((N, K), -128, np.int8)
    w[:, ::3] = 127
    sa = np.ones((M, K // 128), np.float16)
    sw = np.full((N, K // 128), 0.5, np.float16)
    t = [torch.from_numpy(x).cuda() for x in (a, sa, w, sw)]
    y = gemm_out(*t).cpu().numpy()
    y_can, parts = oracle.w8a8_gemm_canonical(a, sa, w, sw, with_partials=True)
    np.testing.assert_array_equal(y, y_can)
    np.testing.assert_array_equal(w8a8_group_partials(t[0], t[2]).cpu().numpy(), parts)


@pytest.mark.parametrize("out_dtype", [torch.bfloat16, torch.float16])
def test_gemm_output_dtypes_and_bias(oracle, out_dtype):
    from ksdraft_b200.kernels.gemm import gemm_out
    rng = np.random.default_rng(5)
    M, N, K = 200, 384, 768
    ac, as_ = _q(oracle, rng.standard_normal((M, K)).astype(np.float32))
    wc, ws = _q(oracle, (rng.standard_normal((N, K)) * 0.05).astype(np.float32))
    bias = torch.randn(N).cuda()
    y = gemm_out(ac, as_, wc, ws, out_dtype=out_dtype, bias=bias).cpu()
    y_can = oracle.w8a8_gemm_canonical(ac.cpu().numpy(), as_.cpu().numpy(), wc.cpu().numpy(),
                                       ws.cpu().numpy())
    y_can = torch.from_numpy(y_can) + bias.cpu()
    assert torch.equal(y, y_can.to(out_dtype))


def test_gemm_fp16_saturation_and_nonfinite_flag(oracle):
    from ksdraft_b200.kernels.gemm import gemm_out
    M, N, K = 128, 128, 128
    a = np.full((M, K), 127, np.int8)
    w = np.full((N, K), 127, np.int8)
    sa = np.full((M, 1), 4.0, np.float16)
    sw = np.full((N, 1), 4.0, np.float16)            # 127*127*128*16 = 33M > 65504
    t = [torch.from_numpy(x).cuda() for x in (a, sa, w, sw)]
    y = gemm_out(*t, out_dtype=torch.float16, clamp_f16=True).cpu()
    assert torch.all(y == 65504)
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    y2 = gemm_out(*t, out_dtype=torch.float16, status=status).cpu()
    assert torch.isinf(y2).all() and int(status.item()) == 8


def test_gemm_config2_shapes_sampled_rows(oracle):
    """KS3 layer shapes (M=4096): oracle on 48 sampled rows (row-independence)."""
    from ksdraft_b200.kernels.gemm import gemm_out
    rng = np.random.default_rng(9)
    for (M, N, K) in ((4096, 5888, 1536), (4096, 1536, 5888), (5888, 1536, 4096)):
        ac, as_ = _q(oracle, rng.standard_normal((M, K)).astype(np.float32))
        wc, ws = _q(oracle, (rng.standard_normal((N, K)) * 0.02).astype(np.float32))
        y = gemm_out(ac, as_, wc, ws).cpu().numpy()
        rows = np.sort(rng.choice(M, 48, replace=False))
        rows[-1] = M - 1
        y_can = oracle.w8a8_gemm_canonical(ac.cpu().numpy()[rows], as_.cpu().numpy()[rows],
                                           wc.cpu().numpy(), ws.cpu().numpy())
        np.testing.assert_array_equal(y[rows], y_can)


def test_gemm_reference_errors():
    from ksdraft_b200.kernels.gemm import w8a8_gemm
    a = torch.zeros(4, 256, dtype=torch.int8, device="cuda")
    s = torch.ones(4, 2, dtype=torch.float16, device="cuda")
    with pytest.raises(ValueError, match="K mismatch"):
        w8a8_gemm(a, s, torch.zeros(4, 128, dtype=torch.int8, device="cuda"), s[:, :1])
    with pytest.raises(ValueError, match="scale group mismatch"):
        w8a8_gemm(a, s, a, s[:, :1])
    with pytest.raises(ValueError, match="exceeds"):
        w8a8_gemm(a, s[:, :1], a, s[:, :1])


def test_int8_linear_eval_matches_oracle(oracle):
    from ksdraft_b200.kernels.linear import Int8Linear
    torch.manual_seed(4)
    ref = torch.nn.Linear(256, 128, bias=True)
    lin = Int8Linear.from_float(ref.cuda()).eval()
    x = torch.randn(48, 256, device="cuda")
    with torch.no_grad():
        y = lin(x).cpu().numpy()
    xc, xs = oracle.quantize_last_dim(x.cpu().numpy())
    wc, ws = oracle.quantize_last_dim(ref.weight.detach().cpu().numpy())
    y_o = oracle.w8a8_gemm_canonical(xc, xs, wc, ws) + ref.bias.detach().cpu().numpy()
    np.testing.assert_array_equal(y, y_o.astype(np.float32))
    y_fp = ref(x).detach().cpu().numpy()
    assert _rel(y, y_fp) < 0.05            # tests/test_int8.py:43-55 contract


def test_int8_linear_ste_grads_match_reference(golden):
    """Training forward + backward of Int8Linear (STE, linear.py:75-97) against
    the reference's own CPU run: y, dx (with the scale-gradient term), dW, db."""
    from ksdraft_b200.kernels.linear import Int8Linear
    g = golden("linear")
    for i in range(3):
        w = torch.from_numpy(g[f"c{i}_w"])
        has_b = f"c{i}_b" in g
        lin = Int8Linear(w.shape[1], w.shape[0], bias=has_b).cuda()
        with torch.no_grad():
            lin.weight.copy_(w)
            if has_b:
                lin.bias.copy_(torch.from_numpy(g[f"c{i}_b"]))
        lin.train()
        x = torch.from_numpy(g[f"c{i}_x"]).cuda().requires_grad_(True)
        y = lin(x)
        y.backward(torch.from_numpy(g[f"c{i}_gy"]).cuda())
        assert _rel(y.detach().cpu().numpy(), g[f"c{i}_y"]) < 1e-5
        assert _rel(x.grad.cpu().numpy(), g[f"c{i}_dx"]) < 1e-5, i
        assert _rel(lin.weight.grad.cpu().numpy(), g[f"c{i}_dw"]) < 1e-5
        if has_b:
            assert _rel(lin.bias.grad.cpu().numpy(), g[f"c{i}_db"]) < 1e-5
        lin.eval()
        with torch.no_grad():
            ye = lin(x.detach()).cpu().numpy()
        assert _rel(ye, g[f"c{i}_y_eval"]) < 1e-5    # W8A8 eval vs the reference tier


@pytest.mark.parametrize("M,N,K", [(70, 13, 256), (129, 201, 384), (300, 136, 128)])
@pytest.mark.parametrize("out_dtype", [torch.float32, torch.bfloat16, torch.float16])
def test_gemm_staged_and_direct_output_paths(oracle, M, N, K, out_dtype):
    """Rows whose byte length is not a multiple of 16 take the direct-store
    epilogue, the others the shared-memory staged TMA stores (ragged edges
    clipped); both give the canonical bits in every output dtype."""
    from ksdraft_b200.kernels.gemm import gemm_out
    rng = np.random.default_rng(M + N + K)
    ac, as_ = _q(oracle, rng.standard_normal((M, K)).astype(np.float32))
    wc, ws = _q(oracle, (rng.standard_normal((N, K)) * 0.05).astype(np.float32))
    y = gemm_out(ac, as_, wc, ws, out_dtype=out_dtype).cpu()
    y_can = torch.from_numpy(oracle.w8a8_gemm_canonical(
        ac.cpu().numpy(), as_.cpu().numpy(), wc.cpu().numpy(), ws.cpu().numpy()))
    assert torch.equal(y, y_can.to(out_dtype))
