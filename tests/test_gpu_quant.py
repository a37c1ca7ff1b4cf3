"""GPU parity of the GS128 quantisers against the reference fixtures and the oracle."""

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def _bits(a):
    return np.ascontiguousarray(a).view(np.uint16)


def test_quantize_last_dim_golden(golden):
    from ksdraft_b200.kernels.quant import quantize_last_dim
    g = golden("quant")
    names = sorted({k.rsplit("_", 1)[0] for k in g if k.endswith("_x")})
    for name in names:
        x = torch.from_numpy(g[f"{name}_x"])
        if name == "bf16":
            x = x.to(torch.bfloat16)
        elif name == "f16":
            x = x.to(torch.float16)
        c, s = quantize_last_dim(x.cuda())
        np.testing.assert_array_equal(c.cpu().numpy(), g[f"{name}_codes"], err_msg=name)
        np.testing.assert_array_equal(_bits(s.cpu().numpy()), _bits(g[f"{name}_scales"]),
                                      err_msg=name)


@pytest.mark.parametrize("shape", [(1, 1), (3, 127), (5, 129), (33, 1536), (257, 5888),
                                   (2, 3, 300), (0, 128), (4, 0)])
def test_quantize_random_vs_oracle(oracle, shape):
    from ksdraft_b200.kernels.quant import quantize_last_dim
    gen = torch.Generator().manual_seed(sum(shape))
    x = torch.randn(*shape, generator=gen) * torch.rand(*shape[:-1], 1, generator=gen) * 10
    c, s = quantize_last_dim(x.cuda())
    assert c.shape == x.shape and s.shape == (*shape[:-1], (shape[-1] + 127) // 128)
    if x.numel() == 0:
        return
    co, so = oracle.quantize_last_dim(x.numpy())
    np.testing.assert_array_equal(c.cpu().numpy(), co)
    np.testing.assert_array_equal(_bits(s.cpu().numpy()), _bits(so))


def test_quantize_strided_rows(oracle):
    from ksdraft_b200.kernels.quant import quantize_last_dim
    base = torch.randn(64, 512)
    x = base[:, 128:384]            # row stride 512, 16-byte aligned start
    c, s = quantize_last_dim(x.cuda())
    co, so = oracle.quantize_last_dim(x.contiguous().numpy())
    np.testing.assert_array_equal(c.cpu().numpy(), co)
    with pytest.raises(TypeError):
        quantize_last_dim(torch.ones(4, 4, dtype=torch.int32).cuda())


def test_quantize_rejects_cpu_tensors():
    from ksdraft_b200.kernels.quant import quantize_last_dim
    with pytest.raises(RuntimeError, match="CUDA"):
        quantize_last_dim(torch.randn(4, 128))


@pytest.mark.parametrize("dither", [0.25, 0.5, 1.0])
def test_dither_counter_rng_replays(oracle, dither):
    from ksdraft_b200.train.stages import quantize_last_dim_dithered
    x = torch.randn(37, 300) * 3
    seed = 123456789 + int(dither * 100)
    c, s = quantize_last_dim_dithered(x.cuda(), 128, dither, seed=seed, offset=4)
    co, so = oracle.quantize_rows_c(x.numpy(), dither=dither, seed=seed, offset=4)
    np.testing.assert_array_equal(c.cpu().numpy(), co)
    np.testing.assert_array_equal(_bits(s.cpu().numpy()), _bits(so))
    c2, _ = quantize_last_dim_dithered(x.cuda(), 128, dither, seed=seed, offset=4)
    assert torch.equal(c, c2)                       # replayable from the seed
    c0, s0 = quantize_last_dim_dithered(x.cuda(), 128, 0.0)
    ce, se = oracle.quantize_last_dim(x.numpy())
    np.testing.assert_array_equal(c0.cpu().numpy(), ce)   # dither 0 = exact grid
    changed = (c.cpu().numpy() != ce).mean()
    assert 0.0 < changed < 0.6


def test_philox_device_matches_oracle(oracle):
    from ksdraft_b200 import _lib
    out = torch.empty(1000, device="cuda")
    rc = _lib.lib().ksd8_philox_uniform(2024, 7, 1000, out.data_ptr(), _lib.stream_ptr())
    _lib.check(rc, "philox")
    np.testing.assert_array_equal(out.cpu().numpy(), oracle.philox_uniform(2024, 7, 1000))


@pytest.mark.parametrize("R,C", [(128, 64), (300, 70), (4096, 1536), (1, 5), (129, 1)])
def test_quantize_cols_float(oracle, R, C):
    from ksdraft_b200.kernels.quant import quantize_cols
    x = torch.randn(R, C) * 2
    c, s = quantize_cols(x.cuda())
    co, so = oracle.quantize_last_dim(np.ascontiguousarray(x.numpy().T))
    np.testing.assert_array_equal(c.cpu().numpy(), co)
    np.testing.assert_array_equal(_bits(s.cpu().numpy()), _bits(so))


def test_quantize_cols_fp16_rounding_of_bf16(oracle):
    from ksdraft_b200.kernels.quant import quantize_cols
    g = (torch.randn(256, 384) * 1e-2).to(torch.bfloat16)
    c, s = quantize_cols(g.cuda(), round_f16=True)
    g16 = g.float().to(torch.float16).float().numpy()
    co, so = oracle.quantize_last_dim(np.ascontiguousarray(g16.T))
    np.testing.assert_array_equal(c.cpu().numpy(), co)


@pytest.mark.parametrize("R,C", [(1536, 5888), (300, 200), (128, 128)])
def test_quantize_cols_dequant_requant(oracle, R, C):
    """quantize_last_dim(dequantize_last_dim(codes, scales).t()) in one pass."""
    from ksdraft_b200.kernels.quant import quantize_cols, quantize_last_dim
    w = torch.randn(R, C) * 0.02
    wc, ws = quantize_last_dim(w.cuda())
    c, s = quantize_cols(wc, x_scales=ws)
    real = oracle.dequantize_last_dim(wc.cpu().numpy(), ws.cpu().numpy())
    co, so = oracle.quantize_last_dim(np.ascontiguousarray(real.T))
    np.testing.assert_array_equal(c.cpu().numpy(), co)
    np.testing.assert_array_equal(_bits(s.cpu().numpy()), _bits(so))


def _special_rows(R, K, gen):
    """Rows that exercise every branch of the fast code/scale paths: exact
    rounding ties, subnormal fp16 scales, scales clamped at 65504, zero groups."""
    x = torch.randn(R, K, generator=gen) * 3
    s = 2.0 ** -3
    tie = (torch.randint(-126, 126, (K,), generator=gen).float() + 0.5) * s
    tie[::128] = 127 * s                       # amax 127 s: scale s, y = k + 1/2
    x[0] = tie
    if R > 1:
        x[1] = torch.randn(K, generator=gen) * 1e-7     # scale below 2^-14 (fp16 subnormal)
    if R > 2:
        x[2] = torch.randn(K, generator=gen) * 3e7      # amax / 127 above 65504
    if R > 3:
        x[3] = 0.0
    return x


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16, torch.float16])
@pytest.mark.parametrize("R,K", [(1, 128), (7, 384), (33, 1536), (300, 5888)])
def test_staged_rows_kernel_matches_plain_and_oracle(oracle, dtype, R, K):
    """The cp.async.bulk row kernel against the thread-load kernel (bit for
    bit) and the oracle, including ties, tiny and clamped scales."""
    from ksdraft_b200.kernels.quant import quantize_rows_into
    gen = torch.Generator().manual_seed(R * 7 + K)
    x = _special_rows(R, K, gen).to(dtype)
    if dtype == torch.float16:
        x = torch.nan_to_num(x, posinf=60000.0, neginf=-60000.0)
    xc = x.cuda()
    out = []
    for plain in (False, True):
        c = torch.empty(R, K, dtype=torch.int8, device="cuda")
        s = torch.empty(R, K // 128, dtype=torch.float16, device="cuda")
        quantize_rows_into(xc, c, s, plain_loads=plain)
        out.append((c.cpu().numpy(), s.cpu().numpy()))
    np.testing.assert_array_equal(out[0][0], out[1][0])
    np.testing.assert_array_equal(_bits(out[0][1]), _bits(out[1][1]))
    co, so = oracle.quantize_last_dim(x.float().numpy())
    np.testing.assert_array_equal(out[0][0], co)
    np.testing.assert_array_equal(_bits(out[0][1]), _bits(so))


@pytest.mark.parametrize("R,K,dither", [(37, 384, 0.5), (37, 384, 1.0), (64, 256, 0.25),
                                         (5888, 1536, 0.5)])
def test_staged_rows_kernel_dither_and_round_f16(oracle, R, K, dither):
    from ksdraft_b200.kernels.quant import quantize_rows_into
    gen = torch.Generator().manual_seed(R + K)
    x = _special_rows(R, K, gen) * 0.02
    res = {}
    for plain in (False, True):
        for mode in ("dither", "f16"):
            c = torch.empty(R, K, dtype=torch.int8, device="cuda")
            s = torch.empty(R, K // 128, dtype=torch.float16, device="cuda")
            kw = dict(dither=dither, seed=99, offset=12) if mode == "dither" else \
                dict(round_f16=True)
            quantize_rows_into(x.cuda(), c, s, plain_loads=plain, **kw)
            res[plain, mode] = (c.cpu().numpy(), s.cpu().numpy())
    for mode in ("dither", "f16"):
        np.testing.assert_array_equal(res[False, mode][0], res[True, mode][0])
        np.testing.assert_array_equal(_bits(res[False, mode][1]), _bits(res[True, mode][1]))
    if R * K <= 40000:
        co, so = oracle.quantize_rows_c(x.numpy(), dither=dither, seed=99, offset=12)
        np.testing.assert_array_equal(res[False, "dither"][0], co)


def _cols_pair(x, **kw):
    from ksdraft_b200.kernels.quant import quantize_cols
    a = quantize_cols(x, **kw)
    b = quantize_cols(x, plain_loads=True, **kw)
    for u, v in zip(a, b):
        assert torch.equal(u.cpu().view(torch.int8) if u.dtype == torch.int8 else
                           u.cpu().view(torch.int16),
                           v.cpu().view(torch.int8) if v.dtype == torch.int8 else
                           v.cpu().view(torch.int16))
    return a


@pytest.mark.parametrize("R,C", [(1536, 5888), (4096, 1536), (300, 256), (129, 384), (1, 128)])
def test_staged_cols_dequant_matches_plain_and_oracle(oracle, R, C):
    """TMA-staged dequant -> transpose -> requant: ragged row tiles, a single
    row, and rows scaled by 1/2 so that codes fall exactly on ties."""
    from ksdraft_b200.kernels.quant import quantize_last_dim
    gen = torch.Generator().manual_seed(R + C)
    w = torch.randn(R, C, generator=gen) * 0.02
    wc, ws = quantize_last_dim(w.cuda())
    if R >= 4:
        # column requant scale 1 (a 127 in a row of scale 1), odd codes in rows
        # of scale 1/2: every such y = code / 2 is an exact half-integer
        wc[0] = 127
        ws[0] = 1.0
        wc[1::2] = (torch.randint(-63, 64, (len(range(1, R, 2)), C), device="cuda") * 2 + 1
                    ).to(torch.int8)
        ws[1::2] = 0.5
        ws[2] = 2.0 ** -24                    # tiny rows next to large ones
    c, s = _cols_pair(wc, x_scales=ws)
    real = oracle.dequantize_last_dim(wc.cpu().numpy(), ws.cpu().numpy())
    co, so = oracle.quantize_last_dim(np.ascontiguousarray(real.T))
    np.testing.assert_array_equal(c.cpu().numpy(), co)
    np.testing.assert_array_equal(_bits(s.cpu().numpy()), _bits(so))


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16, torch.float16])
@pytest.mark.parametrize("R,C,rf16", [(4096, 1536, True), (200, 1000, True), (257, 132, False),
                                      (128, 64, False)])
def test_staged_cols_float_matches_plain_and_oracle(oracle, dtype, R, C, rf16):
    gen = torch.Generator().manual_seed(R * 3 + C)
    x = _special_rows(C, R, gen).t().contiguous()          # special columns
    x = x.to(dtype)
    if dtype == torch.float16:
        x = torch.nan_to_num(x, posinf=60000.0, neginf=-60000.0)
    c, s = _cols_pair(x.cuda(), round_f16=rf16)
    xf = x.float()
    if rf16:
        xf = xf.to(torch.float16).float()
    co, so = oracle.quantize_last_dim(np.ascontiguousarray(xf.numpy().T))
    np.testing.assert_array_equal(c.cpu().numpy(), co)
    np.testing.assert_array_equal(_bits(s.cpu().numpy()), _bits(so))
