"""GPU parity of the fused KS3 cell (pack, spine+requant, VJP, full layer)."""

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def _bits(a):
    return np.ascontiguousarray(a).view(np.uint16)


def _rel(a, b):
    a, b = np.asarray(a, np.float64), np.asarray(b, np.float64)
    return np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30)


def _pack_dev(g):
    return {k: torch.from_numpy(np.ascontiguousarray(g[k])).cuda()
            for k in ("spine_codes", "spine_scale", "ws_codes", "ws_scales", "wh_codes",
                      "wh_scales")}


def test_pack_matches_reference(golden):
    from ksdraft_b200.kernels.ks3_int8 import make_tanh_lut, pack_small
    g = golden("ks3_spine")
    sq, ss, wsc, wss, whc, whs = pack_small(torch.from_numpy(g["coefficients"]).cuda(),
                                            torch.from_numpy(g["raw_scale"]).cuda(),
                                            torch.from_numpy(g["raw_shift"]).cuda())
    np.testing.assert_array_equal(sq.cpu().numpy(), g["spine_codes"])
    np.testing.assert_array_equal(_bits(ss.cpu().numpy()), _bits(g["spine_scale"]))
    np.testing.assert_array_equal(wsc.cpu().numpy().reshape(-1), g["ws_codes"].reshape(-1))
    np.testing.assert_array_equal(whc.cpu().numpy().reshape(-1), g["wh_codes"].reshape(-1))
    np.testing.assert_array_equal(_bits(wss.cpu().numpy()).reshape(-1),
                                  _bits(g["ws_scales"]).reshape(-1))
    np.testing.assert_array_equal(_bits(whs.cpu().numpy()).reshape(-1),
                                  _bits(g["wh_scales"]).reshape(-1))
    np.testing.assert_array_equal(make_tanh_lut("cuda").cpu().numpy(), g["lut"])


@pytest.mark.parametrize("mode", ["int8", "fp16", "fp32"])
def test_spine_quant_matches_reference(golden, mode):
    from ksdraft_b200.kernels.ks3_int8 import spine_quant
    g = golden("ks3_spine")
    p = _pack_dev(g)
    coords = torch.from_numpy(g[f"{mode}_coords"]).cuda()
    lut = torch.from_numpy(g["lut"]).cuda()
    hq, hs = spine_quant(coords, p["spine_codes"], p["spine_scale"], p["ws_codes"],
                         p["ws_scales"], p["wh_codes"], p["wh_scales"], lut, mode)
    if mode == "int8":
        np.testing.assert_array_equal(hq.cpu().numpy(), g[f"{mode}_hq"])
        np.testing.assert_array_equal(_bits(hs.cpu().numpy()), _bits(g[f"{mode}_hs"]))
    else:   # tanh: CUDA tanhf vs the CPU's, rounded -> rare one-code differences
        assert (hq.cpu().numpy() != g[f"{mode}_hq"]).mean() < 2e-3
        assert _rel(hs.cpu().numpy().astype(np.float32), g[f"{mode}_hs"]) < 1e-3


def test_spine_quant_random_vs_oracle(oracle):
    """Large random coordinates (M=4096, C=5888 layer shape) vs the C oracle."""
    from ksdraft_b200.kernels.ks3_int8 import make_tanh_lut, pack_small, spine_quant
    rng = np.random.default_rng(0)
    C, M = 5888, 512
    coeffs = (rng.standard_normal((C, 6)) * 0.3).astype(np.float32)
    rs = rng.uniform(-2, 3, C).astype(np.float32)
    rh = rng.uniform(-2, 2, C).astype(np.float32)
    p = pack_small(*(torch.from_numpy(t).cuda() for t in (coeffs, rs, rh)))
    po = oracle.ks3_pack(coeffs, rs, rh)
    coords = (rng.standard_normal((M, C)) * 5).astype(np.float16)
    lut = make_tanh_lut("cuda")
    hq, hs = spine_quant(torch.from_numpy(coords).cuda(), *p, lut, "int8")
    hq_o, hs_o = oracle.ks3_spine_quant(coords, po, oracle.make_tanh_lut(), "int8")
    np.testing.assert_array_equal(hq.cpu().numpy(), hq_o)
    np.testing.assert_array_equal(_bits(hs.cpu().numpy()), _bits(hs_o))


def test_spine_table_path_equals_generic_path():
    """Table-driven int8 kernel == per-element kernel, incl. zero/tiny/huge h."""
    from ksdraft_b200.kernels.ks3_int8 import (make_tanh_lut, pack_small, spine_quant,
                                               spine_quant_generic)
    rng = np.random.default_rng(7)
    C, M = 1024, 700
    coeffs = (rng.standard_normal((C, 6)) * rng.choice([0.01, 0.3, 3.0], (C, 1))).astype(
        np.float32)
    rs = rng.uniform(-3, 4, C).astype(np.float32)
    rh = rng.uniform(-3, 3, C).astype(np.float32)
    p = pack_small(*(torch.from_numpy(t).cuda() for t in (coeffs, rs, rh)))
    scale = rng.choice([1e-4, 1e-2, 1.0, 30.0, 3000.0], (M, 1))
    coords = (rng.standard_normal((M, C)) * scale).astype(np.float16)
    coords[:8] = 0
    coords[8:16, :64] = np.float16(65504)
    coords[16:24, :64] = np.float16(-65504)
    coords[24:32] = np.float16(6e-8)
    cd = torch.from_numpy(coords).cuda()
    lut = make_tanh_lut("cuda")
    hq_f, hs_f = spine_quant(cd, *p, lut, "int8")
    hq_g, hs_g = spine_quant_generic(cd, *p, lut, "int8")
    assert torch.equal(hq_f, hq_g)
    assert torch.equal(hs_f.view(torch.int16), hs_g.view(torch.int16))


def _layer_inputs(golden):
    g = golden("ks3_layer")
    from ksdraft_b200.kernels.ks3_int8 import KS3Int8Cell
    from ksdraft_b200.model.ks3 import KS3
    d, C = g["down"].shape[1], g["down"].shape[0]
    cell = KS3(d, C)
    with torch.no_grad():
        cell.down.weight.copy_(torch.from_numpy(g["down"]))
        cell.up.weight.copy_(torch.from_numpy(g["up"]))
        cell.coefficients.copy_(torch.from_numpy(g["coefficients"]).reshape(C, 6))
        cell.raw_scale.copy_(torch.from_numpy(g["raw_scale"]))
        cell.raw_shift.copy_(torch.from_numpy(g["raw_shift"]))
    q = KS3Int8Cell(cell.cuda(), group=128, nonlinear="int8", trainable=True)
    x = torch.from_numpy(g["x"]).to(torch.bfloat16).cuda().requires_grad_(True)
    gout = torch.from_numpy(g["grad"]).to(torch.bfloat16).cuda()
    return g, q, x, gout


def test_ks3_layer_vs_reference_golden(golden):
    """fwd + bwd of the trainable cell vs the reference's own CPU run."""
    g, q, x, gout = _layer_inputs(golden)
    y = q(x)
    y.backward(gout)
    assert _rel(y.float().detach().cpu().numpy(), g["y"]) < 1e-2
    assert y.dtype == torch.bfloat16 and x.grad.dtype == torch.bfloat16
    assert q.master_down.grad is not None and q.master_up.grad is not None
    for name, got, tol in (("dx", x.grad, 5e-2), ("ddown", q.master_down.grad, 5e-2),
                           ("dup", q.master_up.grad, 5e-2),
                           ("dcoeff", q.master_coefficients.grad, 5e-2),
                           ("dscale", q.master_raw_scale.grad, 5e-2),
                           ("dshift", q.master_raw_shift.grad, 5e-2)):
        r = _rel(got.float().cpu().numpy().reshape(-1), g[name].reshape(-1))
        assert r < tol, (name, r)


def test_ks3_layer_stages_bit_exact_vs_oracle(golden, oracle):
    """Every stage of the GPU layer against the oracle pipeline on the same inputs."""
    from ksdraft_b200.kernels.ks3_int8 import _KS3Int8Train, ks3_backward
    from ksdraft_b200.kernels.quant import quantize_last_dim
    g, q, x, gout = _layer_inputs(golden)
    r = oracle.ks3_layer(x.detach().float().cpu().numpy(), g["down"], g["up"],
                         g["coefficients"], g["raw_scale"], g["raw_shift"],
                         gout.float().cpu().numpy())
    q._repack_masters()
    xq, xs = quantize_last_dim(x.detach().reshape(-1, x.shape[-1]))
    hq, hs, coords = q._project(xq, xs)
    np.testing.assert_array_equal(xq.cpu().numpy(), r["xq"])
    np.testing.assert_array_equal(_bits(coords.cpu().numpy()), _bits(r["coords"]))
    np.testing.assert_array_equal(hq.cpu().numpy(), r["hq"])
    np.testing.assert_array_equal(_bits(hs.cpu().numpy()), _bits(r["hs"]))
    y = _KS3Int8Train.apply(x, q.master_down, q.master_up, q.master_coefficients,
                            q.master_raw_scale, q.master_raw_shift, q)
    y_o = torch.from_numpy(r["y"]).to(torch.bfloat16)
    assert torch.equal(y.detach().cpu(), y_o)
    dx, ddown, dup, dcoeff, dscale, dshift, _ = ks3_backward(q, gout, xq, xs, hq, hs, coords,
                                                             x.shape)
    # through the VJP, tanhf (CUDA vs glibc) may move an fp16 rounding: tolerance
    dx_o = torch.from_numpy(r["dx"]).to(torch.bfloat16).float().numpy()   # dx is bf16
    assert dx.dtype == torch.bfloat16
    assert _rel(dx.float().cpu().numpy(), dx_o) < 1e-3
    assert _rel(ddown.float().cpu().numpy(), r["ddown"]) < 1e-3
    assert _rel(dup.float().cpu().numpy(), r["dup"]) < 1e-3
    assert _rel(dcoeff.float().cpu().numpy().reshape(-1, 6), r["dcoeff"].astype(np.float32)) \
        < 1e-3
    assert _rel(dscale.float().cpu().numpy(), r["dscale"].astype(np.float32)) < 1e-3
    assert _rel(dshift.float().cpu().numpy(), r["dshift"].astype(np.float32)) < 1e-3


def test_vjp_kernel_vs_oracle(oracle):
    """VJP on random value/coords: dc codes (both quantisations) and column sums."""
    from ksdraft_b200 import _lib
    from ksdraft_b200.kernels.ks3_int8 import pack_small
    rng = np.random.default_rng(1)
    M, C = 300, 384
    coeffs = (rng.standard_normal((C, 6)) * 0.05).astype(np.float32)
    rs = np.full(C, 0.75, np.float32)
    rh = rng.uniform(-1, 1, C).astype(np.float32)
    p = pack_small(*(torch.from_numpy(t).cuda() for t in (coeffs, rs, rh)))
    po = oracle.ks3_pack(coeffs, rs, rh)
    value = (rng.standard_normal((M, C)) * 1e-2).astype(np.float16)
    coords = (rng.standard_normal((M, C)) * 2).astype(np.float16)
    v_d, c_d = torch.from_numpy(value).cuda(), torch.from_numpy(coords).cuda()
    nt = (M + 127) // 128
    dcq = torch.empty(M, C, dtype=torch.int8, device="cuda")
    dcs = torch.empty(M, C // 128, dtype=torch.float16, device="cuda")
    dctq = torch.empty(C, M, dtype=torch.int8, device="cuda")
    dcts = torch.empty(C, nt, dtype=torch.float16, device="cuda")
    part = torch.empty(nt, 8, C, device="cuda")
    rc = _lib.lib().ksd8_ks3_vjp(v_d.data_ptr(), c_d.data_ptr(), M, C, p[0].data_ptr(),
                                 p[1].data_ptr(), p[2].data_ptr(), p[3].data_ptr(),
                                 p[4].data_ptr(), p[5].data_ptr(), dcq.data_ptr(),
                                 dcs.data_ptr(), dctq.data_ptr(), dcts.data_ptr(),
                                 part.data_ptr(), None, _lib.stream_ptr())
    _lib.check(rc, "vjp")
    dc, sums = oracle.ks3_vjp(value, coords, po)
    dcq_o, dcs_o = oracle.quantize_rows_c(dc)
    dctq_o, dcts_o = oracle.quantize_rows_c(np.ascontiguousarray(dc.T))
    assert (dcq.cpu().numpy() != dcq_o).mean() < 1e-3
    assert (dctq.cpu().numpy() != dctq_o).mean() < 1e-3
    got = part.sum(0).cpu().numpy()
    assert _rel(got, sums) < 1e-3


def test_project_fused_interface(golden):
    from ksdraft_b200.kernels.ks3_int8 import make_tanh_lut
    from ksdraft_b200.kernels.ks3_triton import project_fused
    from ksdraft_b200.kernels.quant import quantize_last_dim
    g = golden("ks3_layer")
    x = torch.from_numpy(g["x"]).cuda()
    xq, xs = quantize_last_dim(x)
    down_q = torch.from_numpy(g["down_q"]).cuda()
    down_s = torch.from_numpy(g["down_s"]).cuda()
    C = down_q.shape[0]
    from ksdraft_b200.kernels.ks3_int8 import pack_small
    sq, ss, wsc, wss, whc, whs = pack_small(torch.from_numpy(g["coefficients"]).cuda(),
                                            torch.from_numpy(g["raw_scale"]).cuda(),
                                            torch.from_numpy(g["raw_shift"]).cuda())
    scale16 = (wsc.float() * wss.float()).reshape(-1).half()
    shift16 = (whc.float() * whs.float()).reshape(-1).half()
    hq, hs = project_fused(xq, xs, down_q, down_s, sq, ss, scale16, shift16,
                           make_tanh_lut("cuda"), 128, "int8")
    assert hq.shape == (x.shape[0], C) and hs.shape == (x.shape[0], (C + 127) // 128)
    with pytest.raises(ValueError):
        project_fused(xq, xs, down_q, down_s, sq, ss, scale16, shift16,
                      make_tanh_lut("cuda"), 96, "int8")
