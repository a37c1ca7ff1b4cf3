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
    if mode in ("int8", "fp16"):   # fp16 tanh: correctly rounded, as the reference's
        np.testing.assert_array_equal(hq.cpu().numpy(), g[f"{mode}_hq"])
        np.testing.assert_array_equal(_bits(hs.cpu().numpy()), _bits(g[f"{mode}_hs"]))
    else:   # fp32 tanh: CUDA tanhf vs the CPU's fp32 tanh -> rare one-code differences
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
    from ksdraft_b200.kernels.ks3_int8 import KS3Int8Cell, ks3_weights
    cell = ks3_weights(*(torch.from_numpy(g[k]).cuda() for k in
                         ("down", "up", "coefficients", "raw_scale", "raw_shift")))
    q = KS3Int8Cell(cell, group=128, nonlinear="int8", trainable=True)
    x = torch.from_numpy(g["x"]).to(torch.bfloat16).cuda().requires_grad_(True)
    gout = torch.from_numpy(g["grad"]).to(torch.bfloat16).cuda()
    return g, q, x, gout


def test_ks3_layer_vs_reference_golden(golden):
    """fwd + bwd of the trainable cell vs the reference's own CPU run."""
    g, q, x, gout = _layer_inputs(golden)
    y = q(x)
    y.backward(gout)
    ry = _rel(y.float().detach().cpu().numpy(), g["y"])
    print(f"y rel-L2 vs reference end to end = {ry:.2e}")
    assert ry < 1e-3
    assert y.dtype == torch.bfloat16 and x.grad.dtype == torch.bfloat16
    assert q.master_down.grad is not None and q.master_up.grad is not None
    # 1e-3 relative L2 for every output and gradient
    for name, got, tol in (("dx", x.grad, 1e-3), ("ddown", q.master_down.grad, 1e-3),
                           ("dup", q.master_up.grad, 1e-3),
                           ("dcoeff", q.master_coefficients.grad, 1e-3),
                           ("dscale", q.master_raw_scale.grad, 1e-3),
                           ("dshift", q.master_raw_shift.grad, 1e-3)):
        r = _rel(got.float().cpu().numpy().reshape(-1), g[name].reshape(-1))
        print(f"{name} rel-L2 vs reference end to end = {r:.2e}")
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
    # the VJP's dc codes are exact, so the GEMM outputs are the oracle's bits; the
    # column sums add in another fp32 order (one fp16 ulp at most after rounding)
    dx_o = torch.from_numpy(r["dx"]).to(torch.bfloat16)   # dx is bf16
    assert dx.dtype == torch.bfloat16
    assert torch.equal(dx.cpu(), dx_o)
    np.testing.assert_array_equal(ddown.float().cpu().numpy(),
                                  np.asarray(r["ddown"], np.float16).astype(np.float32))
    np.testing.assert_array_equal(dup.float().cpu().numpy(),
                                  np.asarray(r["dup"], np.float16).astype(np.float32))
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
    np.testing.assert_array_equal(dcq.cpu().numpy(), dcq_o)
    np.testing.assert_array_equal(_bits(dcs.cpu().numpy()), _bits(dcs_o))
    np.testing.assert_array_equal(dctq.cpu().numpy(), dctq_o)
    np.testing.assert_array_equal(_bits(dcts.cpu().numpy()), _bits(dcts_o))
    got = part.sum(0).cpu().numpy()
    assert _rel(got, sums) < 1e-3


def test_device_fp16_tanh_table_exhaustive(golden):
    """The fp16 tanh the KS3 kernels use equals the reference's CPU torch.tanh on
    every non-negative finite fp16 input (ks3_int8.py:366-367)."""
    from ksdraft_b200 import _lib
    ref = golden("tanh16")["bits"]
    out = torch.empty(ref.size, dtype=torch.int16, device="cuda")
    _lib.check(_lib.lib().ksd8_fp16_tanh_table(ref.size, out.data_ptr(), _lib.stream_ptr()),
               "fp16_tanh_table")
    np.testing.assert_array_equal(out.cpu().numpy().view(np.uint16), ref)


def _vjp_dev(value16, coords16, q):
    from ksdraft_b200 import _lib
    M, C = coords16.shape
    nt = (M + 127) // 128
    dcq = torch.empty(M, C, dtype=torch.int8, device="cuda")
    dcs = torch.empty(M, C // 128, dtype=torch.float16, device="cuda")
    dctq = torch.empty(C, M, dtype=torch.int8, device="cuda")
    dcts = torch.empty(C, nt, dtype=torch.float16, device="cuda")
    part = torch.empty(nt, 8, C, device="cuda")
    rc = _lib.lib().ksd8_ks3_vjp(value16.data_ptr(), coords16.data_ptr(), M, C,
                                 q.spine_codes.data_ptr(), q.spine_scale.data_ptr(),
                                 q.warp_scale_codes.data_ptr(), q.warp_scale_scales.data_ptr(),
                                 q.warp_shift_codes.data_ptr(), q.warp_shift_scales.data_ptr(),
                                 dcq.data_ptr(), dcs.data_ptr(), dctq.data_ptr(), dcts.data_ptr(),
                                 part.data_ptr(), None, _lib.stream_ptr())
    _lib.check(rc, "vjp")
    return dcq, dcs, dctq, dcts, part


def test_vjp_on_reference_coords_is_bit_exact(golden):
    """Fed the reference's own value and coordinates (ks3_int8.py:352, :241-242),
    the GPU VJP writes the reference's dc codes and scales, along charts and
    along tokens, bit for bit; the reduced coefficient / warp gradients are
    within 1e-3 (fp32 summation order before the fp16 rounding)."""
    from ksdraft_b200 import _lib
    g, q, x, gout = _layer_inputs(golden)
    q._repack_masters()
    value = torch.from_numpy(g["value"]).cuda()
    coords = torch.from_numpy(g["coords"]).cuda()
    dcq, dcs, dctq, dcts, part = _vjp_dev(value, coords, q)
    np.testing.assert_array_equal(dcq.cpu().numpy(), g["dcq"])
    np.testing.assert_array_equal(_bits(dcs.cpu().numpy()), _bits(g["dcs"]))
    np.testing.assert_array_equal(dctq.cpu().numpy(), g["dcT_q"])
    np.testing.assert_array_equal(_bits(dcts.cpu().numpy()), _bits(g["dcT_s"]))
    C = coords.shape[1]
    outs = [torch.empty(C, 6, dtype=torch.float16, device="cuda"),
            torch.empty(C, dtype=torch.float16, device="cuda"),
            torch.empty(C, dtype=torch.float16, device="cuda")]
    rc = _lib.lib().ksd8_ks3_vjp_reduce(part.data_ptr(), part.shape[0], C,
                                        q.warp_scale_raw.data_ptr(), q.warp_shift_raw.data_ptr(),
                                        *(o.data_ptr() for o in outs), None, _lib.stream_ptr())
    _lib.check(rc, "vjp_reduce")
    for got, name in zip(outs, ("dcoeff", "dscale", "dshift")):
        r = _rel(got.float().cpu().numpy().reshape(-1), g[name].reshape(-1))
        print(f"{name} rel-L2 vs reference (reference coords) = {r:.2e}")
        assert r < 1e-3, (name, r)


def test_layer_downstream_of_reference_coords_within_1e3(golden):
    """Everything after the coordinate GEMM, fed the reference's own intermediate
    codes: the requantised transposes are bit-exact and y, dx, ddown, dup are
    within 1e-3 rel-L2 of the reference's run (ks3_int8.py:326-429)."""
    from ksdraft_b200.kernels.gemm import gemm_out
    from ksdraft_b200.kernels.quant import quantize_cols
    g, q, x, gout = _layer_inputs(golden)
    q._repack_masters()
    dev = "cuda"
    t = {k: torch.from_numpy(np.ascontiguousarray(g[k])).to(dev) for k in g
         if k.endswith(("_q", "_s")) or k in ("hq", "hs", "xq", "xs", "dcq", "dcs")}
    # requantised transposes from the reference's codes: bit-exact
    downT = quantize_cols(q.down_codes, x_scales=q.down_scales)
    np.testing.assert_array_equal(downT[0].cpu().numpy(), g["downT_q"])
    xT = quantize_cols(t["xq"], x_scales=t["xs"])
    np.testing.assert_array_equal(xT[0].cpu().numpy(), g["xT_q"])
    hT = quantize_cols(t["hq"], x_scales=t["hs"])
    np.testing.assert_array_equal(hT[0].cpu().numpy(), g["hT_q"])
    gT = quantize_cols(gout, round_f16=True)
    np.testing.assert_array_equal(gT[0].cpu().numpy(), g["gT_q"])
    y = gemm_out(t["hq"], t["hs"], q.up_codes, q.up_scales, out_dtype=torch.bfloat16)
    dx = gemm_out(t["dcq"], t["dcs"], *downT, out_dtype=torch.bfloat16)
    ddown = gemm_out(t["dcT_q"], t["dcT_s"], *xT, out_dtype=torch.float16)
    dup = gemm_out(t["gT_q"], t["gT_s"], *hT, out_dtype=torch.float16)
    for name, got in (("y", y), ("dx", dx), ("ddown", ddown), ("dup", dup)):
        r = _rel(got.float().cpu().numpy().reshape(-1), g[name].reshape(-1))
        print(f"{name} rel-L2 vs reference (reference codes) = {r:.2e}")
        assert r < 1e-3, (name, r)


def test_project_fused_values(golden, oracle):
    """project_fused (ks3_triton.py:159-195 interface, composed spine semantics)
    writes the oracle's h codes and scales on the GPU's own coordinates, and the
    reference's own codes wherever its coordinates agree."""
    from ksdraft_b200.kernels.gemm import gemm_out
    from ksdraft_b200.kernels.ks3_int8 import make_tanh_lut, pack_small
    from ksdraft_b200.kernels.ks3_triton import project_fused
    from ksdraft_b200.kernels.quant import quantize_last_dim
    g = golden("ks3_layer")
    x = torch.from_numpy(g["x"]).cuda()
    xq, xs = quantize_last_dim(x)
    down_q = torch.from_numpy(g["down_q"]).cuda()
    down_s = torch.from_numpy(g["down_s"]).cuda()
    C = down_q.shape[0]
    sq, ss, wsc, wss, whc, whs = pack_small(torch.from_numpy(g["coefficients"]).cuda(),
                                            torch.from_numpy(g["raw_scale"]).cuda(),
                                            torch.from_numpy(g["raw_shift"]).cuda())
    scale16 = (wsc.float() * wss.float()).reshape(-1).half()
    shift16 = (whc.float() * whs.float()).reshape(-1).half()
    hq, hs = project_fused(xq, xs, down_q, down_s, sq, ss, scale16, shift16,
                           make_tanh_lut("cuda"), 128, "int8")
    assert hq.shape == (x.shape[0], C) and hs.shape == (x.shape[0], (C + 127) // 128)
    coords = gemm_out(xq, xs, down_q, down_s, out_dtype=torch.float16, clamp_f16=True)
    po = oracle.ks3_pack(g["coefficients"].reshape(-1, 6), g["raw_scale"], g["raw_shift"])
    hq_o, hs_o = oracle.ks3_spine_quant(coords.cpu().numpy(), po, oracle.make_tanh_lut(), "int8")
    np.testing.assert_array_equal(hq.cpu().numpy(), hq_o)
    np.testing.assert_array_equal(_bits(hs.cpu().numpy()), _bits(hs_o))
    same_rows = (coords.cpu().numpy().view(np.uint16) == g["coords"].view(np.uint16)).all(1)
    assert same_rows.any()
    np.testing.assert_array_equal(hq.cpu().numpy()[same_rows], g["hq"][same_rows])
    with pytest.raises(ValueError):
        project_fused(xq, xs, down_q, down_s, sq, ss, scale16, shift16,
                      make_tanh_lut("cuda"), 96, "int8")
