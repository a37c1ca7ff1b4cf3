"""Pin the CPU oracle against fixtures produced by the reference itself (CPU only).

Bit-exact for integer / byte outputs (codes, scales, LUT, match signs) and for
the fp16-sequence spine given the reference's own inputs; within tolerance
where the reference's fp32 matmul summation order is involved.
"""

import hashlib

import numpy as np
import pytest
import torch


def test_quantize_matches_reference(golden, oracle):
    g = golden("quant")
    names = sorted({k.rsplit("_", 1)[0] for k in g if k.endswith("_x")})
    assert len(names) >= 10
    for name in names:
        x = g[f"{name}_x"]
        c_np, s_np = oracle.quantize_last_dim(x)
        c_c, s_c = oracle.quantize_rows_c(x.reshape(-1, x.shape[-1]))
        np.testing.assert_array_equal(c_np, g[f"{name}_codes"], err_msg=name)
        np.testing.assert_array_equal(s_np.view(np.uint16), g[f"{name}_scales"].view(np.uint16))
        np.testing.assert_array_equal(c_c, g[f"{name}_codes"].reshape(c_c.shape), err_msg=name)
        np.testing.assert_array_equal(s_c.view(np.uint16),
                                      g[f"{name}_scales"].reshape(s_c.shape).view(np.uint16))


def test_dither_formula_matches_reference_given_its_noise(golden, oracle):
    g = golden("dither")
    for i in range(3):
        x, u, d = g[f"c{i}_x"], g[f"c{i}_u"], float(g[f"c{i}_dither"])
        c, s = oracle.quantize_last_dim_dithered(x, d, u)
        np.testing.assert_array_equal(c, g[f"c{i}_codes"])
        np.testing.assert_array_equal(s.view(np.uint16), g[f"c{i}_scales"].view(np.uint16))
        cc, sc = oracle.quantize_rows_c(x, dither=d, u=u)
        np.testing.assert_array_equal(cc, g[f"c{i}_codes"])


def test_dither_zero_is_exact_grid(oracle):
    x = np.random.default_rng(0).standard_normal((8, 256)).astype(np.float32) * 3
    c0, s0 = oracle.quantize_rows_c(x, dither=0.0, seed=5)
    c1, s1 = oracle.quantize_last_dim(x)
    np.testing.assert_array_equal(c0, c1)
    cd, _ = oracle.quantize_rows_c(x, dither=0.5, seed=5)
    changed = (cd != c1).mean()
    assert 0.0 < changed < 0.6   # tests/test_stages.py:36-45 contract


def test_philox_known_answer(oracle):
    # Philox4x32-10 known-answer vectors of Salmon et al. (Random123 kat_vectors):
    # counter = 0, key = 0  -> 6627e8d5 e169c58d bc57ac4c 9b00dbd8
    # counter = ff.., key = ff.. -> 408f276d 41c83b0e a20bc7c6 6d5451fd
    u = oracle.philox_uniform(0, 0, 4)
    words = [0x6627E8D5, 0xE169C58D, 0xBC57AC4C, 0x9B00DBD8]
    np.testing.assert_array_equal(u, np.array([(w >> 8) * 2.0**-24 for w in words], np.float32))


def test_gemm_config1_matches_reference_tier(golden, oracle):
    g = golden("gemm")
    torch.manual_seed(0)
    A = torch.randn(256, 1536).numpy()
    W = (torch.randn(1536, 1536) * 0.02).numpy()
    ac, as_ = oracle.quantize_last_dim(A)
    wc, ws = oracle.quantize_last_dim(W)
    for name, t in (("ac", ac), ("as", as_), ("wc", wc), ("ws", ws)):
        dig = np.frombuffer(hashlib.sha256(np.ascontiguousarray(t).tobytes()).digest(), np.uint8)
        np.testing.assert_array_equal(dig, g[f"cfg1_{name}_sha256"], err_msg=name)
    y_ref_tier = oracle.w8a8_gemm_reference_tier(ac, as_, wc, ws)
    y_can = oracle.w8a8_gemm_canonical(ac, as_, wc, ws)
    for y in (y_ref_tier, y_can):
        np.testing.assert_allclose(y[:64], g["cfg1_y64"], rtol=1e-4, atol=1e-3)
        assert abs(y.astype(np.float64).sum() - g["cfg1_y_sum"]) < 1e-3 * abs(
            g["cfg1_y_sqsum"]) ** 0.5
    rel = np.linalg.norm(y_can[:64] - g["cfg1_y64"]) / np.linalg.norm(g["cfg1_y64"])
    assert rel < 1e-6


def test_gemm_shapes_match_reference_tier(golden, oracle):
    g = golden("gemm")
    for i in range(5):
        ac, as_, wc, ws = g[f"s{i}_ac"], g[f"s{i}_as"], g[f"s{i}_wc"], g[f"s{i}_ws"]
        y = oracle.w8a8_gemm_reference_tier(ac, as_, wc, ws)
        np.testing.assert_allclose(y, g[f"s{i}_y"], rtol=1e-4, atol=1e-3)
        K = ac.shape[1]
        Kp = as_.shape[1] * 128
        acp = np.pad(ac, ((0, 0), (0, Kp - K)))
        wcp = np.pad(wc, ((0, 0), (0, Kp - K)))
        yc, parts = oracle.w8a8_gemm_canonical(acp, as_, wcp, ws, with_partials=True)
        np.testing.assert_allclose(yc, g[f"s{i}_y"], rtol=1e-4, atol=1e-3)
        np.testing.assert_array_equal(parts, oracle.group_partials_numpy(acp, wcp))


def test_tanh_lut_matches_reference(golden, oracle):
    np.testing.assert_array_equal(oracle.make_tanh_lut(), golden("ks3_spine")["lut"])


def test_ks3_pack_matches_reference(golden, oracle):
    g = golden("ks3_spine")
    p = oracle.ks3_pack(g["coefficients"], g["raw_scale"], g["raw_shift"])
    np.testing.assert_array_equal(p["spine_codes"], g["spine_codes"])
    np.testing.assert_array_equal(p["spine_scale"].view(np.uint16),
                                  g["spine_scale"].view(np.uint16))
    for k in ("ws_codes", "wh_codes"):
        np.testing.assert_array_equal(p[k], g[k].reshape(p[k].shape), err_msg=k)
    for k in ("ws_scales", "wh_scales"):
        np.testing.assert_array_equal(p[k].view(np.uint16),
                                      g[k].reshape(p[k].shape).view(np.uint16), err_msg=k)


@pytest.mark.parametrize("mode", ["int8", "fp16", "fp32"])
def test_ks3_spine_matches_reference(golden, oracle, mode):
    g = golden("ks3_spine")
    pack = dict(spine_codes=g["spine_codes"], spine_scale=g["spine_scale"],
                ws_codes=g["ws_codes"], ws_scales=g["ws_scales"], wh_codes=g["wh_codes"],
                wh_scales=g["wh_scales"])
    hq, hs, h = oracle.ks3_spine_quant(g[f"{mode}_coords"], pack, g["lut"], mode, want_h=True)
    if mode == "fp32":
        np.testing.assert_allclose(h, g[f"{mode}_h"], rtol=5e-5, atol=1e-5)
        assert (hq != g[f"{mode}_hq"]).mean() < 1e-3
    else:
        # fp16 mode goes through tanh; int8 mode is integer/fp16 only: bit-exact
        if mode == "int8":
            np.testing.assert_array_equal(h, g[f"{mode}_h"])
            np.testing.assert_array_equal(hq, g[f"{mode}_hq"])
            np.testing.assert_array_equal(hs.view(np.uint16), g[f"{mode}_hs"].view(np.uint16))
        else:
            assert (h != g[f"{mode}_h"]).mean() < 1e-3
            np.testing.assert_allclose(h, g[f"{mode}_h"], rtol=2e-3, atol=1e-3)


def _rel(a, b):
    a, b = np.asarray(a, np.float64), np.asarray(b, np.float64)
    return np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30)


def test_ks3_layer_stages_match_reference(golden, oracle):
    """Each oracle stage fed the reference's own inputs reproduces its outputs."""
    g = golden("ks3_layer")
    xq, xs = oracle.quantize_rows_c(g["x"])
    np.testing.assert_array_equal(xq, g["xq"])
    np.testing.assert_array_equal(xs.view(np.uint16), g["xs"].view(np.uint16))
    dq, ds = oracle.quantize_rows_c(g["down"])
    np.testing.assert_array_equal(dq, g["down_q"])
    uq, us = oracle.quantize_rows_c(g["up"])
    np.testing.assert_array_equal(uq, g["up_q"])
    # spine + requant given the reference's coords: bit-exact
    pack = oracle.ks3_pack(g["coefficients"], g["raw_scale"], g["raw_shift"])
    hq, hs = oracle.ks3_spine_quant(g["coords"], pack, oracle.make_tanh_lut(), "int8")
    np.testing.assert_array_equal(hq, g["hq"])
    np.testing.assert_array_equal(hs.view(np.uint16), g["hs"].view(np.uint16))
    # grad quantisation through fp16 and the requantised up^T: bit-exact
    gq, gs = oracle.quantize_rows_c(g["grad"], round_f16=True)
    np.testing.assert_array_equal(gq, g["gq"])
    upT_q, upT_s = oracle.quantize_rows_c(oracle.dequantize_last_dim(uq, us).T)
    np.testing.assert_array_equal(upT_q, g["upT_q"])
    np.testing.assert_array_equal(upT_s.view(np.uint16), g["upT_s"].view(np.uint16))
    # coordinates / value: the canonical group sum vs the reference's fp32 matmul
    coords = oracle.w8a8_gemm_canonical(xq, xs, dq, ds).astype(np.float16)
    assert (coords != g["coords"]).mean() < 0.02
    assert _rel(coords, g["coords"]) < 1e-3


def test_ks3_layer_end_to_end_within_tolerance(golden, oracle):
    g = golden("ks3_layer")
    r = oracle.ks3_layer(g["x"], g["down"], g["up"], g["coefficients"], g["raw_scale"],
                         g["raw_shift"], g["grad"])
    # y and dx are bf16 in the reference run (the input dtype)
    bf = lambda a: torch.from_numpy(np.asarray(a, np.float32)).to(torch.bfloat16).float().numpy()
    assert _rel(bf(r["y"]), g["y"]) < 1e-3
    r = dict(r, dx=bf(r["dx"]))
    for name in ("dx", "ddown", "dup", "dcoeff", "dscale", "dshift"):
        ref = g[name].reshape(np.asarray(r[name]).shape)
        assert _rel(r[name], ref) < 1e-3, (name, _rel(r[name], ref))


def test_rosa_matches_reference(golden, oracle):
    g = golden("rosa")
    keys = [k[:-5] for k in g if k.endswith("_sign") and not k.startswith("long")]
    for pre in keys:
        q, k, v = g[f"{pre}_q"], g[f"{pre}_k"], g[f"{pre}_v"]
        for method in ("bruteforce", "dp"):
            s, L, E = oracle.rosa_match(q, k, v, method=method)
            np.testing.assert_array_equal(s, g[f"{pre}_sign"], err_msg=f"{pre} {method}")
    q, k, v = g["long_q"], g["long_k"], g["long_v"]
    for method in ("bruteforce", "dp"):
        s, L, E = oracle.rosa_match(q, k, v, method=method)
        np.testing.assert_array_equal(s, g["long_sign"], err_msg=method)
        assert L.max() == 62                     # the reference's cap is exercised
        s5, L5, _ = oracle.rosa_match(q, k, v, max_match_len=5, method=method)
        np.testing.assert_array_equal(s5, g["long_sign_ml5"])
        assert L5.max() == 5


def test_rosa_bruteforce_and_dp_agree_on_indices(oracle):
    rng = np.random.default_rng(3)
    for T in (1, 2, 7, 64, 65, 130):
        q = rng.integers(0, 2, (5, T), dtype=np.int8)
        k = q.copy()
        k[:, T // 2:] = rng.integers(0, 2, (5, T - T // 2), dtype=np.int8)
        v = rng.integers(0, 2, (5, T), dtype=np.int8)
        a = oracle.rosa_match(q, k, v, method="bruteforce")
        b = oracle.rosa_match(q, k, v, method="dp")
        for x, y in zip(a, b):
            np.testing.assert_array_equal(x, y)


def test_rosa_python_definition(oracle):
    rng = np.random.default_rng(11)
    for _ in range(30):
        T = int(rng.integers(2, 16))
        q, k, v = (rng.integers(0, 2, T).tolist() for _ in range(3))
        s, _, _ = oracle.rosa_match(np.array([q]), np.array([k]), np.array([v]))
        assert s[0].tolist() == oracle.rosa_sign_python(q, k, v)


def test_tanh16_table_matches_reference(golden, oracle):
    """The fp16 tanh of the KS3 backward (torch.tanh on fp16, ks3_int8.py:366-367)
    on every non-negative finite fp16 input: the oracle's correctly rounded table
    equals the reference's op bit for bit."""
    ref = golden("tanh16")["bits"]
    np.testing.assert_array_equal(oracle.tanh16_table(ref.size), ref)
    # and the same op on this machine's torch, fp16 and fp16-valued fp32 inputs
    x = torch.from_numpy(np.arange(ref.size, dtype=np.uint16).view(np.float16))
    np.testing.assert_array_equal(torch.tanh(x).numpy().view(np.uint16), ref)
    np.testing.assert_array_equal(torch.tanh(x.float()).half().numpy().view(np.uint16), ref)


def test_vjp_reproduces_reference_dc(golden, oracle):
    """Fed the reference's own value and coordinates, the oracle VJP gives the
    reference's dc (value + dmean, ks3_int8.py:354-402) bit for bit, and both of
    its quantisations (:410, :418)."""
    g = golden("ks3_layer")
    pack = oracle.ks3_pack(g["coefficients"].reshape(-1, 6), g["raw_scale"], g["raw_shift"])
    dc, sums = oracle.ks3_vjp(g["value"], g["coords"], pack)
    np.testing.assert_array_equal(dc.astype(np.float32), g["dc"])
    dcq, dcs = oracle.quantize_rows_c(dc)
    np.testing.assert_array_equal(dcq, g["dcq"])
    np.testing.assert_array_equal(dcs.view(np.uint16), g["dcs"].view(np.uint16))
    dcTq, dcTs = oracle.quantize_rows_c(np.ascontiguousarray(dc.T))
    np.testing.assert_array_equal(dcTq, g["dcT_q"])
    np.testing.assert_array_equal(dcTs.view(np.uint16), g["dcT_s"].view(np.uint16))
    dcoeff, dscale, dshift = oracle.ks3_vjp_finish(sums, g["raw_scale"], g["raw_shift"])
    for got, ref in ((dcoeff, g["dcoeff"]), (dscale, g["dscale"]), (dshift, g["dshift"])):
        got = np.asarray(got, np.float32).reshape(-1)
        assert _rel(got, ref.reshape(-1)) < 1e-3


def test_int8_linear_ste_matches_reference(golden, oracle):
    """Int8Linear STE (linear.py:75-97) restated with the oracle quantiser and an
    fp32 matmul, including the gradient that crosses the input's GS128 scale:
    forward and gradients within fp32 summation-order noise."""
    g = golden("linear")
    for i in range(3):
        b = g.get(f"c{i}_b")
        y, dx, dw, db = oracle.int8_linear_ste(g[f"c{i}_x"], g[f"c{i}_w"], b, g[f"c{i}_gy"])
        assert _rel(y, g[f"c{i}_y"]) < 1e-5
        assert _rel(dx, g[f"c{i}_dx"]) < 1e-5
        assert _rel(dw, g[f"c{i}_dw"]) < 1e-5
        if b is not None:
            assert _rel(db, g[f"c{i}_db"]) < 1e-5
        # without the scale term the input gradient is far off: the term is real
        wq, ws = oracle.quantize_rows_c(g[f"c{i}_w"])
        plain = g[f"c{i}_gy"] @ oracle.dequantize_last_dim(wq, ws)
        assert _rel(plain, g[f"c{i}_dx"]) > 0.1


def _credit_grads(oracle, g, name):
    """q / k / v gradients of HardRosaGPU (rosa_credit_gpu.py:79-112) from the
    oracle's brute-force credits, in the reference's float32 arithmetic."""
    q, k, v = (g[f"{name}_{c}"] for c in "qkv")
    B, T, S = q.shape
    gy, payload = g[f"{name}_gy"], g[f"{name}_payload"]
    bits = [(x > 0).astype(np.int8).transpose(0, 2, 1).reshape(B * S, T) for x in (q, k, v)]
    gs = (gy.transpose(0, 2, 1) * payload[None, :, None]).astype(np.float32).reshape(B * S, T)
    cr = oracle.rosa_credits(*bits, gs)
    out = []
    for c, b, pre in zip(cr, bits, (q, k, v)):
        delta = (c * (1 - 2 * b.astype(np.float64))).astype(np.float32).reshape(B, S, T)
        s = 1.0 / (1.0 + np.exp(-pre.astype(np.float64)))
        out.append(delta.transpose(0, 2, 1) * (s * (1 - s)).astype(np.float32))
    return out


@pytest.mark.parametrize("name", ["small", "runs", "mid"])
def test_rosa_credits_match_reference(golden, oracle, name):
    """The oracle's brute-force counterfactual credits, mapped through the
    Bernoulli factor, give the q / k / v gradients of the reference's own
    HardRosaGPU (tests/golden/rosa_credits.npz, run on the CPU)."""
    g = golden("rosa_credits")
    for got, c in zip(_credit_grads(oracle, g, name), "qkv"):
        ref = g[f"{name}_g{c}"]
        err = np.abs(got - ref).max() / max(np.abs(ref).max(), 1e-30)
        assert err < 1e-5, (name, c, err)
