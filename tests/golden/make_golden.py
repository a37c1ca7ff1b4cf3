"""Generate the golden fixtures of tests/golden/ by running the REFERENCE itself.

    python tests/golden/make_golden.py --ref /path/to/ksdraft-checkout [--only TOPIC ...]

Imports the reference package (curvedinf/ksdraft) read-only and runs its own
CPU tier on seeded inputs; writes one compressed .npz per topic.  Only this
container has the reference checkout, so the fixtures are committed and the
GPU box never needs the reference at run time.
"""

from __future__ import annotations

import argparse
import os
import sys
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent


def f16(t):
    return t.detach().cpu().to(torch.float16).numpy()


def f32(t):
    return t.detach().cpu().float().numpy()


def i8(t):
    return t.detach().cpu().to(torch.int8).numpy()


def save(name, **arrays):
    np.savez_compressed(HERE / f"{name}.npz", **arrays)
    print(f"wrote {name}.npz ({(HERE / f'{name}.npz').stat().st_size / 1e6:.2f} MB)")


def gen_quant():
    from ksdraft.kernels.quant import quantize_last_dim
    g = torch.Generator().manual_seed(0)
    cases = {
        "randn3": torch.randn(64, 256, generator=g) * 3,
        "partial": torch.randn(4, 100, generator=g),
        "partial2": torch.randn(7, 300, generator=g) * 0.1,
        "zeros": torch.zeros(2, 128),
        "tiny": torch.randn(3, 256, generator=g) * 1e-9,
        "huge": torch.randn(3, 256, generator=g) * 1e7,
        "mixed": torch.cat([torch.randn(5, 128, generator=g) * 10 ** e for e in range(-4, 5)]),
        "ties": (torch.randint(-254, 255, (16, 128), generator=g).float() * 0.5),
    }
    out = {}
    for name, x in cases.items():
        c, s = quantize_last_dim(x)
        out[f"{name}_x"] = f32(x)
        out[f"{name}_codes"] = i8(c)
        out[f"{name}_scales"] = f16(s)
    xb = (torch.randn(9, 384, generator=g) * 2).to(torch.bfloat16)
    c, s = quantize_last_dim(xb)
    out["bf16_x"] = f32(xb)
    out["bf16_codes"], out["bf16_scales"] = i8(c), f16(s)
    xh = (torch.randn(9, 384, generator=g) * 2).to(torch.float16)
    c, s = quantize_last_dim(xh)
    out["f16_x"] = f32(xh)
    out["f16_codes"], out["f16_scales"] = i8(c), f16(s)
    save("quant", **out)


def gen_dither():
    from ksdraft.train.stages import quantize_last_dim_dithered
    out = {}
    for i, (shape, dither) in enumerate((((8, 256), 0.5), ((5, 300), 0.25), ((4, 128), 1.0))):
        x = torch.randn(*shape, generator=torch.Generator().manual_seed(10 + i)) * 3
        Kp = (shape[1] + 127) // 128 * 128
        u = torch.rand((shape[0], Kp // 128, 128), generator=torch.Generator().manual_seed(99 + i))
        c, s = quantize_last_dim_dithered(x, 128, dither,
                                          generator=torch.Generator().manual_seed(99 + i))
        out[f"c{i}_x"], out[f"c{i}_u"] = f32(x), f32(u.reshape(shape[0], Kp))
        out[f"c{i}_codes"], out[f"c{i}_scales"] = i8(c), f16(s)
        out[f"c{i}_dither"] = np.float32(dither)
    save("dither", **out)


def gen_gemm():
    from ksdraft.kernels.gemm import w8a8_gemm
    from ksdraft.kernels.quant import quantize_last_dim
    out = {}
    # benchmark config 1: seed 0, A ~ N(0,1) [256,1536], W ~ N(0,0.02) [1536,1536]
    torch.manual_seed(0)
    A = torch.randn(256, 1536)
    W = torch.randn(1536, 1536) * 0.02
    ac, as_ = quantize_last_dim(A)
    wc, ws = quantize_last_dim(W)
    y = w8a8_gemm(ac, as_, wc, ws)
    # inputs are regenerated from the seed by the tests (torch CPU RNG); the
    # fixture keeps digests of the reference's codes/scales and 64 output rows
    import hashlib
    for name, t in (("ac", i8(ac)), ("as", f16(as_)), ("wc", i8(wc)), ("ws", f16(ws))):
        out[f"cfg1_{name}_sha256"] = np.frombuffer(
            hashlib.sha256(np.ascontiguousarray(t).tobytes()).digest(), np.uint8)
    out.update(cfg1_y64=f32(y[:64]), cfg1_y_sum=np.float64(y.double().sum()),
               cfg1_y_sqsum=np.float64(y.double().square().sum()))
    # shapes of tests/test_int8.py:73 (incl. partial groups via padding)
    g = torch.Generator().manual_seed(3)
    for i, (M, K, N) in enumerate(((16, 256, 128), (64, 128, 96), (33, 384, 64), (128, 128, 128),
                                   (5, 200, 24))):
        a = torch.randn(M, K, generator=g)
        w = torch.randn(N, K, generator=g) * 0.1
        ac, as_ = quantize_last_dim(a)
        wc, ws = quantize_last_dim(w)
        y = w8a8_gemm(ac, as_, wc, ws)
        out.update({f"s{i}_ac": i8(ac), f"s{i}_as": f16(as_), f"s{i}_wc": i8(wc),
                    f"s{i}_ws": f16(ws), f"s{i}_y": f32(y)})
    save("gemm", **out)


def gen_ks3():
    from ksdraft.kernels.ks3_int8 import KS3Int8Cell, make_tanh_lut, pack_spine
    from ksdraft.kernels.quant import quantize_last_dim
    from ksdraft.model.ks3 import KS3
    out = {"lut": i8(make_tanh_lut("cpu"))}
    torch.manual_seed(0)
    cell = KS3(128, 256)
    with torch.no_grad():
        cell.coefficients.normal_(0, 0.3)
        cell.raw_scale.uniform_(-2.0, 3.0)
        cell.raw_shift.uniform_(-2.0, 2.0)
        cell.raw_scale[:4] = torch.tensor([25.0, -30.0, 0.0, 20.0])
    # pack: spine rows + warp scalars
    sq, ss = pack_spine(cell.coefficients.detach().float())
    out.update(coefficients=f32(cell.coefficients), raw_scale=f32(cell.raw_scale),
               raw_shift=f32(cell.raw_shift), spine_codes=i8(sq), spine_scale=f16(ss))
    for mode in ("int8", "fp16", "fp32"):
        q = KS3Int8Cell(cell, group=128, nonlinear=mode)
        if mode == "int8":
            out.update(ws_codes=i8(q.warp_scale_codes), ws_scales=f16(q.warp_scale_scales),
                       wh_codes=i8(q.warp_shift_codes), wh_scales=f16(q.warp_shift_scales))
        # coordinates: random fp16 over the LUT range and beyond, plus edge values
        gen = torch.Generator().manual_seed(5)
        M = 96
        coords = (torch.randn(M, 256, generator=gen) * 6).to(torch.float16)
        edge = torch.tensor([0.0, -0.0, 3.2, -3.2, 12.8, -12.8, 12.796875, 65504.0, -65504.0,
                             1e-5, -1e-5, 6e-8, 0.25, 0.5, 1.0, 127.0], dtype=torch.float16)
        coords[:16, :16] = edge[None, :].expand(16, 16)
        coords[16:32, :16] = edge[:, None].expand(16, 16)
        x = coords.float().reshape(M, 256, 1)
        c_all = q.spine_codes.reshape(256, 6)
        cs = [c_all[:, i].reshape(256, 1) for i in range(6)]
        ps = q.spine_scale.reshape(256)
        arith = torch.float32 if mode == "fp32" else torch.float16
        scale, shift = q._warp_scalars(arith)
        h = q._spine_features(x, x, *cs, ps, scale, shift).reshape(M, 256)
        hq, hs = quantize_last_dim(h)
        out.update({f"{mode}_coords": f16(coords), f"{mode}_h": f32(h), f"{mode}_hq": i8(hq),
                    f"{mode}_hs": f16(hs)})
    save("ks3_spine", **out)


def gen_ks3_layer():
    """_KS3Int8Train fwd+bwd (the reference's composed CPU path), small shape."""
    from ksdraft.kernels.gemm import w8a8_gemm
    from ksdraft.kernels.ks3_int8 import KS3Int8Cell
    from ksdraft.kernels.quant import dequantize_last_dim, quantize_last_dim
    from ksdraft.model.ks3 import KS3
    torch.manual_seed(1)
    d, C, M = 256, 384, 256
    cell = KS3(d, C)
    with torch.no_grad():
        cell.down.weight.normal_(0, 0.02)
        cell.up.weight.normal_(0, 0.02)
    q = KS3Int8Cell(cell, group=128, nonlinear="int8", trainable=True)
    x = torch.randn(M, d).to(torch.bfloat16).requires_grad_(True)
    gout = (torch.randn(M, d) * 1e-2).to(torch.bfloat16)
    y = q(x)
    # record the backward's own intermediates (ks3_int8.py:345-424) by wrapping
    # the module-level quantiser and GEMM it calls, in call order
    import ksdraft.kernels.ks3_int8 as K
    rec_q, rec_g = [], []
    orig_q, orig_g = K.quantize_last_dim, K.w8a8_gemm

    def q_rec(t, group=128):
        r = orig_q(t, group)
        rec_q.append((t.detach().clone(), r))
        return r

    def g_rec(*a):
        r = orig_g(*a)
        rec_g.append(r.detach().clone())
        return r
    K.quantize_last_dim, K.w8a8_gemm = q_rec, g_rec
    try:
        y.backward(gout)
    finally:
        K.quantize_last_dim, K.w8a8_gemm = orig_q, orig_g
    # quantiser calls: g, up^T, dc, down^T, dc^T, x^T, g^T, h^T; GEMMs: value, dx, ddown, dup
    assert len(rec_q) == 8 and len(rec_g) == 4, (len(rec_q), len(rec_g))
    dc = rec_q[2][0]
    bwd = dict(dc=f32(dc), dcq=i8(rec_q[2][1][0]), dcs=f16(rec_q[2][1][1]),
               downT_q=i8(rec_q[3][1][0]), downT_s=f16(rec_q[3][1][1]),
               dcT_q=i8(rec_q[4][1][0]), dcT_s=f16(rec_q[4][1][1]),
               xT_q=i8(rec_q[5][1][0]), xT_s=f16(rec_q[5][1][1]),
               gT_q=i8(rec_q[6][1][0]), gT_s=f16(rec_q[6][1][1]),
               hT_q=i8(rec_q[7][1][0]), hT_s=f16(rec_q[7][1][1]),
               value_bwd=f16(rec_g[0]), dx32=f32(rec_g[1]), ddown32=f32(rec_g[2]),
               dup32=f32(rec_g[3]))
    out = dict(**bwd, x=f32(x), grad=f32(gout), down=f32(q.master_down), up=f32(q.master_up),
               coefficients=f32(q.master_coefficients), raw_scale=f32(q.master_raw_scale),
               raw_shift=f32(q.master_raw_shift), y=f32(y), dx=f32(x.grad),
               ddown=f32(q.master_down.grad), dup=f32(q.master_up.grad),
               dcoeff=f32(q.master_coefficients.grad), dscale=f32(q.master_raw_scale.grad),
               dshift=f32(q.master_raw_shift.grad))
    # intermediates, recomputed with the reference's own functions (ks3_int8.py:326-424)
    with torch.no_grad():
        xq, xs = quantize_last_dim(x.detach().float())
        coords = w8a8_gemm(xq, xs, q.down_codes, q.down_scales).to(torch.float16) \
            .clamp(-65504.0, 65504.0)
        hfeat, _ = q._project(xq, xq, xs, q.down_codes, q.down_scales)
        hq, hs = quantize_last_dim(hfeat)
        g16 = gout.float().to(torch.float16)
        gq, gs = quantize_last_dim(g16.float())
        upT = quantize_last_dim(dequantize_last_dim(q.up_codes, q.up_scales).t().contiguous())
        value = w8a8_gemm(gq, gs, *upT).to(torch.float16)
    out.update(xq=i8(xq), xs=f16(xs), coords=f16(coords), hq=i8(hq), hs=f16(hs), gq=i8(gq),
               gs=f16(gs), upT_q=i8(upT[0]), upT_s=f16(upT[1]), value=f16(value),
               down_q=i8(q.down_codes), down_s=f16(q.down_scales), up_q=i8(q.up_codes),
               up_s=f16(q.up_scales))
    save("ks3_layer", **out)


def gen_rosa():
    from ksdraft.model.rosa import _match_payload_sign
    out = {}
    g = torch.Generator().manual_seed(7)
    # random short streams (tests/test_rosa.py:39-49 regime) batched by length
    for T in (1, 2, 3, 5, 9, 16):
        q = torch.randint(0, 2, (24, T), generator=g, dtype=torch.int8)
        k = torch.randint(0, 2, (24, T), generator=g, dtype=torch.int8)
        v = torch.randint(0, 2, (24, T), generator=g, dtype=torch.int8)
        s = _match_payload_sign(q, k, v)
        out.update({f"T{T}_q": i8(q), f"T{T}_k": i8(k), f"T{T}_v": i8(v), f"T{T}_sign": f32(s)})
    # long streams with repeated spans: matches longer than the 62-bit cap
    T, S = 160, 6
    q = torch.randint(0, 2, (S, T), generator=g, dtype=torch.int8)
    k = q.clone()
    k[:, 100:] = torch.randint(0, 2, (S, 60), generator=g, dtype=torch.int8)
    k[1] = torch.randint(0, 2, (T,), generator=g, dtype=torch.int8)
    k[2, :80] = q[2, 80:]
    q[3] = 0
    k[3] = 0
    v = torch.randint(0, 2, (S, T), generator=g, dtype=torch.int8)
    chunks = [_match_payload_sign(q[i:i + 1], k[i:i + 1], v[i:i + 1]) for i in range(S)]
    out.update(long_q=i8(q), long_k=i8(k), long_v=i8(v), long_sign=f32(torch.cat(chunks)))
    # explicit max_match_len
    s5 = torch.cat([_match_payload_sign(q[i:i + 1], k[i:i + 1], v[i:i + 1], max_match_len=5)
                    for i in range(S)])
    out.update(long_sign_ml5=f32(s5))
    # hand case of tests/test_rosa.py:25-36
    out.update(hand_q=np.array([[0, 1, 1, 1]], np.int8), hand_k=np.array([[1, 0, 1, 1]], np.int8),
               hand_v=np.array([[1, 0, 0, 1]], np.int8),
               hand_sign=np.array([[-1.0, -1.0, -1.0, 1.0]], np.float32))
    save("rosa", **out)


def gen_tanh16():
    """torch.tanh on every non-negative finite fp16 value (the op of
    ks3_int8.py:366-367), as uint16 bits."""
    bits = torch.arange(0, 0x7C00, dtype=torch.int32).to(torch.int16)
    t = torch.tanh(bits.view(torch.float16))
    save("tanh16", bits=t.view(torch.int16).numpy().view(np.uint16))


def gen_linear():
    """Int8Linear STE training forward/backward (linear.py:75-97) and the eval W8A8
    forward (:62-73), small shapes, on the reference's CPU tier."""
    from ksdraft.kernels.linear import Int8Linear
    out = {}
    g = torch.Generator().manual_seed(21)
    for i, (M, K, N, bias) in enumerate(((64, 256, 96, True), (37, 300, 128, False),
                                         (128, 512, 200, True))):
        lin = Int8Linear(K, N, bias=bias)
        with torch.no_grad():
            lin.weight.copy_(torch.randn(N, K, generator=g) * 0.05)
            if bias:
                lin.bias.copy_(torch.randn(N, generator=g) * 0.1)
        x = (torch.randn(M, K, generator=g) * 2).requires_grad_(True)
        gy = torch.randn(M, N, generator=g) * 1e-2
        lin.train()
        y = lin(x)
        y.backward(gy)
        out.update({f"c{i}_x": f32(x), f"c{i}_w": f32(lin.weight), f"c{i}_gy": f32(gy),
                    f"c{i}_y": f32(y), f"c{i}_dx": f32(x.grad), f"c{i}_dw": f32(lin.weight.grad)})
        if bias:
            out.update({f"c{i}_b": f32(lin.bias), f"c{i}_db": f32(lin.bias.grad)})
        lin.eval()
        with torch.no_grad():
            out[f"c{i}_y_eval"] = f32(lin(x.detach()))
    save("linear", **out)


def gen_draft_step():
    """One training step of a small KSDraftModel on the reference's int8 tier
    (to_int8 with trainable KS3 cells, hard Rosa path on the CPU, float head):
    the trainer's step body (train/__init__.py:145-163) up to the gradients."""
    from ksdraft.config import KSDraftConfig
    from ksdraft.kernels.ks3_int8 import KS3Int8Cell
    from ksdraft.model import KSDraftModel
    from ksdraft.model.int8_convert import to_int8
    from ksdraft.train import distillation_losses
    cfg = KSDraftConfig(vocab_size=512, layers=2, d_model=128, rosa_streams=128, ks3_charts=256)
    torch.manual_seed(0)
    model = KSDraftModel(cfg, teacher_dim=64)
    rng = np.random.default_rng(0)
    with torch.no_grad():
        for name, t in model.state_dict().items():
            leaf = name.rsplit(".", 1)[-1]
            if "norm" in name and leaf == "weight" or name.endswith("ln_attn.weight") \
                    or name.endswith("ln_ffn.weight"):
                v = 1.0 + 0.1 * rng.standard_normal(t.shape)
            elif leaf in ("bias", "gate_bias") or leaf.startswith("time_mix"):
                v = 0.1 * rng.standard_normal(t.shape)
            elif leaf == "payload":
                v = 1.0 + 0.2 * rng.standard_normal(t.shape)
            elif leaf == "raw_scale":
                v = rng.uniform(0.3, 1.2, t.shape)
            elif leaf == "raw_shift":
                v = rng.uniform(-0.5, 0.5, t.shape)
            elif leaf == "coefficients":
                v = 0.05 * rng.standard_normal(t.shape)
            else:
                v = 0.05 * rng.standard_normal(t.shape)
            t.copy_(torch.from_numpy(v.astype(np.float32)))
    weights = {k: f32(v) for k, v in model.state_dict().items() if k != "head.weight"}
    q = to_int8(model)
    for blk, src in zip(q.blocks, model.blocks):
        blk.ffn = KS3Int8Cell(src.ffn, 128, "int8", trainable=True)
    q.train()
    g = torch.Generator().manual_seed(3)
    tokens = torch.randint(0, cfg.vocab_size, (2, 65), generator=g)
    states = torch.randn(2, 64, 64, generator=g)
    logits, feats = q(tokens[:, :-1], teacher_states=states)
    loss, parts = distillation_losses(logits, tokens, feats, q.embedding.weight, None, None,
                                      0.5, 0.0)
    loss.backward()
    grads = {}
    for name, p in q.named_parameters():
        key = name.replace("ffn.master_down", "ffn.down.weight") \
            .replace("ffn.master_up", "ffn.up.weight").replace("ffn.master_", "ffn.")
        if p.grad is not None:
            grads["grad." + key] = f32(p.grad)
    assert "grad.blocks.0.rosa.q_proj.weight" not in grads   # the hard-symbol boundary
    save("draft_step", tokens=tokens.numpy(), states=f32(states), loss=np.float32(loss.item()),
         ce=np.float32(parts["ce"]), transfer=np.float32(parts["transfer"]),
         **{"w." + k: v for k, v in weights.items()}, **grads)


def gen_draft_eval():
    """Whole-sequence evaluation forward of the draft_step model (same weights,
    read back from draft_step.npz) on the reference's int8 tier (to_int8: W8A8
    Rosa and teacher projections, INT8 KS3 cells, float head), the whole-context
    semantics that drafting must reproduce: logits of the last 24 positions."""
    from ksdraft.config import KSDraftConfig
    from ksdraft.model import KSDraftModel
    from ksdraft.model.int8_convert import to_int8
    cfg = KSDraftConfig(vocab_size=512, layers=2, d_model=128, rosa_streams=128, ks3_charts=256)
    model = KSDraftModel(cfg, teacher_dim=64)
    src = np.load(HERE / "draft_step.npz")
    sd = {k[2:]: torch.from_numpy(src[k]) for k in src.files if k.startswith("w.")}
    sd["head.weight"] = sd["embedding.weight"]
    model.load_state_dict(sd)
    q = to_int8(model).eval()
    # Rosa bits are signs of fp32 projections: one within fp32 rounding of zero
    # flips with the summation order (dequantise + fp32 matmul here, exact
    # int32 groups on the GPU) and moves every later match of its stream.  The
    # inputs are drawn until every q / k / v projection of every layer is
    # clear of zero by 1e-5 of its tensor's mean magnitude (the two paths agree to
    # 2.2e-6 of it).
    projs = []
    for blk in q.blocks:
        for nm in ("q_proj", "k_proj", "v_proj"):
            getattr(blk.rosa, nm).register_forward_hook(
                lambda m, i, o: projs.append(o.detach()))
    for seed in range(9, 200):
        g = torch.Generator().manual_seed(seed)
        base = torch.randint(0, 40, (2, 48), generator=g)
        tokens = torch.cat([base, base[:, :40], torch.randint(0, 512, (2, 32), generator=g)], 1)
        states = torch.randn(2, tokens.shape[1], 64, generator=g)
        projs.clear()
        with torch.no_grad():
            logits, _ = q(tokens, teacher_states=states)
        margin = min(float((p.abs() / p.abs().mean()).min()) for p in projs)
        if margin > 1e-5:
            break
    print(f"draft_eval: seed {seed}, smallest |projection| / mean {margin:.2e}")
    save("draft_eval", tokens=tokens.numpy(), states=f32(states), logits_tail=f32(logits[:, -24:]),
         seed=np.int64(seed), margin=np.float32(margin))


def gen_rosa_credits():
    """HardRosaGPU (ksdraft/kernels/rosa_credit_gpu.py:51-112, torch ops, run on
    the CPU here) forward and backward: the hard output and the gradients of
    q / k / v (counterfactual credits through the Bernoulli map) and payload,
    on random projections (tests/test_rosa_credit_gpu.py:12-19 regime) and on
    projections whose signs come in long runs (long matches, the 62-bit cap)."""
    from ksdraft.kernels.rosa_credit_gpu import HardRosaGPU
    out = {}
    g = torch.Generator().manual_seed(21)
    cases = {"small": (2, 16, 8, False), "runs": (1, 63, 6, True), "mid": (2, 40, 5, False)}
    for name, (B, T, S, runs) in cases.items():
        q, k, v = (torch.randn(B, T, S, generator=g) * 2 for _ in range(3))
        if runs:   # signs flip with probability 0.1 per position
            for x in (q, k, v):
                flips = (torch.rand(B, T, S, generator=g) < 0.1).to(torch.int64)
                sgn = 1.0 - 2.0 * (torch.cumsum(flips, 1) % 2).float()
                x.copy_(x.abs() * sgn)
        payload = torch.randn(S, generator=g).abs() + 0.5
        gy = torch.randn(B, T, S, generator=g)
        leaves = [t.clone().requires_grad_(True) for t in (q, k, v, payload)]
        y = HardRosaGPU.apply(*leaves)
        y.backward(gy)
        out.update({f"{name}_q": f32(q), f"{name}_k": f32(k), f"{name}_v": f32(v),
                    f"{name}_payload": f32(payload), f"{name}_gy": f32(gy), f"{name}_y": f32(y),
                    f"{name}_gq": f32(leaves[0].grad), f"{name}_gk": f32(leaves[1].grad),
                    f"{name}_gv": f32(leaves[2].grad), f"{name}_gp": f32(leaves[3].grad)})
    save("rosa_credits", **out)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref", default=os.environ.get("KSD8_REFERENCE"),
                    help="checkout of the reference package (or set KSD8_REFERENCE)")
    ap.add_argument("--only", nargs="*", default=None, help="topics to regenerate")
    args = ap.parse_args()
    if not args.ref:
        ap.error("--ref (or KSD8_REFERENCE) must name the reference checkout")
    sys.path.insert(0, args.ref)
    torch.set_num_threads(8)
    topics = {"quant": gen_quant, "dither": gen_dither, "gemm": gen_gemm, "ks3_spine": gen_ks3,
              "ks3_layer": gen_ks3_layer, "rosa": gen_rosa, "tanh16": gen_tanh16,
              "linear": gen_linear, "draft_step": gen_draft_step, "draft_eval": gen_draft_eval,
              "rosa_credits": gen_rosa_credits}
    for name, fn in topics.items():
        if args.only is None or name in args.only:
            fn()


if __name__ == "__main__":
    main()
