"""CPU oracle of KSDraft's INT8 hot path — TEST INFRASTRUCTURE ONLY.

Imported by tests/, __graft_entry__.smoke() and bench.py's CPU-baseline /
reference arm, as the checker and the CPU baseline.  The ksdraft_b200 product
never imports it.  It restates the reference algorithms (file:line cites are
paths within curvedinf/ksdraft) in numpy, plus the C restatements of
oracle/ksd8_oracle.c for the byte/integer and fp16-sequence arithmetic.
Parity pinning: tests/test_oracle_golden.py checks every function here
against fixtures produced by the reference itself (tests/golden/make_golden.py).
"""

from __future__ import annotations

import ctypes as C
from pathlib import Path

import numpy as np

from . import build as _build

_lib = None


def lib() -> C.CDLL:
    global _lib
    if _lib is None:
        path = _build.LIB
        if not path.exists():
            path = _build.build()
        L = C.CDLL(str(path))
        P = C.c_void_p
        i64, u64, f32, i32 = C.c_int64, C.c_uint64, C.c_float, C.c_int
        sig = {
            "or_philox_uniform": [u64, u64, i64, P],
            "or_quantize_rows": [P, i64, i64, i32, f32, u64, u64, P, P, P],
            "or_dequantize_rows": [P, P, i64, i64, P],
            "or_w8a8_gemm": [P, P, P, P, i64, i64, i64, P, P],
            "or_ks3_pack": [P, P, P, i64, P, P, P, P, P, P],
            "or_ks3_spine_quant": [P, i64, i64, P, P, P, P, P, P, P, i32, P, P, P],
            "or_ks3_vjp": [P, P, i64, i64, P, P, P, P, P, P, P, P],
            "or_rosa_match_bruteforce": [P, P, P, i64, i64, i32, P, P, P],
            "or_rosa_match_dp": [P, P, P, i64, i64, i32, P, P, P, P, i32],
            "or_tanh16_table": [i64, P],
        }
        for name, args in sig.items():
            fn = getattr(L, name)
            fn.argtypes = args
            fn.restype = None
        _lib = L
    return _lib


def _p(a: np.ndarray | None):
    return None if a is None else a.ctypes.data_as(C.c_void_p)


def _c(a, dtype):
    return np.ascontiguousarray(a, dtype=dtype)


def f16bits(a: np.ndarray) -> np.ndarray:
    return np.ascontiguousarray(a, dtype=np.float16).view(np.uint16)


def from_f16bits(b: np.ndarray) -> np.ndarray:
    return np.ascontiguousarray(b, dtype=np.uint16).view(np.float16)


# ------------------------------------------------------------------ quantisers

def quantize_last_dim(x: np.ndarray, group: int = 128):
    """numpy restatement of ksdraft/kernels/quant.py:30-52 (fp32 math)."""
    x = np.asarray(x, dtype=np.float32)
    K = x.shape[-1]
    Kp = (K + group - 1) // group * group
    if Kp != K:
        pad = [(0, 0)] * (x.ndim - 1) + [(0, Kp - K)]
        x = np.pad(x, pad)
    g = x.reshape(*x.shape[:-1], Kp // group, group)
    amax = np.abs(g).max(axis=-1) if g.size else np.zeros(g.shape[:-1], np.float32)
    scale = np.clip(amax.astype(np.float32) / np.float32(127.0), np.float32(2.0**-24),
                    np.float32(65504.0)).astype(np.float16).astype(np.float32)
    codes = np.clip(np.rint(g / scale[..., None]), -127, 127).astype(np.int8)
    codes = codes.reshape(*x.shape[:-1], Kp)[..., :K]
    return np.ascontiguousarray(codes), scale.astype(np.float16)


def quantize_rows_c(x: np.ndarray, *, round_f16=False, dither=0.0, seed=0, offset=0, u=None):
    """C restatement (ksd8_oracle.c:or_quantize_rows); 2-D fp32 input."""
    x = _c(x, np.float32)
    R, K = x.shape
    G = (K + 127) // 128
    codes = np.empty((R, K), np.int8)
    scales = np.empty((R, G), np.uint16)
    uu = _c(u, np.float32) if u is not None else None
    lib().or_quantize_rows(_p(x), R, K, int(round_f16), float(dither), seed, offset, _p(uu),
                           _p(codes), _p(scales))
    return codes, from_f16bits(scales)


def dequantize_last_dim(codes: np.ndarray, scales: np.ndarray, group: int = 128) -> np.ndarray:
    K = codes.shape[-1]
    Kp = (K + group - 1) // group * group
    c = codes.astype(np.float32)
    if Kp != K:
        c = np.pad(c, [(0, 0)] * (c.ndim - 1) + [(0, Kp - K)])
    g = c.reshape(*c.shape[:-1], Kp // group, group) * scales.astype(np.float32)[..., None]
    return g.reshape(*c.shape[:-1], Kp)[..., :K]


def philox_uniform(seed: int, offset: int, n: int) -> np.ndarray:
    out = np.empty(n, np.float32)
    lib().or_philox_uniform(seed, offset, n, _p(out))
    return out


def quantize_last_dim_dithered(x: np.ndarray, dither: float, u: np.ndarray):
    """stages.py:27-50 with the uniform noise U supplied (padded (R, Kp) grid)."""
    x = np.asarray(x, np.float32)
    K = x.shape[-1]
    Kp = (K + 127) // 128 * 128
    xp = np.pad(x, [(0, 0)] * (x.ndim - 1) + [(0, Kp - K)]) if Kp != K else x
    g = xp.reshape(*xp.shape[:-1], Kp // 128, 128)
    amax = np.abs(g).max(axis=-1)
    scale = np.clip(amax / np.float32(127.0), np.float32(2.0**-24),
                    np.float32(65504.0)).astype(np.float16).astype(np.float32)
    codes = g / scale[..., None]
    noise = (u.reshape(g.shape).astype(np.float32) - np.float32(0.5)) * np.float32(2.0 * dither)
    codes = np.clip(np.rint(codes + noise), -127, 127).astype(np.int8)
    return codes.reshape(*xp.shape[:-1], Kp)[..., :K], scale.astype(np.float16)


# ------------------------------------------------------------------ GEMM

def w8a8_gemm_reference_tier(a_codes, a_scales, w_codes, w_scales, group=128):
    """The reference's CPU tier (ksdraft/kernels/gemm.py:76-82): dequantise, fp32 matmul."""
    M, K = a_codes.shape
    N = w_codes.shape[0]
    G = a_scales.shape[-1]
    Kp = G * group
    if K < Kp:
        a_codes = np.pad(a_codes, ((0, 0), (0, Kp - K)))
        w_codes = np.pad(w_codes, ((0, 0), (0, Kp - K)))
    a = a_codes.reshape(M, G, group).astype(np.float32) * a_scales.reshape(M, G, 1).astype(
        np.float32)
    w = w_codes.reshape(N, G, group).astype(np.float32) * w_scales.reshape(N, G, 1).astype(
        np.float32)
    return a.reshape(M, Kp) @ w.reshape(N, Kp).T


def w8a8_gemm_canonical(a_codes, a_scales, w_codes, w_scales, with_partials=False):
    """Per-group int32 dots + the canonical fp32 group sum (bit-exact target of the GPU)."""
    a = _c(a_codes, np.int8)
    w = _c(w_codes, np.int8)
    M, K = a.shape
    N = w.shape[0]
    out = np.empty((M, N), np.float32)
    part = np.empty((K // 128, M, N), np.int32) if with_partials else None
    lib().or_w8a8_gemm(_p(a), _p(f16bits(a_scales)), _p(w), _p(f16bits(w_scales)), M, N, K,
                       _p(out), _p(part))
    return (out, part) if with_partials else out


def group_partials_numpy(a_codes, w_codes):
    M, K = a_codes.shape
    G = K // 128
    a = a_codes.reshape(M, G, 128).astype(np.int64)
    w = w_codes.reshape(w_codes.shape[0], G, 128).astype(np.int64)
    return np.einsum("mgk,ngk->gmn", a, w).astype(np.int32)


# ------------------------------------------------------------------ LM head

def _pad128(c):
    pad = -c.shape[-1] % 128
    return np.pad(c, [(0, 0)] * (c.ndim - 1) + [(0, pad)]) if pad else c


def lm_head_ce(x, w, targets):
    """INT8-tier LM head + mean cross-entropy and its backward.

    Forward follows Int8Linear semantics (ksdraft/kernels/linear.py:67-73:
    per-token and per-row GS128, w8a8_gemm) for the tied head of
    ksdraft/model/draft.py:39,51,82, then F.cross_entropy (mean,
    ksdraft/train/__init__.py:77) in float64.  Backward: dlogits = (softmax -
    onehot) / M, then dx = q(dl) q(W^T)^T and dW = q(dl^T) q(x^T)^T, W8A8 as
    the cell backward of ksdraft/kernels/ks3_int8.py:410-424.
    Returns (loss, logits fp32, dx fp32, dW fp32)."""
    x = np.asarray(x, np.float32)
    w = np.asarray(w, np.float32)
    t = np.asarray(targets, np.int64)
    M = x.shape[0]
    xq, xs = quantize_last_dim(x)
    wq, ws = quantize_last_dim(w)
    logits = w8a8_gemm_canonical(_pad128(xq), xs, _pad128(wq), ws)
    l64 = logits.astype(np.float64)
    mx = l64.max(1, keepdims=True)
    se = np.exp(l64 - mx).sum(1, keepdims=True)
    lse = (np.log(se) + mx)[:, 0]
    loss = float(np.mean(lse - l64[np.arange(M), t]))
    p = np.exp(l64 - lse[:, None])
    p[np.arange(M), t] -= 1.0
    dl = (p / M).astype(np.float32)
    dq, ds = quantize_last_dim(dl)
    wT_q, wT_s = quantize_last_dim(dequantize_last_dim(wq, ws).T.copy())
    dx = w8a8_gemm_canonical(_pad128(dq), ds, _pad128(wT_q), wT_s)
    dlT_q, dlT_s = quantize_last_dim(dl.T.copy())
    xT_q, xT_s = quantize_last_dim(x.T.copy())
    dw = w8a8_gemm_canonical(_pad128(dlT_q), dlT_s, _pad128(xT_q), xT_s)
    return loss, logits, dx, dw


# ------------------------------------------------------------------ KS3

def ste_scale_grad(x: np.ndarray, codes: np.ndarray, gx: np.ndarray) -> np.ndarray:
    """The gradient the reference's STE input path sends through the GS128 scale
    (ksdraft/kernels/linear.py:92-93 quantises the grad-carrying input, so the
    scale = fp16(clamp(amax / 127)) of quant.py:47-49 is differentiable): per
    group, G = sum(gx * codes) rounded to fp16 (the gradient crosses the fp16
    scale tensor), / 127, inside the clamp range only, split evenly over the
    elements tied at amax, times sign(x).  x, codes, gx: (M, K)."""
    M, K = x.shape
    Kp = -(-K // 128) * 128
    G = Kp // 128

    def pad(a):
        out = np.zeros((M, Kp), np.float32)
        out[:, :K] = a
        return out.reshape(M, G, 128)
    xp, cp, gp = pad(x), pad(codes), pad(gx)
    a = np.abs(xp)
    amax = a.max(-1, keepdims=True)
    tie = a == amax
    n_tie = tie.sum(-1, keepdims=True)
    g16 = (gp * cp).sum(-1, keepdims=True).astype(np.float16).astype(np.float32)
    s32 = amax / np.float32(127.0)
    inside = (s32 >= np.float32(2.0**-24)) & (s32 <= np.float32(65504.0))
    extra = np.where(tie, np.sign(xp) * (g16 / np.float32(127.0)) / n_tie, 0.0) * inside
    return extra.reshape(M, Kp)[:, :K].astype(np.float32)


def int8_linear_ste(x, w, b, gy):
    """Int8Linear training forward + backward (ksdraft/kernels/linear.py:75-97):
    y = deq(q(x)) @ deq(q(w))^T + b in fp32; dW = gy^T deq(q(x)) (straight
    through the weight quantiser, which runs without grad, :46-56); dx = gy
    deq(q(w)) plus the scale term of ste_scale_grad; db = sum gy."""
    xq, xs = quantize_rows_c(x)
    wq, ws = quantize_rows_c(w)
    xd = dequantize_last_dim(xq, xs)
    wd = dequantize_last_dim(wq, ws)
    y = xd @ wd.T
    if b is not None:
        y = y + b
    gx = gy @ wd
    dx = gx + ste_scale_grad(x, xq.astype(np.float32), gx)
    dw = gy.T @ xd
    db = gy.sum(0) if b is not None else None
    return y.astype(np.float32), dx, dw.astype(np.float32), db


def tanh16_table(n: int = 0x4600) -> np.ndarray:
    """uint16 bits of the correctly rounded fp16 tanh of the fp16 values with bits
    0..n-1 (what the reference's CPU torch.tanh gives for fp16 inputs,
    ks3_int8.py:366-367)."""
    out = np.empty(n, np.uint16)
    lib().or_tanh16_table(n, _p(out))
    return out


def make_tanh_lut() -> np.ndarray:
    """ks3_int8.py:50-54 restated: round(tanh(i * 3.2/127) * 127), i in [-128, 127]."""
    idx = np.arange(-128, 128, dtype=np.float32)
    v = np.tanh(idx * np.float32(3.2 / 127.0)) * np.float32(127.0)
    return np.clip(np.rint(v), -127, 127).astype(np.int8)


def ks3_pack(coefficients, raw_scale, raw_shift):
    c = _c(coefficients, np.float32).reshape(-1, 6)
    C_ = c.shape[0]
    rs, rh = _c(raw_scale, np.float32), _c(raw_shift, np.float32)
    out = dict(spine_codes=np.empty((C_, 6), np.int8), spine_scale=np.empty(C_, np.uint16),
               ws_codes=np.empty((C_, 1), np.int8), ws_scales=np.empty((C_, 1), np.uint16),
               wh_codes=np.empty((C_, 1), np.int8), wh_scales=np.empty((C_, 1), np.uint16))
    lib().or_ks3_pack(_p(c), _p(rs), _p(rh), C_, _p(out["spine_codes"]), _p(out["spine_scale"]),
                      _p(out["ws_codes"]), _p(out["ws_scales"]), _p(out["wh_codes"]),
                      _p(out["wh_scales"]))
    for k in ("spine_scale", "ws_scales", "wh_scales"):
        out[k] = from_f16bits(out[k])
    return out


NL = {"fp32": 0, "fp16": 1, "int8": 2}


def ks3_spine_quant(coords16, pack, lut, nonlinear="int8", want_h=False, ws_direct=None):
    """Composed _spine_features + quantize_last_dim(h); coords16 (M, C) float16.

    ws_direct: optional (scale16, shift16) dequantised fp16 arrays (project_fused form)."""
    co = f16bits(coords16)
    M, C_ = co.shape
    G = (C_ + 127) // 128
    h = np.empty((M, C_), np.float32) if want_h else None
    hq = np.empty((M, C_), np.int8)
    hs = np.empty((M, G), np.uint16)
    if ws_direct is None:
        wsc, wss = _c(pack["ws_codes"], np.int8), f16bits(pack["ws_scales"])
        whc, whs = _c(pack["wh_codes"], np.int8), f16bits(pack["wh_scales"])
    else:
        wsc, whc = None, None
        wss, whs = f16bits(ws_direct[0]), f16bits(ws_direct[1])
    lib().or_ks3_spine_quant(_p(co), M, C_, _p(_c(pack["spine_codes"], np.int8)),
                             _p(f16bits(pack["spine_scale"])), _p(wsc), _p(wss), _p(whc),
                             _p(whs), _p(_c(lut, np.int8)), NL[nonlinear], _p(h), _p(hq),
                             _p(hs))
    return (hq, from_f16bits(hs), h) if want_h else (hq, from_f16bits(hs))


def ks3_vjp(value16, coords16, pack):
    """fp16 geometry VJP: (dc fp32 (M, C), column sums (8, C) fp32)."""
    v, co = f16bits(value16), f16bits(coords16)
    M, C_ = v.shape
    dc = np.empty((M, C_), np.float32)
    sums = np.empty((8, C_), np.float32)
    lib().or_ks3_vjp(_p(v), _p(co), M, C_, _p(_c(pack["spine_codes"], np.int8)),
                     _p(f16bits(pack["spine_scale"])), _p(_c(pack["ws_codes"], np.int8)),
                     _p(f16bits(pack["ws_scales"])), _p(_c(pack["wh_codes"], np.int8)),
                     _p(f16bits(pack["wh_scales"])), _p(dc), _p(sums))
    return dc, sums


def ks3_vjp_finish(sums, raw_scale, raw_shift):
    """Rounding + STE factors of ks3_int8.py:381-395 on the column sums."""
    f16 = np.float16
    d = sums.astype(np.float32).astype(f16)                    # .sum(0) results in fp16
    dcoeff = np.stack([d[k] for k in range(6)], -1)            # (C, 6)
    sig = (1.0 / (1.0 + np.exp(-raw_scale.astype(np.float32)))).astype(np.float32)
    th = np.tanh(raw_shift.astype(np.float32))
    dscale = (d[6].astype(np.float32) * sig).astype(f16)
    dshift_t = (d[7].astype(np.float32) * np.float32(0.5)).astype(f16)
    dshift = (dshift_t.astype(np.float32) * (np.float32(1) - th * th)).astype(f16)
    return dcoeff, dscale, dshift


def ks3_layer(x, down, up, coefficients, raw_scale, raw_shift, grad, nonlinear="int8",
              out_dtype=np.float32):
    """Full _KS3Int8Train forward + backward (ks3_int8.py:326-429), rank-1 charts.

    x (M, d) fp32 values (e.g. of bf16), masters fp32, grad (M, d_out) fp32
    values.  Returns a dict with y, dx, ddown, dup, dcoeff, dscale, dshift and
    the intermediates the GPU path materialises."""
    lut = make_tanh_lut()
    dq, ds = quantize_rows_c(down)
    uq, us = quantize_rows_c(up)
    pack = ks3_pack(coefficients, raw_scale, raw_shift)
    xq, xs = quantize_rows_c(x)
    coords = w8a8_gemm_canonical(xq, xs, dq, ds).astype(np.float16)
    coords = np.where(np.isinf(coords), np.sign(coords) * np.float16(65504), coords) \
        .astype(np.float16)
    hq, hs = ks3_spine_quant(coords, pack, lut, nonlinear)
    y = w8a8_gemm_canonical(hq, hs, uq, us)
    # backward
    gq, gs = quantize_rows_c(grad, round_f16=True)
    upT_q, upT_s = quantize_rows_c(dequantize_last_dim(uq, us).T)
    value = w8a8_gemm_canonical(gq, gs, upT_q, upT_s).astype(np.float16)
    dc, sums = ks3_vjp(value, coords, pack)
    dcoeff, dscale, dshift = ks3_vjp_finish(sums, raw_scale, raw_shift)
    dcq, dcs = quantize_rows_c(dc)
    downT_q, downT_s = quantize_rows_c(dequantize_last_dim(dq, ds).T)
    dx = w8a8_gemm_canonical(dcq, dcs, downT_q, downT_s)
    dcT_q, dcT_s = quantize_rows_c(dc.T)
    xT_q, xT_s = quantize_rows_c(dequantize_last_dim(xq, xs).T)
    ddown = w8a8_gemm_canonical(dcT_q, dcT_s, xT_q, xT_s)
    gT_q, gT_s = quantize_rows_c(np.asarray(grad, np.float32).T, round_f16=True)
    hT_q, hT_s = quantize_rows_c(dequantize_last_dim(hq, hs).T)
    dup = w8a8_gemm_canonical(gT_q, gT_s, hT_q, hT_s)
    return dict(y=y, dx=dx, ddown=ddown, dup=dup, dcoeff=dcoeff, dscale=dscale, dshift=dshift,
                xq=xq, xs=xs, coords=coords, hq=hq, hs=hs, value=value, dc=dc, dcq=dcq,
                dcs=dcs, dcT_q=dcT_q, dcT_s=dcT_s, gq=gq, gs=gs, upT_q=upT_q, upT_s=upT_s,
                downT_q=downT_q, downT_s=downT_s, xT_q=xT_q, xT_s=xT_s, gT_q=gT_q,
                gT_s=gT_s, hT_q=hT_q, hT_s=hT_s, sums=sums, pack=pack, down_q=dq, down_s=ds,
                up_q=uq, up_s=us)


# ------------------------------------------------------------------ Rosa

def default_max_len(T: int, max_match_len=None) -> int:
    if max_match_len is None:
        return max(1, min(62, T - 1)) if T > 1 else 0
    return min(max_match_len, T - 1)


def rosa_match(q, k, v, max_match_len=None, method="bruteforce"):
    """_match_payload_sign (rosa.py:40-98) on (S, T) bits: (sign, length, endpoint)."""
    q, k, v = (_c(b, np.int8) for b in (q, k, v))
    S, T = q.shape
    ml = max(0, default_max_len(T, max_match_len))
    sign = np.empty((S, T), np.float32)
    L = np.empty((S, T), np.int32)
    E = np.empty((S, T), np.int32)
    if method == "bruteforce":
        lib().or_rosa_match_bruteforce(_p(q), _p(k), _p(v), S, T, ml, _p(sign), _p(L), _p(E))
    else:
        import os
        slots = os.cpu_count() or 1
        work = np.empty(slots * 2 * max(T, 1), np.int32)
        lib().or_rosa_match_dp(_p(q), _p(k), _p(v), S, T, ml, _p(sign), _p(L), _p(E), _p(work),
                               slots)
    return sign, L, E


def rosa_credits(q, k, v, grad, max_match_len=None):
    """Counterfactual credits of ksdraft/kernels/rosa_credit_gpu.py:25-48
    (_chunk_credits), by brute force: for every stream and every q / k / v bit,
    the whole stream re-matched with that bit flipped (rosa_match, dp), and
    credit = sum_t (sign' - sign) * grad.  q, k, v (S, T) int8 bits, grad (S, T)
    fp32 = dL/d sign.  Returns (cq, ck, cv), each (S, T) float64."""
    q, k, v = (_c(b, np.int8) for b in (q, k, v))
    grad = np.asarray(grad, np.float64)
    S, T = q.shape
    out = [np.zeros((S, T), np.float64) for _ in range(3)]
    base, _, _ = rosa_match(q, k, v, max_match_len, method="dp")
    idx = np.arange(T)
    for s in range(S):
        for which in range(3):
            pert = [np.repeat(x[s][None, :], T, 0) for x in (q, k, v)]   # (T, T): row p flips bit p
            pert[which][idx, idx] ^= 1
            sp, _, _ = rosa_match(*pert, max_match_len, method="dp")
            out[which][s] = ((sp.astype(np.float64) - base[s][None, :]) * grad[s][None, :]).sum(1)
    return tuple(out)


def _bf16(a: np.ndarray) -> np.ndarray:
    """Round fp32 values to bfloat16 (round to nearest even), returned as fp32."""
    u = np.ascontiguousarray(a, np.float32).view(np.uint32)
    r = ((u + 0x7FFF + ((u >> 16) & 1)) & 0xFFFF0000).astype(np.uint32)
    return r.view(np.float32)


def rosa_mixer_int8_eval(x, sig_q, sig_k, sig_v, w, b, payload, w_out, b_out):
    """RosaMixer evaluation forward after to_int8 (ksdraft/model/rosa.py:128-165
    with Int8Linear eval projections, ksdraft/kernels/linear.py:62-73) on bf16
    activations, in this build's fixed GEMM group order.

    x (B, T, d) fp32 holding bf16 values; sig_* (d,) fp32 sigmoid(time_mix_*)
    as the module computes it (torch.sigmoid on the parameter's device);
    w / b: dicts 'q','k','v' of (S, d) / (S,) fp32; payload (S,); w_out (d, S),
    b_out (d,).  Returns y (B, T, d) fp32 holding bf16 values."""
    x = np.asarray(x, np.float32)
    B, T, d = x.shape
    S = payload.shape[0]
    prev = np.concatenate([np.zeros((B, 1, d), np.float32), x[:, :-1]], 1)
    diff = _bf16(x - prev)                              # (x - prev) in x's dtype
    bits = {}
    for c, sig in (("q", sig_q), ("k", sig_k), ("v", sig_v)):
        xin = (prev + diff * np.asarray(sig, np.float32)).reshape(B * T, d)   # fp32
        aq, as_ = quantize_rows_c(xin)
        wq, ws = quantize_rows_c(w[c])
        proj = w8a8_gemm_canonical(aq, as_, wq, ws) + b[c].astype(np.float32)
        bits[c] = (_bf16(proj) > 0).reshape(B, T, S).transpose(0, 2, 1).reshape(B * S, T)
    sign, _, _ = rosa_match(bits["q"].astype(np.int8), bits["k"].astype(np.int8),
                            bits["v"].astype(np.int8), method="dp")
    out = payload.astype(np.float32)[None, :, None] * sign.reshape(B, S, T)
    o = _bf16(out.transpose(0, 2, 1).reshape(B * T, S))     # .to(x.dtype)
    oq, os_ = quantize_rows_c(o)
    wq, ws = quantize_rows_c(w_out)
    y = w8a8_gemm_canonical(oq, os_, wq, ws) + b_out.astype(np.float32)
    return _bf16(y).reshape(B, T, d)


def rosa_sign_python(q, k, v):
    """Pure-Python brute force of the definition (tests/test_rosa.py:7-22 semantics,
    no length cap); small cases only."""
    T = len(q)
    out = [-1.0] * T
    for t in range(T):
        for L in range(min(t, T - 1), 0, -1):
            pat = q[t - L + 1: t + 1]
            best = -1
            for j in range(t - 1, L - 2, -1):
                if k[j - L + 1: j + 1] == pat:
                    best = j
                    break
            if best >= 0:
                out[t] = 1.0 if v[best + 1] else -1.0
                break
    return out
