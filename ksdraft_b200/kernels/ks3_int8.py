"""All-INT8 KS3 cell on B200 (drop-in for ksdraft/kernels/ks3_int8.py).

`KS3Int8Cell` keeps the reference constructor, buffers and modes
(ks3_int8.py:95-154).  `_KS3Int8Train` keeps the autograd contract of
ks3_int8.py:317-429 (same inputs, same saved quantities, same gradient
dtypes including the FP16 handoff with fp32 fallback on overflow).

Forward (composed semantics, the reference's parity oracle `_forward_composed`):
  ksd8_quantize_rows   x -> xq, xs
  ksd8_w8a8_gemm       coords = fp16(xq @ down^T) saturated to +-65504
  ksd8_ks3_spine_quant h = spine(coords) -> hq, hs (GS128 along charts)
  ksd8_w8a8_gemm       y = hq @ up^T, written in the input dtype
Backward:
  ksd8_quantize_rows   g -> fp16 -> gq, gs
  ksd8_quantize_cols   up^T requantised (dequant -> transpose -> requant)
  ksd8_w8a8_gemm       value = fp16(gq @ upT^T)                 (dgrad of up)
  ksd8_ks3_vjp         dc (quantised along charts and along tokens) + partials
  ksd8_ks3_vjp_reduce  dcoeff, dscale, dshift (fp16)
  ksd8_w8a8_gemm       dx = dcq @ downT^T                        (dgrad of down)
  ksd8_w8a8_gemm       ddown = dcT @ xT^T, dup = gT @ hT^T       (wgrads)
"""

from __future__ import annotations

from types import SimpleNamespace

import torch
from torch import nn

from .. import _lib
from .gemm import gemm_out, w8a8_gemm  # noqa: F401 (reference names)
from .quant import GROUP_SIZE, _check_group, dequantize_last_dim, quantize_cols, \
    quantize_last_dim

TANH_DOMAIN = 3.2
FP16 = torch.float16


def make_tanh_lut(device) -> torch.Tensor:
    """256-entry INT8 tanh table over [-3.2, 3.2] (ks3_int8.py:50-54).

    Built on the host with the reference's own torch expression (a constant
    table), then moved to `device`."""
    idx = torch.arange(-128, 128, dtype=torch.float32)
    lut = (torch.tanh(idx * (TANH_DOMAIN / 127.0)) * 127.0).round().clamp(-127.0, 127.0)
    return lut.to(torch.int8).to(device)


def ks3_weights(down: torch.Tensor, up: torch.Tensor, coefficients: torch.Tensor,
                raw_scale: torch.Tensor, raw_shift: torch.Tensor) -> SimpleNamespace:
    """A plain holder of one KS3 decoder's five fp32 tensors under the attribute
    names KS3Int8Cell reads from the reference's fp32 cell: down.weight
    (charts, d), up.weight (d, charts), coefficients (charts, 6), raw_scale and
    raw_shift (charts,), num_charts and subspace_rank (rank-1 charts only)."""
    charts = down.shape[0]
    if coefficients.numel() != charts * 6:
        raise NotImplementedError("ksdraft_b200 implements rank-1 charts (subspace_rank == 1)")
    return SimpleNamespace(down=SimpleNamespace(weight=down), up=SimpleNamespace(weight=up),
                           coefficients=coefficients.reshape(charts, 6), raw_scale=raw_scale,
                           raw_shift=raw_shift, num_charts=charts, subspace_rank=1)


def init_ks3_weights(d_model: int, charts: int, *, generator: torch.Generator | None = None,
                     device=None, std: float = 0.02, coeff_std: float = 0.05) -> SimpleNamespace:
    """Seeded synthetic KS3 weights for benches and tests: projections N(0, std)
    (the benchmark configs' weight init), spine coefficients N(0, coeff_std),
    warp raw scale 0.75 and raw shift 0.  Drawn on `generator`'s device."""
    gdev = generator.device if generator is not None else torch.device("cpu")

    def randn(*shape):
        return torch.randn(*shape, generator=generator, device=gdev)
    w = ks3_weights(randn(charts, d_model) * std, randn(d_model, charts) * std,
                    randn(charts, 6) * coeff_std, torch.full((charts,), 0.75, device=gdev),
                    torch.zeros(charts, device=gdev))
    if device is not None:
        for t in (w.down, w.up):
            t.weight = t.weight.to(device)
        w.coefficients = w.coefficients.to(device)
        w.raw_scale, w.raw_shift = w.raw_scale.to(device), w.raw_shift.to(device)
    return w


def _pack_device(t: torch.Tensor) -> torch.device:
    if t.is_cuda:
        return t.device
    if not torch.cuda.is_available():
        raise RuntimeError("KS3Int8Cell packs its weights with the ksd8 CUDA kernels; "
                           "no CUDA device is available (there is no CPU path)")
    return torch.device("cuda", torch.cuda.current_device())


def pack_small(coefficients: torch.Tensor, raw_scale: torch.Tensor, raw_shift: torch.Tensor):
    """Spine rows + warp scalars -> (spine_codes (C,6), spine_scale (C,), ws_codes (C,1),
    ws_scales (C,1), wh_codes (C,1), wh_scales (C,1)) via ksd8_ks3_pack."""
    dev = coefficients.device
    C = raw_scale.numel()
    coeffs = coefficients.detach().float().reshape(-1, 6).contiguous()
    if coeffs.shape[0] != C:
        raise NotImplementedError("ksdraft_b200 implements rank-1 charts (subspace_rank == 1)")
    rs = raw_scale.detach().float().reshape(-1).contiguous()
    rh = raw_shift.detach().float().reshape(-1).contiguous()
    sq = torch.empty(C, 6, dtype=torch.int8, device=dev)
    ss = torch.empty(C, dtype=FP16, device=dev)
    wsc = torch.empty(C, 1, dtype=torch.int8, device=dev)
    wss = torch.empty(C, 1, dtype=FP16, device=dev)
    whc = torch.empty(C, 1, dtype=torch.int8, device=dev)
    whs = torch.empty(C, 1, dtype=FP16, device=dev)
    rc = _lib.lib().ksd8_ks3_pack(coeffs.data_ptr(), rs.data_ptr(), rh.data_ptr(), C,
                                  sq.data_ptr(), ss.data_ptr(), wsc.data_ptr(), wss.data_ptr(),
                                  whc.data_ptr(), whs.data_ptr(), None, _lib.stream_ptr(dev))
    _lib.check(rc, "ks3_pack")
    return sq, ss, wsc, wss, whc, whs


def pack_spine(coefficients: torch.Tensor, group: int = GROUP_SIZE):
    """(charts*rank, 6) rows -> codes (rows, 6), one fp16 scale per row (ks3_int8.py:87-92)."""
    rows = coefficients.reshape(-1, 6)
    codes, scales = quantize_last_dim(rows, group)
    return codes, scales.flatten().to(FP16)


def spine_table(spine_codes, spine_scale, ws_codes, ws_scales, wh_codes, wh_scales,
                lut) -> torch.Tensor:
    """(charts, 256) fp16 table of the 'int8' spine term per (chart, LUT index)."""
    C = spine_scale.numel()
    table = torch.empty(C, 256, dtype=FP16, device=spine_codes.device)
    rc = _lib.lib().ksd8_ks3_spine_table(
        C, spine_codes.data_ptr(), spine_scale.data_ptr(), _lib.ptr(ws_codes),
        ws_scales.data_ptr(), _lib.ptr(wh_codes), wh_scales.data_ptr(), lut.data_ptr(),
        table.data_ptr(), None, _lib.stream_ptr(spine_codes.device))
    _lib.check(rc, "ks3_spine_table")
    return table


def spine_quant(coords: torch.Tensor, spine_codes, spine_scale, ws_codes, ws_scales, wh_codes,
                wh_scales, lut, nonlinear: str, table: torch.Tensor | None = None
                ) -> tuple[torch.Tensor, torch.Tensor]:
    """Composed spine (_spine_features) on fp16 coords + GS128 requant of h.

    In 'int8' mode the per-(chart, index) table is built (or taken from
    `table`) and the table-driven kernel runs; the results are identical."""
    M, C = coords.shape
    G = (C + GROUP_SIZE - 1) // GROUP_SIZE
    hq = torch.empty(M, C, dtype=torch.int8, device=coords.device)
    hs = torch.empty(M, G, dtype=FP16, device=coords.device)
    if nonlinear == "int8" and table is None:
        table = spine_table(spine_codes, spine_scale, ws_codes, ws_scales, wh_codes, wh_scales,
                            lut)
    rc = _lib.lib().ksd8_ks3_spine_quant(
        coords.data_ptr(), M, C, spine_codes.data_ptr(), spine_scale.data_ptr(),
        _lib.ptr(ws_codes), ws_scales.data_ptr(), _lib.ptr(wh_codes), wh_scales.data_ptr(),
        lut.data_ptr(), _lib.NL[nonlinear], _lib.ptr(table if nonlinear == "int8" else None),
        hq.data_ptr(), hs.data_ptr(), None, _lib.stream_ptr(coords.device))
    _lib.check(rc, "ks3_spine_quant")
    return hq, hs


def spine_quant_generic(coords, spine_codes, spine_scale, ws_codes, ws_scales, wh_codes,
                        wh_scales, lut, nonlinear: str):
    """The per-element (table-free) kernel for every mode; parity cross-check."""
    M, C = coords.shape
    G = (C + GROUP_SIZE - 1) // GROUP_SIZE
    hq = torch.empty(M, C, dtype=torch.int8, device=coords.device)
    hs = torch.empty(M, G, dtype=FP16, device=coords.device)
    rc = _lib.lib().ksd8_ks3_spine_quant(
        coords.data_ptr(), M, C, spine_codes.data_ptr(), spine_scale.data_ptr(),
        _lib.ptr(ws_codes), ws_scales.data_ptr(), _lib.ptr(wh_codes), wh_scales.data_ptr(),
        lut.data_ptr(), _lib.NL[nonlinear], None, hq.data_ptr(), hs.data_ptr(), None,
        _lib.stream_ptr(coords.device))
    _lib.check(rc, "ks3_spine_quant")
    return hq, hs


class KS3Int8Cell(nn.Module):
    """W8A8 GS128 KS3 with the all-INT8 runtime (forward + Section-8 backward)."""

    def __init__(self, cell, group: int = GROUP_SIZE, nonlinear: str = "int8",
                 *, trainable: bool = False):
        super().__init__()
        if nonlinear not in ("fp32", "fp16", "int8"):
            raise ValueError("nonlinear must be fp32, fp16 or int8")
        _check_group(group)
        self.group = group
        self.nonlinear = nonlinear
        self.num_subspaces = cell.num_charts
        self.subspace_rank = cell.subspace_rank
        if self.subspace_rank != 1:
            raise NotImplementedError("ksdraft_b200 implements rank-1 charts (subspace_rank == 1)")
        self.in_features = cell.down.weight.shape[1]
        self.out_features = cell.up.weight.shape[0]
        features = self.num_subspaces * self.subspace_rank
        if cell.down.weight.shape[0] != features or cell.up.weight.shape[1] != features:
            raise ValueError("Projection shapes do not match subspace count and rank")
        home = cell.down.weight.device
        dev = _pack_device(cell.down.weight)
        down = cell.down.weight.detach().float().to(dev)
        up = cell.up.weight.detach().float().to(dev)
        coeffs = cell.coefficients.detach().float().reshape(self.num_subspaces,
                                                            self.subspace_rank, 6).to(dev)
        raw_scale = cell.raw_scale.detach().float().reshape(self.num_subspaces).to(dev)
        raw_shift = cell.raw_shift.detach().float().reshape(self.num_subspaces).to(dev)

        dq, ds = quantize_last_dim(down, group)
        uq, us = quantize_last_dim(up, group)
        sq, ss, wsc, wss, whc, whs = pack_small(coeffs, raw_scale, raw_shift)
        for name, val in (("down_codes", dq), ("down_scales", ds), ("up_codes", uq),
                          ("up_scales", us), ("spine_codes", sq), ("spine_scale", ss)):
            self.register_buffer(name, val.to(home))
        self.register_buffer("warp_scale_raw", raw_scale.to(home))
        self.register_buffer("warp_shift_raw", raw_shift.to(home))
        for name, val in (("warp_scale_codes", wsc), ("warp_scale_scales", wss),
                          ("warp_shift_codes", whc), ("warp_shift_scales", whs)):
            self.register_buffer(name, val.to(home))
        self.register_buffer("tanh_lut", make_tanh_lut(home))
        self.trainable = trainable
        if trainable:
            for name, value in (("down", down), ("up", up), ("coefficients", coeffs),
                                ("raw_scale", raw_scale), ("raw_shift", raw_shift)):
                setattr(self, "master_" + name, nn.Parameter(value.clone().to(home)))

    # ---- scalar dequantisation into the active arithmetic domain ----

    def _warp_scalars(self, dtype: torch.dtype):
        scale = dequantize_last_dim(self.warp_scale_codes, self.warp_scale_scales,
                                    self.group).reshape(-1).to(dtype)
        shift = dequantize_last_dim(self.warp_shift_codes, self.warp_shift_scales,
                                    self.group).reshape(-1).to(dtype)
        return scale, shift

    @torch.no_grad()
    def _repack_masters(self):
        dither = float(getattr(self, "_dither", 0.0))
        if dither > 0:
            from ..train.stages import quantize_last_dim_dithered
            seed = getattr(self, "_dither_seed", None)
            dq, ds = quantize_last_dim_dithered(self.master_down, self.group, dither, seed=seed)
            uq, us = quantize_last_dim_dithered(
                self.master_up, self.group, dither,
                seed=None if seed is None else seed + 1)
        else:
            dq, ds = quantize_last_dim(self.master_down, self.group)
            uq, us = quantize_last_dim(self.master_up, self.group)
        sq, ss, wsc, wss, whc, whs = pack_small(self.master_coefficients, self.master_raw_scale,
                                                self.master_raw_shift)
        self.down_codes, self.down_scales = dq, ds
        self.up_codes, self.up_scales = uq, us
        self.spine_codes, self.spine_scale = sq, ss
        self.warp_scale_codes, self.warp_scale_scales = wsc, wss
        self.warp_shift_codes, self.warp_shift_scales = whc, whs
        self.warp_scale_raw = self.master_raw_scale.detach()
        self.warp_shift_raw = self.master_raw_shift.detach()

    def _project(self, xq: torch.Tensor, xs: torch.Tensor):
        """coords = fp16 clamp(xq @ down^T); h codes/scales of the spine features."""
        coords = gemm_out(_pad_k(xq), xs, _pad_k(self.down_codes), self.down_scales,
                          out_dtype=FP16, clamp_f16=True)
        hq, hs = spine_quant(coords, self.spine_codes, self.spine_scale, self.warp_scale_codes,
                             self.warp_scale_scales, self.warp_shift_codes,
                             self.warp_shift_scales, self.tanh_lut, self.nonlinear)
        return hq, hs, coords

    def _out_dtype(self, x: torch.Tensor) -> torch.dtype:
        dt = torch.get_autocast_gpu_dtype() if torch.is_autocast_enabled("cuda") else x.dtype
        return dt if dt in (torch.float32, torch.bfloat16, torch.float16) else torch.float32

    def _forward_composed(self, x: torch.Tensor) -> torch.Tensor:
        _lib.require_cuda(x)
        x2 = x.reshape(-1, x.shape[-1])
        xq, xs = quantize_last_dim(x2, self.group)
        hq, hs, _ = self._project(xq, xs)
        y = gemm_out(_pad_k(hq), hs, _pad_k(self.up_codes), self.up_scales,
                     out_dtype=self._out_dtype(x))
        return y.reshape(*x.shape[:-1], self.out_features)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        if self.trainable:
            return _KS3Int8Train.apply(
                x, self.master_down, self.master_up, self.master_coefficients,
                self.master_raw_scale, self.master_raw_shift, self)
        return self._forward_composed(x)


def _handoff(t16: torch.Tensor, bad: bool, fp32_fn=None) -> torch.Tensor:
    """FP16 gradient handoff (ks3_int8.py:75-84): fp16 unless it overflowed."""
    if not bad:
        return t16
    return fp32_fn() if fp32_fn is not None else t16.float()


class _KS3Int8Train(torch.autograd.Function):
    """Training forward/backward of the all-INT8 cell on the ksd8 kernels."""

    @staticmethod
    def forward(ctx, inputs, down, up, coefficients, raw_scale, raw_shift, cell):
        y, saved = ks3_train_forward(cell, inputs)
        ctx.cell = cell
        ctx.input_shape = inputs.shape
        ctx.save_for_backward(*saved)
        return y

    @staticmethod
    def backward(ctx, grad_out):
        cell = ctx.cell
        xq, xs, hq, hs, coords = ctx.saved_tensors
        return ks3_backward(cell, grad_out, xq, xs, hq, hs, coords, ctx.input_shape)


def _pad_k(codes: torch.Tensor) -> torch.Tensor:
    """Zero codes up to the next multiple of 128 along the last dim (a partial
    final group contributes nothing, gemm.py:71-73)."""
    pad = -codes.shape[-1] % GROUP_SIZE
    return torch.nn.functional.pad(codes, (0, pad)) if pad else codes


def ks3_train_forward(cell, inputs):
    """Training forward of ks3_int8.py:326-338: re-pack the masters, quantise x,
    project, spine, up-projection.  Returns (y, (xq, xs, hq, hs, coords))."""
    _lib.require_cuda(inputs)
    cell._repack_masters()
    x = inputs.reshape(-1, inputs.shape[-1])
    xq, xs = quantize_last_dim(x, cell.group)
    hq, hs, coords = cell._project(xq, xs)
    y = gemm_out(_pad_k(hq), hs, _pad_k(cell.up_codes), cell.up_scales,
                 out_dtype=cell._out_dtype(inputs))
    return y.reshape(*inputs.shape[:-1], cell.out_features), (xq, xs, hq, hs, coords)


def _wgrad_into(out, aq, as_, bq, bs, flag):
    """fp32 wgrad with the FP16 handoff rounding, and its predicated fp32
    re-run when any element overflowed fp16 (decided on the device)."""
    gemm_out(aq, as_, bq, bs, out=out, round_f16=True, status=flag)
    gemm_out(aq, as_, bq, bs, out=out, status=flag, if_status=True)


def ks3_backward(cell, grad_out, xq, xs, hq, hs, coords, input_shape, check_handoff=True,
                 grads_into=None, on_grad=None):
    """Backward of ks3_int8.py:341-429.

    Returns (dx, ddown, dup, dcoeff, dscale, dshift, None) as the reference's
    autograd Function.  With `grads_into` (a dict of fp32 tensors shaped like
    the masters: down, up, coefficients, raw_scale, raw_shift) the parameter
    gradients are instead written there, as the values the FP16 handoff
    (ks3_int8.py:75-84) gives after the cast to the fp32 masters, and only dx
    is returned.  That path decides the overflow fallback on the device (a
    predicated fp32 re-run of the wgrad GEMM), so it never waits for the GPU.
    There `on_grad(names)` is called as soon as those gradients are written
    (the data-parallel step starts their all-reduce there); the up-projection
    wgrad, which needs only g and h, comes first so that its reduction
    overlaps the rest of the backward."""
    M, C = coords.shape
    dev = coords.device
    g = grad_out.reshape(-1, cell.out_features)
    if g.stride(-1) != 1:
        g = g.contiguous()
    lib = _lib.lib()
    stream = _lib.stream_ptr(dev)
    flags = torch.zeros(3, dtype=torch.int32, device=dev)
    notify = on_grad if on_grad is not None else (lambda names: None)

    gT_q = None
    if grads_into is not None:
        # dup = q(g^T) @ q(h^T)^T first (ks3_int8.py:421-424)
        gT_q, gT_s = quantize_cols(g, round_f16=True)
        hT_q, hT_s = quantize_cols(hq, x_scales=hs, x_group=cell.group)
        if M % GROUP_SIZE:
            gT_q, hT_q = _pad_k(gT_q), _pad_k(hT_q)
        _wgrad_into(grads_into["up"], gT_q, gT_s, hT_q, hT_s, flags[2:3])
        notify(("up",))

    # value = fp16(q(g16) @ q(dequant(up)^T)^T)   (ks3_int8.py:345-352)
    gq = torch.empty(M, cell.out_features, dtype=torch.int8, device=dev)
    gs = torch.empty(M, (cell.out_features + 127) // 128, dtype=FP16, device=dev)
    from .quant import quantize_rows_into
    quantize_rows_into(g, gq, gs, round_f16=True)
    upT_q, upT_s = quantize_cols(cell.up_codes, x_scales=cell.up_scales, x_group=cell.group)
    value = gemm_out(gq, gs, upT_q, upT_s, out_dtype=FP16)

    # geometry VJP + both quantisations of dc (ks3_int8.py:354-418)
    n_tiles = (M + 127) // 128
    dcq = torch.empty(M, C, dtype=torch.int8, device=dev)
    dcs = torch.empty(M, C // 128, dtype=FP16, device=dev)
    dctq = torch.empty(C, M, dtype=torch.int8, device=dev)
    dcts = torch.empty(C, n_tiles, dtype=FP16, device=dev)
    partials = torch.empty(n_tiles, 8, C, dtype=torch.float32, device=dev)
    rc = lib.ksd8_ks3_vjp(value.data_ptr(), coords.data_ptr(), M, C, cell.spine_codes.data_ptr(),
                          cell.spine_scale.data_ptr(), cell.warp_scale_codes.data_ptr(),
                          cell.warp_scale_scales.data_ptr(), cell.warp_shift_codes.data_ptr(),
                          cell.warp_shift_scales.data_ptr(), dcq.data_ptr(), dcs.data_ptr(),
                          dctq.data_ptr(), dcts.data_ptr(), partials.data_ptr(), None, stream)
    _lib.check(rc, "ks3_vjp")
    raw_scale = cell.warp_scale_raw.float().contiguous()
    raw_shift = cell.warp_shift_raw.float().contiguous()
    if grads_into is not None:
        # dcoeff / dscale / dshift are fp16 already in the reference (:387-394):
        # the handoff hands them over unchanged and the masters see float(fp16),
        # which the reduction writes straight into the gradient buffer
        outs = [grads_into[n] for n in ("coefficients", "raw_scale", "raw_shift")]
        assert all(t.is_contiguous() and t.dtype == torch.float32 for t in outs)
        rc = lib.ksd8_ks3_vjp_reduce_f32(partials.data_ptr(), n_tiles, C, raw_scale.data_ptr(),
                                         raw_shift.data_ptr(), *(t.data_ptr() for t in outs),
                                         flags[0:1].data_ptr(), stream)
        _lib.check(rc, "ks3_vjp_reduce_f32")
        notify(("coefficients", "raw_scale", "raw_shift"))
    else:
        dcoeff = torch.empty(C, cell.subspace_rank, 6, dtype=FP16, device=dev)
        dscale = torch.empty(C, dtype=FP16, device=dev)
        dshift = torch.empty(C, dtype=FP16, device=dev)
        rc = lib.ksd8_ks3_vjp_reduce(partials.data_ptr(), n_tiles, C, raw_scale.data_ptr(),
                                     raw_shift.data_ptr(), dcoeff.data_ptr(), dscale.data_ptr(),
                                     dshift.data_ptr(), flags[0:1].data_ptr(), stream)
        _lib.check(rc, "ks3_vjp_reduce")

    # ddown = q(dc^T) @ q(x^T)^T, quantised along tokens (ks3_int8.py:417-420)
    xT_q, xT_s = quantize_cols(xq, x_scales=xs, x_group=cell.group)
    if M % GROUP_SIZE:  # the wgrads contract over tokens: zero-pad K (gemm.py:71-73)
        dctq, xT_q = _pad_k(dctq), _pad_k(xT_q)
    if grads_into is not None:
        _wgrad_into(grads_into["down"], dctq, dcts, xT_q, xT_s, flags[1:2])
        notify(("down",))

    # dx = q(dc) @ q(dequant(down)^T)^T   (ks3_int8.py:410-412)
    downT_q, downT_s = quantize_cols(cell.down_codes, x_scales=cell.down_scales,
                                     x_group=cell.group)
    dx = gemm_out(dcq, dcs, downT_q, downT_s, out_dtype=grad_out.dtype
                  if grad_out.dtype in (torch.float32, torch.bfloat16, torch.float16)
                  else torch.float32)
    if grads_into is not None:
        return dx.reshape(input_shape).to(grad_out.dtype)
    gT_q, gT_s = quantize_cols(g, round_f16=True)
    hT_q, hT_s = quantize_cols(hq, x_scales=hs, x_group=cell.group)
    if M % GROUP_SIZE:
        gT_q, hT_q = _pad_k(gT_q), _pad_k(hT_q)
    ddown = gemm_out(dctq, dcts, xT_q, xT_s, out_dtype=FP16, status=flags[1:2])
    dup = gemm_out(gT_q, gT_s, hT_q, hT_s, out_dtype=FP16, status=flags[2:3])

    bad = [False, False, False]
    if check_handoff:
        bad = [bool(v) for v in flags.cpu().tolist()]
    dcoeff_o = _handoff(dcoeff, bad[0])
    dscale_o = _handoff(dscale, bad[0])
    dshift_o = _handoff(dshift, bad[0])
    if bad[0]:  # per-tensor decision as the reference: only the non-finite ones go fp32
        dcoeff_o = dcoeff if torch.isfinite(dcoeff).all() else dcoeff.float()
        dscale_o = dscale if torch.isfinite(dscale).all() else dscale.float()
        dshift_o = dshift if torch.isfinite(dshift).all() else dshift.float()
    ddown_o = _handoff(ddown, bad[1], lambda: gemm_out(dctq, dcts, xT_q, xT_s))
    dup_o = _handoff(dup, bad[2], lambda: gemm_out(gT_q, gT_s, hT_q, hT_s))
    dx = dx.reshape(input_shape).to(grad_out.dtype)
    return dx, ddown_o, dup_o, dcoeff_o, dscale_o, dshift_o, None
