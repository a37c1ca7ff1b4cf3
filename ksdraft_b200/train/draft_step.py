"""Full KSDraft INT8 training step on B200 (the model of ksdraft/model/draft.py).

One call runs the reference trainer's step body (ksdraft/train/__init__.py:
145-166) for the int8 tier:

  forward   x = input_norm(E[tokens]) + teacher_proj(teacher_states)   (draft.py:68-74)
            per block (block.py:34-42):
              h      = x + Rosa(ln_attn(x))            hard path, rosa.py:143-165
              h', p  = AdjacentInjection(h, p_prev)    spine.py:56-58
              x      = h' + KS3Int8Cell(ln_ffn(h'))    trainable cell, ks3_int8.py:317-429
            logits = head(output_norm(x)), head tied to E                (draft.py:39,51,82)
  loss      cross-entropy + 0.5 * transfer-space loss of the p's       (train/__init__.py:65-94)
  backward  every gradient written into one flat fp32 buffer
  update    data-parallel mean (NCCL), clip_grad_norm_(1.0), AdamW      (train/__init__.py:164-166)

What runs where:
  * INT8 surfaces on the ksd8 kernels: the Rosa q/k/v projections (time-shift
    mix fused with their per-token quantisation, W8A8 GEMMs with bias, bit
    packing), the stream matcher, the out-projection and teacher projection
    (Int8Linear semantics: W8A8 forward, straight-through backward with the
    reference's scale gradient), the KS3 cells (the all-INT8 forward and
    backward), the tied LM head (W8A8 logits, CE partials, the fused CE
    gradient quantiser and W8A8 dgrad / wgrad), AdamW and gradient clipping.
  * The float exceptions of the reference's int8 tier (int8_convert.py:8-12)
    run in the activation dtype: the DSpine low-rank injection as five cuBLAS
    GEMMs around one ksd8 kernel that applies the gate and ln_ffn (and one for
    their backward, train/injection.py), the transfer-space term and its
    gradient as ksd8 row kernels; input_norm and output_norm are torch
    LayerNorm segments.
  * Gradients follow the reference's hard-symbol boundary (rosa.py:21-29): the
    Rosa q/k/v projections, their time mixes and ln_attn receive no gradient,
    so AdamW leaves them untouched, as torch.optim.AdamW skips parameters
    whose .grad is None.

Data parallel: each rank runs its share of the sequences; every block's
gradients are averaged with an asynchronous NCCL all-reduce as soon as the
block's backward has written them (blocks are contiguous spans of the flat
buffer, in the order the backward produces them), the tied embedding's dense
head gradient right after the head backward, and the sparse embedding rows
(the input gather and the transfer-loss targets) by one all-gather of (ids,
rows) at the end.  Clipping and AdamW then run on the device without a host
round trip.
"""

from __future__ import annotations

import math
import os
from dataclasses import dataclass

import torch
import torch.distributed as dist
import torch.nn.functional as F

from .. import _lib
from ..kernels.gemm import _validate_and_pad, gemm_out
from ..kernels.ks3_int8 import KS3Int8Cell, ks3_backward, ks3_train_forward, ks3_weights
from ..kernels.quant import GROUP_SIZE, dequantize_last_dim, quantize_cols, quantize_last_dim
from ..model.head import ce_grad, ce_grad_quant, ce_partials, combine_ce_partials
from ..model.rosa import _default_max_len, match_words, pack_bits
from . import injection
from .dp import allreduce_mean_async, wait_all

# SMs left to NCCL while a block's gradient reduction overlaps the backward.  The
# config-4 backward is long (tens to hundreds of ms), so a few NCCL CTAs keep up
# with it; on 2 B200s 8 (or 4) reserved SMs gave a 254 ms step, 16 gave 260 ms
# (the KS3 backward's persistent GEMMs lose fewer SMs).
DRAFT_SM_RESERVE = int(os.environ.get("KSD8_DRAFT_SM_RESERVE", "8"))


@dataclass(frozen=True)
class DraftShape:
    """Model dimensions (defaults: configs/flint.yaml's decided draft, benchmark config 4)."""
    vocab: int = 150144
    layers: int = 24
    d_model: int = 1536
    streams: int = 512
    charts: int = 5888
    teacher_dim: int = 384
    inj_rank: int = 32       # AdjacentInjection rank (spine.py:39)
    feature_rank: int = 64   # AdjacentInjection feature_rank (spine.py:39)


def _block_shapes(s: DraftShape):
    """Trainable tensors of one block, in the order the backward completes them."""
    d, c, S, r, fr = s.d_model, s.charts, s.streams, s.inj_rank, s.feature_rank
    return [
        ("ffn.down.weight", (c, d)), ("ffn.up.weight", (d, c)), ("ffn.coefficients", (c, 6)),
        ("ffn.raw_scale", (c,)), ("ffn.raw_shift", (c,)),
        ("ln_ffn.weight", (d,)), ("ln_ffn.bias", (d,)),
        ("injection.feature_down.weight", (fr, d)), ("injection.feature_up.weight", (d, fr)),
        ("injection.gate_q.down.weight", (r, d)), ("injection.gate_q.up.weight", (d, r)),
        ("injection.gate_p.down.weight", (r, d)), ("injection.gate_p.up.weight", (d, r)),
        ("injection.gate_bias", (d,)),
        ("injection.inject.down.weight", (r, d)), ("injection.inject.up.weight", (d, r)),
        ("rosa.out_proj.weight", (d, S)), ("rosa.out_proj.bias", (d,)), ("rosa.payload", (S,)),
    ]


# names of the fp32 model's state dict (ksdraft/model/draft.py), so that weights
# load from and export to the reference format unchanged
KS3_MASTERS = {"down": "ffn.down.weight", "up": "ffn.up.weight",
               "coefficients": "ffn.coefficients", "raw_scale": "ffn.raw_scale",
               "raw_shift": "ffn.raw_shift"}
DSPINE = ("feature_down", "feature_up", "gate_q.down", "gate_q.up", "gate_p.down", "gate_p.up",
          "gate_bias", "inject.down", "inject.up")


def _dspine_name(n: str) -> str:
    return "injection." + (n if n == "gate_bias" else n + ".weight")


def _frozen_shapes(s: DraftShape):
    """Tensors of one block that receive no gradient on the hard Rosa path."""
    d, S = s.d_model, s.streams
    return [("ln_attn.weight", (d,)), ("ln_attn.bias", (d,)),
            ("rosa.q_proj.weight", (S, d)), ("rosa.q_proj.bias", (S,)),
            ("rosa.k_proj.weight", (S, d)), ("rosa.k_proj.bias", (S,)),
            ("rosa.v_proj.weight", (S, d)), ("rosa.v_proj.bias", (S,)),
            ("rosa.time_mix_q", (d,)), ("rosa.time_mix_k", (d,)), ("rosa.time_mix_v", (d,))]


class FlatParams:
    """All trainable fp32 masters as views of one flat buffer, gradients as views
    of a second one with the same offsets (64-element aligned, zero padding).

    Order: embedding, output_norm, blocks L-1 .. 0, teacher_proj, input_norm --
    the order in which the backward finishes them, so each block is one
    contiguous span whose all-reduce can start when its backward is done."""

    ALIGN = 64

    def __init__(self, shape: DraftShape, device):
        entries = [("embedding.weight", (shape.vocab, shape.d_model)),
                   ("output_norm.weight", (shape.d_model,)),
                   ("output_norm.bias", (shape.d_model,))]
        self.block_span = {}
        for layer in reversed(range(shape.layers)):
            first = len(entries)
            entries += [(f"blocks.{layer}.{n}", sh) for n, sh in _block_shapes(shape)]
            self.block_span[layer] = (first, len(entries))
        entries += [("teacher_proj.weight", (shape.d_model, shape.teacher_dim)),
                    ("input_norm.weight", (shape.d_model,)), ("input_norm.bias", (shape.d_model,))]
        self.names = [n for n, _ in entries]
        self.shapes = dict(entries)
        self.offsets = {}
        off = 0
        for n, sh in entries:
            self.offsets[n] = off
            off += (math.prod(sh) + self.ALIGN - 1) // self.ALIGN * self.ALIGN
        self.numel = off
        self.data = torch.zeros(off, dtype=torch.float32, device=device)
        self.grad = torch.zeros(off, dtype=torch.float32, device=device)

    def _view(self, buf, name):
        off, sh = self.offsets[name], self.shapes[name]
        return buf[off:off + math.prod(sh)].view(sh)

    def p(self, name: str) -> torch.Tensor:
        return self._view(self.data, name)

    def g(self, name: str) -> torch.Tensor:
        return self._view(self.grad, name)

    def span(self, first_name: str, last_name: str, buf=None) -> torch.Tensor:
        buf = self.grad if buf is None else buf
        lo = self.offsets[first_name]
        hi = self.offsets[last_name] + math.prod(self.shapes[last_name])
        return buf[lo:hi]

    def block_grad_span(self, layer: int) -> torch.Tensor:
        first, last = self.block_span[layer]
        return self.span(self.names[first], self.names[last - 1])


def init_draft_params(shape: DraftShape, device, seed: int = 0, std: float = 0.02):
    """Seeded synthetic weights (benchmark config 4: N(0, 0.02), quantised GS128 on
    use; LayerNorms at weight 1 / bias 0; Rosa payload 1, time mixes 0; KS3 spine
    coefficients N(0, 0.05), warp raw scale 0.75, raw shift 0).  Returns
    (FlatParams, frozen {name: tensor})."""
    flat = FlatParams(shape, device)
    gen = torch.Generator(device=device).manual_seed(seed)
    with torch.no_grad():
        for n in flat.names:
            t = flat.p(n)
            leaf = n.rsplit(".", 1)[-1]
            if n.endswith(("norm.weight", "ln_ffn.weight")):
                t.fill_(1.0)
            elif n.endswith(("norm.bias", "ln_ffn.bias")):
                t.zero_()
            elif leaf in ("bias", "gate_bias"):
                t.zero_()
            elif leaf == "payload":
                t.fill_(1.0)
            elif leaf == "raw_scale":
                t.fill_(0.75)
            elif leaf == "raw_shift":
                t.zero_()
            elif leaf == "coefficients":
                t.normal_(0.0, 0.05, generator=gen)
            else:
                t.normal_(0.0, std, generator=gen)
        frozen = {}
        for layer in range(shape.layers):
            for n, sh in _frozen_shapes(shape):
                t = torch.empty(sh, dtype=torch.float32, device=device)
                if n == "ln_attn.weight":
                    t.fill_(1.0)
                elif n == "ln_attn.bias" or n.startswith("rosa.time_mix"):
                    t.zero_()
                else:
                    t.normal_(0.0, std, generator=gen)
                frozen[f"blocks.{layer}.{n}"] = t
    return flat, frozen


class _ste_matmul_precision:
    """The straight-through backward GEMMs of Int8Linear (linear.py:88-94) are fp32
    in the reference.  With bf16 activations (whose values TF32 holds exactly)
    they run as TF32 tensor-core GEMMs; in the fp32 parity mode they stay fp32."""

    def __init__(self, act):
        self.use_tf32 = act != torch.float32

    def __enter__(self):
        self.prev = torch.backends.cuda.matmul.allow_tf32
        torch.backends.cuda.matmul.allow_tf32 = self.use_tf32

    def __exit__(self, *exc):
        torch.backends.cuda.matmul.allow_tf32 = self.prev


def _normalize_bwd(u: torch.Tensor, gn: torch.Tensor) -> torch.Tensor:
    """Gradient through F.normalize(u, dim=-1) (eps 1e-12) given the gradient gn
    of its output: (gn - (gn . n) n) / max(|u|, eps), and gn / eps where clamped."""
    norm = u.norm(dim=-1, keepdim=True)
    clamped = norm <= 1e-12
    safe = norm.clamp_min(1e-12)
    n = u / safe
    g = (gn - (gn * n).sum(-1, keepdim=True) * n) / safe
    return torch.where(clamped, gn / 1e-12, g)


def gather_sparse_rows(ids: torch.Tensor, rows: torch.Tensor, world: int, group=None):
    """Sparse gradient rows of the tied embedding from every rank, as (ids, rows /
    world): their scatter-add into the averaged dense gradient gives the mean
    over ranks.  One all-gather of ids and one of rows (every rank holds the
    same number of rows); alone, the rows pass through unchanged."""
    if world == 1:
        return ids, rows
    all_ids = [torch.empty_like(ids) for _ in range(world)]
    all_rows = [torch.empty_like(rows) for _ in range(world)]
    dist.all_gather(all_ids, ids.contiguous(), group=group)
    dist.all_gather(all_rows, rows.contiguous(), group=group)
    return torch.cat(all_ids), torch.cat(all_rows) / world


def check_tokens(tokens: torch.Tensor, vocab: int) -> None:
    """Token ids must index the vocabulary: F.cross_entropy and nn.Embedding raise
    on anything else.  ignore_index (-100) targets are rejected as well: the
    reference trainer never produces them (train/__init__.py:75-77)."""
    lo, hi = int(tokens.min()), int(tokens.max())
    if lo < 0 or hi >= vocab:
        raise ValueError(f"token ids must lie in [0, {vocab}); got [{lo}, {hi}]"
                         + (" (ignore_index targets are not supported)" if lo == -100 else ""))


class DraftTrainStep:
    """The full INT8 training step of a KSDraft model, data parallel over `group`.

    step(tokens, teacher_states) -> loss (device scalar tensor, no host sync):
    tokens (B, T + 1) int64, inputs tokens[:, :-1], targets tokens[:, 1:];
    teacher_states (B, T, teacher_dim) or None.  Host tensors are copied in.
    act_dtype is the residual stream / float-exception dtype (bf16 for the
    benchmark; fp32 gives the reference's fp32-model arithmetic for parity)."""

    def __init__(self, shape: DraftShape, device, *, seed: int = 0, act_dtype=torch.bfloat16,
                 lr: float = 3e-4, weight_decay: float = 0.01, grad_clip: float | None = 1.0,
                 transfer_weight: float = 0.5, group=None, params=None,
                 head_mode: str = "w8a8"):
        injection.check_width(shape.d_model)
        self.shape = shape
        self.dev = torch.device(device)
        self.act = act_dtype
        self.lr, self.wd, self.grad_clip = lr, weight_decay, grad_clip
        self.transfer_weight = transfer_weight
        if head_mode not in ("w8a8", "float"):
            raise ValueError("head_mode must be 'w8a8' or 'float'")
        # "w8a8": the north-star head (W8A8 logits, dgrad and wgrad on the fused CE
        # gradient codes); "float": the reference int8 tier's float exception
        # (int8_convert.py:8-12), an fp32 GEMM head, for parity checks
        self.head_mode = head_mode
        self.group = group
        self.flat, self.frozen = params if params is not None else init_draft_params(
            shape, self.dev, seed)
        self.m = torch.zeros_like(self.flat.data)
        self.v = torch.zeros_like(self.flat.data)
        self.step_count = 0
        self._clip_scratch = torch.empty(_lib.GRAD_CLIP_SCRATCH, device=self.dev)
        self._clip_out = torch.zeros(2, device=self.dev)
        self.cells = [self._make_cell(layer) for layer in range(shape.layers)]
        self._frozen_codes = {}
        self._ln_leaves = {}
        self.last = {}
        self.phase_marks = None   # a list to record (phase name, CUDA event) marks into
        self._capturing = False

    def _mark(self, name: str) -> None:
        """Start phase `name` (device-side timing of the step's parts, when enabled;
        during capture the events become nodes of the graph, re-recorded by every
        replay)."""
        if self.phase_marks is not None:
            ev = torch.cuda.Event(enable_timing=True, external=self._capturing)
            ev.record()
            self.phase_marks.append((name, ev))

    # ---- parameters --------------------------------------------------------

    def _make_cell(self, layer: int) -> KS3Int8Cell:
        P = lambda n: self.flat.p(f"blocks.{layer}.{KS3_MASTERS[n]}")  # noqa: E731
        cell = KS3Int8Cell(ks3_weights(P("down"), P("up"), P("coefficients"), P("raw_scale"),
                                       P("raw_shift")), nonlinear="int8", trainable=True)
        # the cell's fp32 masters become the flat buffer's views
        for n in ("down", "up", "coefficients", "raw_scale", "raw_shift"):
            getattr(cell, "master_" + n).data = P(n).view_as(getattr(cell, "master_" + n))
        return cell

    def _frozen_int8(self, layer: int, name: str):
        """GS128 codes of a weight that never changes (the reference re-quantises
        it on every call, with the same result)."""
        key = (layer, name)
        if key not in self._frozen_codes:
            self._frozen_codes[key] = quantize_last_dim(
                self.frozen[f"blocks.{layer}.rosa.{name}.weight"])
        return self._frozen_codes[key]

    def parameter_dict(self) -> dict[str, torch.Tensor]:
        """{reference state-dict name: fp32 tensor} of every parameter (the fp32
        model's names, ksdraft/model/draft.py; head.weight is embedding.weight)."""
        out = {n: self.flat.p(n) for n in self.flat.names}
        out.update(self.frozen)
        return out

    @torch.no_grad()
    def load_state_dict(self, sd: dict) -> None:
        """Copy a reference fp32-model state dict (names of parameter_dict) in."""
        for n, t in self.parameter_dict().items():
            if n not in sd:
                raise KeyError(f"missing {n}")
            t.copy_(torch.as_tensor(sd[n]).reshape(t.shape))
        self._frozen_codes.clear()

    # ---- forward pieces ------------------------------------------------------

    def _ln(self, x, name):
        """LayerNorm with fp32 master leaves (their gradients are collected by
        _ln_param_grads after the segment's backward)."""
        w = self.flat.p(f"{name}.weight").detach().requires_grad_(True)
        b = self.flat.p(f"{name}.bias").detach().requires_grad_(True)
        self._ln_leaves[name] = (w, b)
        return F.layer_norm(x, (x.shape[-1],), w.to(self.act), b.to(self.act))

    def _ln_param_grads(self, name):
        w, b = self._ln_leaves.pop(name)
        self.flat.g(f"{name}.weight").copy_(w.grad)
        self.flat.g(f"{name}.bias").copy_(b.grad)

    def _rosa_forward(self, layer: int, x3: torch.Tensor):
        """Hard Rosa forward (rosa.py:143-165) on ln_attn(x): returns (r, saved) with
        r (B*T, d) in the activation dtype."""
        B, T, d = x3.shape
        S = self.shape.streams
        pre = f"blocks.{layer}."
        with torch.no_grad():
            a = F.layer_norm(x3, (d,), self.frozen[pre + "ln_attn.weight"].to(self.act),
                             self.frozen[pre + "ln_attn.bias"].to(self.act)).contiguous()
            G = (d + GROUP_SIZE - 1) // GROUP_SIZE
            codes = [torch.empty(B * T, d, dtype=torch.int8, device=self.dev) for _ in range(3)]
            scales = [torch.empty(B * T, G, dtype=torch.float16, device=self.dev)
                      for _ in range(3)]
            mixes = [torch.sigmoid(self.frozen[pre + f"rosa.time_mix_{c}"]).contiguous()
                     for c in "qkv"]
            rc = _lib.lib().ksd8_rosa_timemix_quantize(
                a.data_ptr(), _lib.dtype_code(a), B, T, d, *(m.data_ptr() for m in mixes),
                codes[0].data_ptr(), scales[0].data_ptr(), codes[1].data_ptr(),
                scales[1].data_ptr(), codes[2].data_ptr(), scales[2].data_ptr(), None,
                _lib.stream_ptr(self.dev))
            _lib.check(rc, "rosa_timemix_quantize")
            words = []
            for i, c in enumerate("qkv"):
                wq, ws = self._frozen_int8(layer, f"{c}_proj")
                # bits = proj > 0 (rosa.py:156-158); bf16 keeps the sign of fp32
                proj = gemm_out(codes[i], scales[i], wq, ws, out_dtype=torch.bfloat16,
                                bias=self.frozen[pre + f"rosa.{c}_proj.bias"])
                words.append(pack_bits(proj, B, T, S, T * S, S, 1))
            sign = torch.empty(B, T, S, dtype=self.act, device=self.dev)
            match_words(*words, B, S, T, _default_max_len(T, None), out=sign,
                        strides=(T * S, S, 1))
            payload = self.flat.p(pre + "rosa.payload")
            o = (sign * payload).to(self.act).reshape(B * T, S)     # rosa.py:164-165
            oq, os_ = quantize_last_dim(o)
            wq, ws = quantize_last_dim(self.flat.p(pre + "rosa.out_proj.weight"))
            oqp, wqp = _validate_and_pad(oq, os_, wq, ws, GROUP_SIZE)   # streams % 128
            r = gemm_out(oqp, os_, wqp, ws, out_dtype=self.act,
                         bias=self.flat.p(pre + "rosa.out_proj.bias"))
        return r, (sign, o, oq, os_, wq, ws)

    def _rosa_backward(self, layer: int, dr: torch.Tensor, saved) -> None:
        """Int8Linear STE backward of out_proj (linear.py:75-97) and the payload
        gradient; the hard bits stop everything upstream (rosa.py:21-29)."""
        sign, o, oq, os_, wq, ws = saved
        pre = f"blocks.{layer}.rosa."
        dr32 = dr.float()
        B, T, S = sign.shape
        xd = dequantize_last_dim(oq, os_)                           # (M, S) fp32
        with _ste_matmul_precision(self.act):
            torch.matmul(dr32.t(), xd, out=self.flat.g(pre + "out_proj.weight"))
            gx = dr32 @ dequantize_last_dim(wq, ws)                 # (M, S)
        torch.sum(dr32, 0, out=self.flat.g(pre + "out_proj.bias"))
        # o = (payload * sign).to(act): d payload[s] = sum over tokens of do * sign,
        # do = the STE input gradient of gx (incl. the GS128 scale term), one kernel
        M = B * T
        n_parts = max(1, min(M, 4 * torch.cuda.get_device_properties(self.dev)
                                 .multi_processor_count))
        parts = torch.empty(n_parts, S, dtype=torch.float32, device=self.dev)
        _lib.check(_lib.lib().ksd8_rosa_payload_bwd(
            o.data_ptr(), oq.data_ptr(), gx.data_ptr(), sign.data_ptr(), _lib.dtype_code(o), M, S,
            parts.data_ptr(), n_parts, None, _lib.stream_ptr(self.dev)), "rosa_payload_bwd")
        torch.sum(parts, 0, out=self.flat.g(pre + "payload"))

    def _dspine_weights(self, layer: int):
        return {n: self.flat.p(f"blocks.{layer}.{_dspine_name(n)}") for n in DSPINE}

    # ---- the step --------------------------------------------------------------

    # ---- CUDA graph of the step ------------------------------------------------

    def capture(self, tokens: torch.Tensor, teacher_states: torch.Tensor | None = None,
                warmup: int = 2, phase_marks: bool = False) -> None:
        """Record forward + backward (everything up to the gradients) into one CUDA
        graph over static device copies of `tokens` / `teacher_states` (shapes fixed
        from here on); replay() then runs a step with no per-kernel host work.
        Data parallel over NCCL, the gradient all-reduces and the embedding-row
        all-gathers are captured too (every rank captures and replays the same
        sequence; release() before destroying the process group).  Runs `warmup`
        eager steps first (kernel attributes, cached codes, communicators)
        without updating the weights.  With phase_marks, the phase events are
        captured too (graph_marks), for graph_phases() after a replay."""
        if (dist.is_available() and dist.is_initialized()
                and dist.get_world_size(self.group) > 1
                and dist.get_backend(self.group) != "nccl"):
            raise RuntimeError("capture() of a data-parallel step needs the NCCL backend")
        check_tokens(tokens, self.shape.vocab)
        self._g_tokens = tokens.to(self.dev).clone()
        self._g_states = None if teacher_states is None else teacher_states.to(self.dev).clone()
        from ..kernels.gemm import GemmTimer
        timer, GemmTimer.active = GemmTimer.active, None   # a GEMM timer sees the graph only
        side = torch.cuda.Stream(self.dev)
        side.wait_stream(torch.cuda.current_stream(self.dev))
        with torch.cuda.stream(side):
            for _ in range(warmup):
                self.forward_backward(self._g_tokens, self._g_states, _checked=True)
        torch.cuda.current_stream(self.dev).wait_stream(side)
        torch.cuda.synchronize(self.dev)
        GemmTimer.active = timer
        self._graph = torch.cuda.CUDAGraph()
        launches0 = _lib.LAUNCHES
        marks, self.phase_marks = self.phase_marks, ([] if phase_marks else None)
        self._capturing = True
        try:
            # thread-local capture mode: the process group's watchdog thread keeps
            # polling its events while this thread captures
            with torch.cuda.graph(self._graph, capture_error_mode="thread_local"):
                self._g_loss = self.forward_backward(self._g_tokens, self._g_states,
                                                     _checked=True)
                self._g_last = dict(self.last)
        finally:
            self._capturing = False
            self.graph_marks, self.phase_marks = self.phase_marks, marks
        self.captured_launches = _lib.LAUNCHES - launches0   # ksd8 kernels per replay
        torch.cuda.synchronize(self.dev)

    def replay(self, tokens: torch.Tensor, teacher_states: torch.Tensor | None = None,
               update: bool = True) -> torch.Tensor:
        """One step through the captured graph: copy the inputs (host or device)
        into the static buffers, replay, then AdamW eagerly (its bias correction
        changes every step).  Returns the loss tensor the graph writes."""
        if tokens.device.type == "cpu":
            check_tokens(tokens, self.shape.vocab)
        self._g_tokens.copy_(tokens, non_blocking=True)
        if self._g_states is not None:
            self._g_states.copy_(teacher_states, non_blocking=True)
        self._graph.replay()
        self.last = self._g_last
        if update:
            self._update()
        return self._g_loss

    def release(self) -> None:
        """Drop the captured graph (and the collectives it holds)."""
        self._graph = None
        self.graph_marks = None

    def graph_phases(self) -> dict:
        """ms per phase of the last replay (phase_marks captured), summed by name."""
        marks = self.graph_marks or []
        out = {}
        for (name, ev), (_, nxt) in zip(marks, marks[1:]):
            out[name] = out.get(name, 0.0) + ev.elapsed_time(nxt)
        return out

    def _to_device(self, t):
        if t is None or t.device == self.dev:
            return t
        return t.to(self.dev, non_blocking=True)

    def __call__(self, tokens: torch.Tensor, teacher_states: torch.Tensor | None = None):
        """forward + backward + data-parallel mean + clip + AdamW; returns the loss."""
        return self.forward_backward(tokens, teacher_states, update=True)

    def forward_backward(self, tokens: torch.Tensor, teacher_states: torch.Tensor | None = None,
                         update: bool = False, _checked: bool = False):
        """The step up to the (rank-averaged) gradients in self.flat.grad, plus the
        optimizer update when `update`.  Returns the loss (device scalar)."""
        if not _checked:
            check_tokens(tokens, self.shape.vocab)
        tokens = self._to_device(tokens)
        teacher_states = self._to_device(teacher_states)
        inp, tgt = tokens[:, :-1], tokens[:, 1:]
        B, T = inp.shape
        M, d = B * T, self.shape.d_model
        lib = _lib.lib()
        world = dist.get_world_size(self.group) if (self.group is not None or (
            dist.is_available() and dist.is_initialized())) else 1
        pending = []
        overlapping = [False]

        def reduce_span(span):
            works = allreduce_mean_async(span, self.group)
            if works and not overlapping[0]:
                _lib.check(lib.ksd8_set_sm_reserve(DRAFT_SM_RESERVE), "set_sm_reserve")
                overlapping[0] = True
            pending.append(works)

        try:
            loss = self._run(inp, tgt, teacher_states, B, T, M, d, reduce_span, world)
            self._mark("reduce_wait")
            self._finish_grads(pending)
            if update:
                self._update()
            self._mark("end")
        finally:
            if overlapping[0]:
                lib.ksd8_set_sm_reserve(0)
        return loss

    def _run(self, inp, tgt, teacher_states, B, T, M, d, reduce_span, world):
        s = self.shape
        act = self.act
        E = self.flat.p("embedding.weight")
        ids = inp.reshape(-1)
        tids = tgt.reshape(-1)

        # ---- forward: embedding, input norm, teacher projection (draft.py:68-74)
        self._mark("embed_fwd")
        x0 = E.index_select(0, ids).to(act).requires_grad_(True)
        with torch.enable_grad():
            x1 = self._ln(x0, "input_norm")
        x = x1.detach()
        ts_saved = None
        if teacher_states is not None:
            # teacher_proj(states.to(weight dtype)): quantised from the states' exact values
            tsf = teacher_states.reshape(M, s.teacher_dim)
            tq, tsc = quantize_last_dim(tsf)
            wq, ws = quantize_last_dim(self.flat.p("teacher_proj.weight"))
            tqp, wqp = _validate_and_pad(tq, tsc, wq, ws, GROUP_SIZE)
            x = x + gemm_out(tqp, tsc, wqp, ws, out_dtype=act)      # Int8Linear fwd
            ts_saved = (tq, tsc)

        # ---- blocks: Rosa, DSpine injection + ln_ffn, KS3 (block.py:34-42)
        saved = []
        p_first = None
        t_norm = F.normalize(E.index_select(0, tids).float(), dim=-1)   # transfer targets
        ts_terms = []
        for layer in range(s.layers):
            pre = f"blocks.{layer}."
            self._mark("rosa_fwd")
            r, rosa_saved = self._rosa_forward(layer, x.view(B, T, d))
            self._mark("dspine_ln_fwd")
            iw = injection.InjectionWeights(self._dspine_weights(layer), act)
            b, h2, p, inj_saved = injection.forward(
                x + r, p_first, iw, self.flat.p(pre + "ln_ffn.weight"),
                self.flat.p(pre + "ln_ffn.bias"), B, T)
            term, rows = injection.transfer_rows(p, t_norm)
            ts_terms.append(term.mean())
            self._mark("ks3_fwd")
            k, ks3_saved = ks3_train_forward(self.cells[layer], b)
            del b
            x = h2 + k
            saved.append((rosa_saved, inj_saved, rows, ks3_saved))
            p_first = p.view(B, T, d)[:, 0]

        # ---- head + loss (draft.py:82, train/__init__.py:77-94)
        self._mark("head_fwd")
        xL = x.detach().requires_grad_(True)
        with torch.enable_grad():
            xf = self._ln(xL, "output_norm")
        if self.head_mode == "float":
            xf32 = xf.detach().float()
            with _ste_matmul_precision(torch.float32):
                logits = xf32 @ E.t()                                  # (M, V) fp32
        else:
            xfq, xfs = quantize_last_dim(xf.detach())
            Eq, Es = quantize_last_dim(E)
            logits = gemm_out(xfq, xfs, Eq, Es)                       # (M, V) fp32
        mx, sm, tg = ce_partials(logits, tids, 0)
        gmax, gsum, loss_rows = combine_ce_partials(mx, sm, tg, None)
        ce = loss_rows.mean()
        ts = torch.stack(ts_terms).sum() / max(1, s.layers)
        loss = ce + self.transfer_weight * ts
        self.last = {"ce": ce.detach(), "transfer": ts.detach()}

        # ---- backward: head (W8A8 dgrad / wgrad on the fused CE gradient codes)
        self._mark("head_bwd")
        if self.head_mode == "float":
            dl = ce_grad(logits, tids, 0, gmax, gsum, 1.0 / M)
            del logits
            with _ste_matmul_precision(torch.float32):
                dxf = dl @ E
                torch.matmul(dl.t(), xf32, out=self.flat.g("embedding.weight"))
            del dl
        else:
            dq, dsc, dlT_q, dlT_s = ce_grad_quant(logits, tids, 0, gmax, gsum, 1.0 / M)
            del logits
            EqT = quantize_cols(Eq, x_scales=Es)
            EqT = (F.pad(EqT[0], (0, -EqT[0].shape[1] % GROUP_SIZE)), EqT[1])
            dxf = gemm_out(dq, dsc, *EqT, out_dtype=torch.float32)
            xfT = quantize_cols(xfq, x_scales=xfs)
            xfT = (F.pad(xfT[0], (0, -M % GROUP_SIZE)), xfT[1])
            gemm_out(dlT_q, dlT_s, *xfT, out=self.flat.g("embedding.weight"))  # tied: dE = dW
        reduce_span(self.flat.g("embedding.weight"))
        with torch.enable_grad():
            xf.backward(dxf.to(act))
        self._ln_param_grads("output_norm")
        reduce_span(self.flat.span("output_norm.weight", "output_norm.bias"))
        dx = xL.grad.reshape(M, d).float()

        # ---- backward: blocks
        coef = self.transfer_weight / max(1, s.layers) / M
        dt_norm = torch.zeros(M, d, dtype=torch.float32, device=self.dev)
        dp_next_first = None
        n_parts = max(1, min(M, 4 * torch.cuda.get_device_properties(self.dev)
                                 .multi_processor_count))
        for layer in reversed(range(s.layers)):
            (rosa_saved, inj_saved, rows, ks3_saved) = saved[layer]
            pre = f"blocks.{layer}."
            cell = self.cells[layer]
            views = {n: self.flat.g(pre + KS3_MASTERS[n]).view_as(getattr(cell, "master_" + n))
                     for n in KS3_MASTERS}
            self._mark("ks3_bwd")
            db = ks3_backward(cell, dx.to(act), *ks3_saved, (M, d), grads_into=views)
            self._mark("dspine_ln_bwd")
            grads = {n: self.flat.g(pre + _dspine_name(n)) for n in DSPINE}
            grads["ln_w"] = self.flat.g(pre + "ln_ffn.weight")
            grads["ln_b"] = self.flat.g(pre + "ln_ffn.bias")
            # injection + ln_ffn backward, with this block's transfer-space term
            dh, dp_next_first = injection.backward(
                inj_saved, db.reshape(M, d), dx, B, T, t_norm, dt_norm, rows, coef,
                dp_next_first, grads, n_parts)
            self._mark("rosa_bwd")
            self._rosa_backward(layer, dh, rosa_saved)
            reduce_span(self.flat.block_grad_span(layer))
            dx = dh
            saved[layer] = None

        # ---- backward: teacher projection, input norm, embedding rows
        self._mark("embed_bwd")
        if ts_saved is not None:
            with _ste_matmul_precision(self.act):
                torch.matmul(dx.t(), dequantize_last_dim(*ts_saved),
                             out=self.flat.g("teacher_proj.weight"))
        else:
            self.flat.g("teacher_proj.weight").zero_()
        with torch.enable_grad():
            x1.backward(dx.to(act))
        self._ln_param_grads("input_norm")
        reduce_span(self.flat.span("teacher_proj.weight", "input_norm.bias"))
        rows = torch.cat([x0.grad.float(),
                          _normalize_bwd(E.index_select(0, tids).float(), dt_norm)])
        self._embedding_rows(torch.cat([ids, tids]), rows, world)
        return loss

    def _embedding_rows(self, ids, rows, world):
        """The sparse embedding gradient rows (input gather and transfer targets) of
        every rank, scaled for the mean; added after the dense head gradient's mean."""
        self._sparse = gather_sparse_rows(ids, rows, world, self.group)

    def _finish_grads(self, pending):
        for works in pending:
            wait_all(works)
        ids, rows = self._sparse
        self.flat.g("embedding.weight").index_add_(0, ids, rows)

    def _update(self):
        self._mark("clip_adamw")
        self.step_count += 1
        lib = _lib.lib()
        stream = _lib.stream_ptr(self.dev)
        scale = None
        if self.grad_clip:
            rc = lib.ksd8_grad_clip_coef(self.flat.grad.data_ptr(), self.flat.numel,
                                         float(self.grad_clip), self._clip_scratch.data_ptr(),
                                         self._clip_out.data_ptr(), None, stream)
            _lib.check(rc, "grad_clip_coef")
            scale = self._clip_out[1:2]
        args = (self.flat.data.data_ptr(), self.flat.grad.data_ptr(), _lib.F32,
                self.m.data_ptr(), self.v.data_ptr(), self.flat.numel, self.lr, 0.9, 0.999, 1e-8,
                self.wd, self.step_count)
        if scale is None:
            rc = lib.ksd8_adamw_step(*args, None, stream)
        else:
            rc = lib.ksd8_adamw_step_scaled(*args, scale.data_ptr(), None, stream)
        _lib.check(rc, "adamw_step")

    @property
    def last_grad_norm(self) -> torch.Tensor:
        return self._clip_out[0]
