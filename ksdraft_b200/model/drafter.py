"""Drafting with a KSDraft model on the INT8 tier (benchmark config 5).

The reference describes a proposal API on the draft model,
`propose(target_states, tokens, block_len, topk) -> candidates, logits, refined`
(RESEARCH.md section B), but only implements whole-sequence forwards
(KSDraftModel.forward, ksdraft/model/draft.py:58-82, with the int8 tier of
ksdraft/model/int8_convert.py).  KSDraftDrafter keeps per-context state so
that appending a block of positions costs only those positions:

  prefill(tokens, teacher_states)   whole-context forward (C contexts x T0
                                    positions), then the per-layer caches
  propose(target_states, tokens, k) append a block (C x n positions, the
                                    parallel draft block) and return the top-k
                                    next-token candidates and logits at each
                                    appended position

The forward is the int8 tier's: Int8Linear W8A8 for the Rosa q/k/v/out and
teacher projections, the all-INT8 KS3 cells, the DSpine injection and
LayerNorms as float exceptions in the activation dtype, and the tied LM head
W8A8 (the north star's vocab-sharded head).  What each appended position sees
equals the whole-sequence forward of the extended context:

  * Rosa time-shift mix: the previous position's ln_attn output is cached per
    layer (rosa.py:128-133);
  * Rosa matching: ksd8_rosa_decode_step answers the new positions against
    every earlier key (bit histories plus a sorted run of the context's keys,
    rebuilt when the appended delta outgrows the step kernel's window);
  * DSpine: the previous position's predicted feature p is cached per layer
    (spine.py:64-66); position 0 of a prefill takes the previous layer's
    feature as in KSDraftModel.forward;
  * everything else is per position.

Data parallel serving: with a process group the contexts are split over the
ranks for the 24 layers, the final hidden states are all-gathered, and every
rank scores all rows against its vocabulary shard (VocabParallelHead); the
per-shard top-k are merged by one all-gather.
"""

from __future__ import annotations

from types import SimpleNamespace

import torch
import torch.distributed as dist
import torch.nn.functional as F

from .. import _lib
from ..kernels.gemm import _validate_and_pad, gemm_out
from ..kernels.ks3_int8 import KS3Int8Cell, ks3_weights
from ..kernels.quant import GROUP_SIZE, quantize_last_dim
from ..train import injection
from .head import VocabParallelHead, gather_topk, topk_rows
from .rosa import pack_bits

MAX_LEN = 62            # the reference's cap min(62, T - 1) once T >= 63
DELTA_WORDS = 34        # k words of the appended delta the step kernel holds
MERGE_MAX = 8192        # appended keys one merge sorts in shared memory
LN_EPS = 1e-5


class RosaDecodeState:
    """One layer's matcher state for `rows` = contexts x streams (row = c * S + s):
    q / k / v bit histories and the sorted key run of the matched context."""

    def __init__(self, contexts: int, streams: int, capacity: int, device):
        if capacity % 64:
            raise ValueError("capacity must be a multiple of 64 positions")
        self.contexts, self.streams, self.capacity = contexts, streams, capacity
        rows = contexts * streams
        self.nw = capacity // 64
        self.bits = [torch.zeros(rows, self.nw, dtype=torch.int64, device=device)
                     for _ in range(3)]
        self.sw = torch.empty(rows, capacity, dtype=torch.int64, device=device)
        self.sj = torch.empty(rows, capacity, dtype=torch.int16, device=device)
        self.blk = torch.zeros(rows, capacity // 64, dtype=torch.int16, device=device)
        # sample index: windows of every 64th, then every 8th rank of the run
        self.smp = torch.zeros(rows, capacity // 64 + capacity // 8, dtype=torch.int64,
                               device=device)
        self.n_main = 0
        self.pos = None        # device [t0, n_main] read by the step kernel (CUDA graphs)

    def load_words(self, words, t_len: int) -> None:
        """Bit histories from packed words (rows, ceil(t_len / 64)) of a whole context."""
        if t_len > self.capacity:
            raise ValueError(f"context of {t_len} positions exceeds capacity {self.capacity}")
        for dst, src in zip(self.bits, words):
            dst.zero_()
            dst[:, :src.shape[1]].copy_(src)

    def build(self, n_keys: int) -> None:
        """Main run of the keys of positions max_len - 1 .. n_keys - 1: the keys
        appended since the last build merged into the current run when there is
        one (a copy of it is the merge's input), else all keys sorted."""
        rows = self.contexts * self.streams
        lib, stream = _lib.lib(), _lib.stream_ptr(self.sw.device)
        n_old = self.n_main
        if MAX_LEN - 1 < n_old <= n_keys and n_keys - n_old <= MERGE_MAX:
            sw_in, sj_in = self.sw.clone(), self.sj.clone()
            _lib.check(lib.ksd8_rosa_decode_merge(
                self.bits[1].data_ptr(), rows, self.nw, n_old, n_keys, MAX_LEN,
                sw_in.data_ptr(), sj_in.data_ptr(), self.sw.data_ptr(), self.sj.data_ptr(),
                self.blk.data_ptr(), self.smp.data_ptr(), self.capacity, None, stream),
                "rosa_decode_merge")
        else:
            _lib.check(lib.ksd8_rosa_decode_build(
                self.bits[1].data_ptr(), rows, self.nw, n_keys, MAX_LEN, self.sw.data_ptr(),
                self.sj.data_ptr(), self.blk.data_ptr(), self.smp.data_ptr(), self.capacity,
                None, stream),
                "rosa_decode_build")
        self.n_main = n_keys

    def needs_build(self, t0: int, k_new: int) -> bool:
        """True when the delta keys of a step at t0 would not fit the step kernel."""
        dlo = max(self.n_main, MAX_LEN - 1)
        dhi = t0 + k_new - 2
        if dhi < dlo:
            return False
        w0 = (dlo >> 6) - 1 if dlo > 63 else 0
        return (dhi >> 6) - w0 + 1 > DELTA_WORDS

    def _step(self, projs, t0: int, k_new: int, pay, out, out_cs: int, out_dt: int, ml, me,
              ml_rs: int, prepared: bool = False):
        if not prepared and self.needs_build(t0, k_new):
            self.build(t0)
        if t0 + k_new > self.capacity:
            raise ValueError("decode state capacity exhausted")
        C, S = self.contexts, self.streams
        ptrs = (None, None, None) if projs is None else tuple(p.data_ptr() for p in projs)
        dt = _lib.dtype_code(projs[0]) if projs is not None else 0
        _lib.check(_lib.lib().ksd8_rosa_decode_step(
            *ptrs, dt, C, S, k_new, t0, self.n_main, MAX_LEN,
            *(b.data_ptr() for b in self.bits), self.nw, self.sw.data_ptr(), self.sj.data_ptr(),
            self.blk.data_ptr(), self.smp.data_ptr(), self.capacity, pay.data_ptr(), out,
            out_cs, out_dt, ml, me,
            ml_rs, _lib.ptr(self.pos), None,
            _lib.stream_ptr(self.sw.device)), "rosa_decode_step")

    def step(self, projs, t0: int, payload: torch.Tensor, out: torch.Tensor,
             match_len=None, match_end=None, prepared: bool = False) -> None:
        """Append the bits of projs (3 x (contexts, k_new, streams)) at t0 and write
        payload * sign of the new positions into out (contexts, k_new, streams);
        match_len / match_end (rows, k_new) int32 optional.  prepared: the caller
        has already rebuilt the main run if the step needed it."""
        C, k_new, S = projs[0].shape
        self._step(projs, t0, k_new, payload.detach().float().contiguous(), out.data_ptr(),
                   k_new * S, _lib.dtype_code(out), _lib.ptr(match_len), _lib.ptr(match_end),
                   k_new, prepared)

    def match_context(self, t_len: int, payload: torch.Tensor, out: torch.Tensor,
                      match_len=None, match_end=None) -> None:
        """Match a whole context already in the bit histories (load_words), 32
        positions per launch with the main run rebuilt as it grows: out
        (contexts, t_len, streams) payload * sign, match_len / match_end
        (rows, t_len) int32 optional -- the sequence matcher's results, in
        O(log T) per position whatever the bit statistics."""
        S = self.streams
        pay = payload.detach().float().contiguous()
        self.n_main = 0
        esz = out.element_size()
        for t0 in range(0, t_len, 32):
            k = min(32, t_len - t0)
            ml = match_len.data_ptr() + 4 * t0 if match_len is not None else None
            me = match_end.data_ptr() + 4 * t0 if match_end is not None else None
            self._step(None, t0, k, pay, out.data_ptr() + esz * t0 * S, t_len * S,
                       _lib.dtype_code(out), ml, me, t_len)


def _int8_linear(w: torch.Tensor):
    """GS128 codes of an nn.Linear weight (out, in): Int8Linear's weight pack."""
    return quantize_last_dim(w.detach().float())


def _linear_int8(x2: torch.Tensor, w, bias=None, out_dtype=torch.float32):
    """Int8Linear.forward (linear.py:67-73): per-token GS128 codes of x, W8A8 GEMM,
    fp32 bias in the epilogue."""
    xq, xs = quantize_last_dim(x2)
    xq, wq = _validate_and_pad(xq, xs, w[0], w[1], GROUP_SIZE)
    return gemm_out(xq, xs, wq, w[1], out_dtype=out_dtype, bias=bias)


class KSDraftDrafter:
    """Serving-time INT8 draft model over `contexts` concurrent contexts.

    state: {reference state-dict name: fp32 tensor} of a KSDraftModel
    (ksdraft/model/draft.py, head tied to embedding.weight), e.g.
    DraftTrainStep.parameter_dict() or a reference checkpoint.  shape: its
    DraftShape.  capacity: positions per context the caches hold (prefill +
    appended blocks).  group: process group to split the contexts over (the
    vocabulary is sharded over the same ranks)."""

    def __init__(self, state: dict, shape, device, *, contexts: int, capacity: int,
                 act_dtype=torch.bfloat16, group=None, head_mode: str = "w8a8"):
        injection.check_width(shape.d_model)
        if head_mode not in ("w8a8", "float"):
            raise ValueError("head_mode is 'w8a8' (north star) or 'float' (the reference "
                             "int8 tier's float head, int8_convert.py:8-12)")
        self.head_mode = head_mode
        self.shape, self.dev, self.act = shape, torch.device(device), act_dtype
        self.group = group
        self.world = dist.get_world_size(group) if (group is not None or (
            dist.is_available() and dist.is_initialized())) else 1
        self.rank = dist.get_rank(group) if self.world > 1 else 0
        if contexts % self.world:
            raise ValueError(f"{contexts} contexts do not split over {self.world} ranks")
        self.contexts = contexts
        self.c_local = contexts // self.world
        self.capacity = (capacity + 63) // 64 * 64
        dev = self.dev
        P = lambda n: torch.as_tensor(state[n]).to(dev, torch.float32)  # noqa: E731
        with torch.no_grad():
            self.E = P("embedding.weight").contiguous()
            self.input_norm = (P("input_norm.weight"), P("input_norm.bias"))
            self.output_norm = (P("output_norm.weight"), P("output_norm.bias"))
            self.teacher = (_int8_linear(P("teacher_proj.weight"))
                            if "teacher_proj.weight" in state else None)
            self.layers = []
            for l in range(shape.layers):
                pre = f"blocks.{l}."
                R = lambda n: P(pre + "rosa." + n)  # noqa: E731,B023
                cell = KS3Int8Cell(ks3_weights(P(pre + "ffn.down.weight"), P(pre + "ffn.up.weight"),
                                               P(pre + "ffn.coefficients"),
                                               P(pre + "ffn.raw_scale"), P(pre + "ffn.raw_shift")),
                                   nonlinear="int8", trainable=False)
                W = {n: P(pre + "injection." + (n if n == "gate_bias" else n + ".weight"))
                     for n in ("feature_down", "feature_up", "gate_q.down", "gate_q.up",
                               "gate_p.down", "gate_p.up", "gate_bias", "inject.down",
                               "inject.up")}
                self.layers.append(SimpleNamespace(
                    ln_attn=(P(pre + "ln_attn.weight").to(act_dtype),
                             P(pre + "ln_attn.bias").to(act_dtype)),
                    mixes=[torch.sigmoid(R(f"time_mix_{c}")).contiguous() for c in "qkv"],
                    qkv=[_int8_linear(R(f"{c}_proj.weight")) for c in "qkv"],
                    qkv_bias=[R(f"{c}_proj.bias").contiguous() for c in "qkv"],
                    out=_int8_linear(R("out_proj.weight")),
                    out_bias=R("out_proj.bias").contiguous(),
                    payload=R("payload").contiguous(),
                    iw=injection.InjectionWeights(W, act_dtype),
                    ln_ffn=(P(pre + "ln_ffn.weight").contiguous(),
                            P(pre + "ln_ffn.bias").contiguous()),
                    cell=cell))
            self.head = VocabParallelHead(self.E, group=group if self.world > 1 else None)
        self.states = None
        self.length = 0
        self.pos = torch.zeros(2, dtype=torch.int64, device=self.dev)
        self._graph = None
        self.phase_marks = None   # a list to record (phase name, CUDA event) marks into
        self._capturing = False

    def _mark(self, name: str) -> None:
        """Start phase `name` (device-side timing of a block's parts; inside a
        recorded graph the events are graph nodes, re-recorded by every replay)."""
        if self.phase_marks is not None:
            ev = torch.cuda.Event(enable_timing=True, external=self._capturing)
            ev.record()
            self.phase_marks.append((name, ev))

    def phases(self, marks=None) -> dict:
        """ms per phase name over a list of marks (default: the recorded graph's)."""
        marks = self._g_marks if marks is None else marks
        out = {}
        for (name, ev), (_, nxt) in zip(marks, marks[1:]):
            out[name] = out.get(name, 0.0) + ev.elapsed_time(nxt)
        return out

    # ---- forward -------------------------------------------------------------

    def _layer(self, l: int, x: torch.Tensor, t0: int, p_first, prefill: bool,
               probe: dict | None = None, prepared: bool = False):
        """One DraftBlock (block.py:34-42) on this rank's contexts: x (C, n, d) at
        positions t0 .. t0 + n - 1.  Returns (x_out (C, n, d), p (C, n, d))."""
        L = self.layers[l]
        C, n, d = x.shape
        S = self.shape.streams
        dev, act = self.dev, self.act
        lib = _lib.lib()
        self._mark("rosa_proj")
        a = F.layer_norm(x, (d,), *L.ln_attn, LN_EPS)
        # time-shift mix with the previous position's ln_attn output (zero before
        # position 0): one leading row per context, whose own outputs are dropped
        prev = torch.zeros(C, 1, d, dtype=act, device=dev) if prefill else self.cache_a[l][:, None]
        ax = torch.cat([prev, a], 1).contiguous()
        rows = C * (n + 1)
        G = d // GROUP_SIZE
        codes = [torch.empty(rows, d, dtype=torch.int8, device=dev) for _ in range(3)]
        scales = [torch.empty(rows, G, dtype=torch.float16, device=dev) for _ in range(3)]
        _lib.check(lib.ksd8_rosa_timemix_quantize(
            ax.data_ptr(), _lib.dtype_code(ax), C, n + 1, d, *(m.data_ptr() for m in L.mixes),
            codes[0].data_ptr(), scales[0].data_ptr(), codes[1].data_ptr(), scales[1].data_ptr(),
            codes[2].data_ptr(), scales[2].data_ptr(), None, _lib.stream_ptr(dev)),
            "rosa_timemix_quantize")
        # q / k / v projections in fp32 (the promoted dtype of rosa.py:128-133)
        projs = [gemm_out(codes[i], scales[i], *L.qkv[i], out_dtype=torch.float32,
                          bias=L.qkv_bias[i]).view(C, n + 1, S)[:, 1:].contiguous()
                 for i in range(3)]
        del codes, scales, ax
        self._mark("rosa_match")
        mixed = torch.empty(C, n, S, dtype=act, device=dev)
        st = self.states[l]
        ml = me = None
        if probe is not None:
            ml = torch.empty(C * S, n, dtype=torch.int32, device=dev)
            me = torch.empty_like(ml)
        if prefill:
            # the whole context through the decode matcher (O(log T) per position;
            # the sequence matchers' shared-memory kernels stop at 4096 / 8192)
            st.load_words([pack_bits(p, C, n, S, n * S, S, 1) for p in projs], n)
            st.match_context(n, L.payload, mixed, ml, me)
            st.build(n)
        else:
            st.step(projs, t0, L.payload, mixed, ml, me, prepared)
        if probe is not None:
            probe[l] = (ml, me, mixed)
        self._mark("rosa_out")
        r = _linear_int8(mixed.reshape(C * n, S), L.out, bias=L.out_bias, out_dtype=act)
        h = x.reshape(C * n, d) + r
        self._mark("injection_ln")
        b, h2, p, _ = injection.forward(h, p_first, L.iw, *L.ln_ffn, C, n)
        self._mark("ks3")
        k = L.cell(b)
        x_out = (h2 + k).view(C, n, d)
        p = p.view(C, n, d)
        self.cache_a[l].copy_(a[:, -1])
        self.cache_p[l].copy_(p[:, -1])
        return x_out, p

    def _input(self, tokens: torch.Tensor, states: torch.Tensor | None) -> torch.Tensor:
        """input_norm(E[tokens]) + teacher_proj(states) (draft.py:68-74), (C, n, d)."""
        C, n = tokens.shape
        d = self.shape.d_model
        x = F.layer_norm(self.E[tokens.reshape(-1)].to(self.act), (d,),
                         self.input_norm[0].to(self.act), self.input_norm[1].to(self.act),
                         LN_EPS)
        if states is not None:
            if self.teacher is None:
                raise ValueError("teacher_states passed but the model has no teacher_proj")
            x = x + _linear_int8(states.reshape(C * n, -1), self.teacher, out_dtype=self.act)
        return x.view(C, n, d)

    def _local(self, t: torch.Tensor | None) -> torch.Tensor | None:
        """This rank's contexts of a (contexts, ...) tensor, on the device."""
        if t is None:
            return None
        if t.shape[0] != self.contexts:
            raise ValueError(f"expected {self.contexts} contexts, got {t.shape[0]}")
        t = t[self.rank * self.c_local:(self.rank + 1) * self.c_local]
        return t.to(self.dev, non_blocking=True)

    def _topk(self, xl: torch.Tensor, k: int):
        """Head top-k of final hidden states xl (rows of this rank's contexts):
        gathered over the ranks, scored against every vocabulary shard."""
        d = self.shape.d_model
        xf = F.layer_norm(xl, (d,), self.output_norm[0].to(self.act),
                          self.output_norm[1].to(self.act), LN_EPS).reshape(-1, d)
        if self.world > 1:
            parts = [torch.empty_like(xf) for _ in range(self.world)]
            dist.all_gather(parts, xf.contiguous(), group=self.group)
            xf = torch.cat(parts)
        if self.head_mode == "float":
            logits = xf.float() @ self.head.weight.t()
            v, i = topk_rows(logits, k, offset=self.head.vstart)
            return gather_topk(v, i, k, self.group if self.world > 1 else None)
        return self.head.topk(xf, k)

    def _check_tokens(self, tokens: torch.Tensor) -> None:
        lo, hi = int(tokens.min()), int(tokens.max())
        if lo < 0 or hi >= self.shape.vocab:
            raise ValueError(f"token ids must lie in [0, {self.shape.vocab}); got [{lo}, {hi}]")

    @torch.no_grad()
    def prefill(self, tokens: torch.Tensor, teacher_states: torch.Tensor | None = None,
                topk: int = 8, probe: dict | None = None):
        """Whole-context forward of (contexts, T0) tokens (T0 > 62); builds the
        caches and returns the top-k candidates (ids, logits) of every context's
        next token, (contexts, k) each."""
        self._check_tokens(tokens)
        C, T0 = tokens.shape
        if T0 <= MAX_LEN:
            raise ValueError(f"prefill needs more than {MAX_LEN} positions (the Rosa cap "
                             f"min(62, T - 1) is then fixed); got {T0}")
        if T0 > self.capacity:
            raise ValueError(f"{T0} positions exceed the capacity {self.capacity}")
        tok = self._local(tokens)
        sts = self._local(teacher_states)
        S = self.shape.streams
        self.states = [RosaDecodeState(self.c_local, S, self.capacity, self.dev)
                       for _ in self.layers]
        d = self.shape.d_model
        self.cache_a = [torch.empty(self.c_local, d, dtype=self.act, device=self.dev)
                        for _ in self.layers]
        self.cache_p = [torch.empty_like(c) for c in self.cache_a]
        self._graph = None
        x = self._input(tok, sts)
        p_first = None
        for l in range(len(self.layers)):
            x, p = self._layer(l, x, 0, p_first, True, probe)
            p_first = p[:, 0]
        self.length = T0
        vals, ids = self._topk(x[:, -1:], topk)
        return ids.view(C, topk), vals.view(C, topk)

    def _block(self, t0: int, tok, sts, topk: int, probe=None, prepared: bool = False):
        """Forward of one appended block of this rank's contexts + the head top-k."""
        self._mark("input")
        x = self._input(tok, sts)
        for l in range(len(self.layers)):
            x, _ = self._layer(l, x, t0, self.cache_p[l], False, probe, prepared)
        self._mark("head_topk")
        vals, ids = self._topk(x, topk)
        self._mark("end")
        return ids, vals

    def _prepare(self, t0: int, n: int) -> None:
        """Rebuild every layer's main run if a block at t0 would overflow the step
        kernel's delta window, and publish [t0, n_main] for a graph replay."""
        for st in self.states:
            if st.needs_build(t0, n):
                st.build(t0)
        self.pos.copy_(torch.tensor([t0, self.states[0].n_main], dtype=torch.int64))

    @torch.no_grad()
    def capture(self, n: int, topk: int = 8, with_states: bool = True,
                phase_marks: bool = False) -> None:
        """Record propose() of an n-position block as one CUDA graph (the per-layer
        launches of a decode step are small; replaying them removes the host
        cost).  The step kernel reads the position from device memory, so one
        recording serves every later block; main-run rebuilds stay outside the
        graph.  Call after prefill(); propose() with the same n / topk / teacher
        states presence replays it."""
        if self.states is None:
            raise RuntimeError("prefill() first")
        C, dev = self.c_local, self.dev
        t0 = self.length
        if t0 + n > self.capacity:
            raise ValueError("the caches are full (capacity positions per context)")
        self._g_tok = torch.zeros(C, n, dtype=torch.int64, device=dev)
        self._g_sts = (torch.zeros(C, n, self.shape.teacher_dim, dtype=self.act, device=dev)
                       if with_states else None)
        self._prepare(t0, n)
        for st in self.states:
            st.pos = self.pos
        # one eager pass first (library workspaces, lazily built state), then the
        # caches are restored: it appended placeholder bits at t0, which the
        # replays overwrite
        saved = [c.clone() for c in self.cache_a + self.cache_p]
        from ..kernels.gemm import GemmTimer
        timer, GemmTimer.active = GemmTimer.active, None   # a GEMM timer sees the graph only
        marks, self.phase_marks = self.phase_marks, None
        try:
            self._block(t0, self._g_tok, self._g_sts, topk, prepared=True)
        finally:
            GemmTimer.active = timer
            self.phase_marks = marks
        for c, v in zip(self.cache_a + self.cache_p, saved):
            c.copy_(v)
        torch.cuda.synchronize(dev)
        self._graph = torch.cuda.CUDAGraph()
        launches0 = _lib.LAUNCHES
        marks, self.phase_marks = self.phase_marks, ([] if phase_marks else None)
        self._capturing = True
        try:
            with torch.cuda.graph(self._graph, capture_error_mode="thread_local"):
                self._g_out = self._block(t0, self._g_tok, self._g_sts, topk, prepared=True)
        finally:
            self._capturing = False
            self._g_marks, self.phase_marks = self.phase_marks or [], marks
        self.captured_launches = _lib.LAUNCHES - launches0     # ksd8 kernels per replay
        self._g_key = (n, topk, with_states)
        torch.cuda.synchronize(dev)

    def rebuild(self) -> None:
        """Sort every layer's keys up to the current length into its main run now
        (propose() does it when a block would overflow the delta window)."""
        for st in self.states:
            st.build(self.length)

    @staticmethod
    def steps_per_rebuild(n: int) -> int:
        """Blocks of n positions appended between two main-run rebuilds."""
        return max(1, ((DELTA_WORDS - 2) * 64) // n)

    def release(self) -> None:
        """Drop the recorded graph (and the collectives it holds)."""
        self._graph = None
        if self.states is not None:
            for st in self.states:
                st.pos = None

    @torch.no_grad()
    def propose(self, target_states: torch.Tensor | None, tokens: torch.Tensor, topk: int = 8,
                probe: dict | None = None):
        """Append a block of n positions per context (tokens (contexts, n), n <= 32,
        their teacher states (contexts, n, teacher_dim) or None) and draft from
        it: returns (candidates (contexts, n, k) int64 vocab ids, logits
        (contexts, n, k) fp32, None) -- the top-k next tokens after each
        appended position; the third slot of the reference's signature
        (refined candidates) has no counterpart in the reference code."""
        if self.states is None:
            raise RuntimeError("prefill() first")
        self._check_tokens(tokens)
        C, n = tokens.shape
        if not 1 <= n <= 32:
            raise ValueError(f"a block holds 1..32 positions; got {n}")
        if self.length + n > self.capacity:
            raise ValueError("the caches are full (capacity positions per context)")
        t0 = self.length
        key = (n, topk, target_states is not None)
        if self._graph is not None and probe is None and key == self._g_key:
            self._prepare(t0, n)
            self._g_tok.copy_(self._local(tokens))
            if self._g_sts is not None:
                self._g_sts.copy_(self._local(target_states))
            self._graph.replay()
            ids, vals = (t.clone() for t in self._g_out)
        else:
            if self._graph is not None:
                self._prepare(t0, n)      # the recorded position must not go stale
            ids, vals = self._block(t0, self._local(tokens), self._local(target_states), topk,
                                    probe, prepared=self._graph is not None)
        self.length = t0 + n
        return ids.view(C, n, topk), vals.view(C, n, topk), None
