"""Vocab-sharded W8A8 LM head: cross-entropy training loss and top-k drafting.

The reference head is the tied fp32 ``nn.Linear(d_model, vocab)`` of
ksdraft/model/draft.py:39,51,82, trained with ``F.cross_entropy(logits,
targets)`` (mean over rows, ksdraft/train/__init__.py:77) and a float
exception of the int8 tier (ksdraft/model/int8_convert.py:8-12).  Here the
head runs on the INT8 path with Int8Linear semantics (per-token GS128
activations x per-row GS128 weights, ksdraft/kernels/linear.py:67-73) and its
rows (the vocabulary) are split across the ranks of a process group:

* each rank holds a contiguous vocab shard whose boundaries sit on 128-row
  groups (150144 = 1173 x 128), so every GEMM of the backward keeps K % 128;
* forward: logits shard (M, V_local) fp32 by ksd8_w8a8_gemm, reduced on the
  device to (max, sum exp, target logit) per row by ksd8_ce_partials; the ranks
  combine those (M)-vectors with three all-reduces (max, sum, sum) -- no
  logits cross the interconnect;
* backward: ksd8_ce_grad gives the shard's dlogits; dx = q(dlogits) @
  q(W^T)^T (all-reduced over ranks), dW_shard = q(dlogits^T) @ q(x^T)^T, both
  W8A8 GS128 as the KS3 cell's backward (ksdraft/kernels/ks3_int8.py:410-424);
* drafting: per-rank top-k of the logits shard (ksd8_topk_rows), all-gather of
  the k candidates, and the same kernel merges them.
"""

from __future__ import annotations

import torch
import torch.distributed as dist

from .. import _lib
from ..kernels.gemm import gemm_out
from ..kernels.quant import GROUP_SIZE, quantize_cols, quantize_last_dim


def vocab_shard(vocab: int, rank: int, world: int, group: int = GROUP_SIZE) -> tuple[int, int]:
    """(start, size) of rank's vocab shard: whole 128-row groups, split as evenly
    as possible; the last shard takes the partial group when vocab % 128."""
    n_groups = (vocab + group - 1) // group
    g0 = n_groups * rank // world
    g1 = n_groups * (rank + 1) // world
    start = g0 * group
    return start, min(g1 * group, vocab) - start


def _world(group) -> tuple[int, int]:
    if group is None or not dist.is_available() or not dist.is_initialized():
        return 0, 1
    return dist.get_rank(group), dist.get_world_size(group)


def combine_ce_partials(mx: torch.Tensor, sm: torch.Tensor, tg: torch.Tensor, group=None):
    """Global per-row (max, sum exp, target logit) from every rank's shard
    partials.  Returns (gmax, gsum, loss_rows) with loss_row = log(gsum) + gmax
    - target_logit, the cross-entropy of that row over the whole vocabulary."""
    _, world = _world(group)
    gmax = mx.clone()
    if world > 1:
        dist.all_reduce(gmax, op=dist.ReduceOp.MAX, group=group)
    gsum = sm * torch.exp(mx - gmax)
    tgt = tg.clone()
    if world > 1:
        dist.all_reduce(gsum, group=group)
        dist.all_reduce(tgt, group=group)
    return gmax, gsum, torch.log(gsum) + gmax - tgt


def ce_partials(logits: torch.Tensor, targets: torch.Tensor, vstart: int):
    """Device (max, sum exp, target logit) per row of a logits shard."""
    _lib.require_cuda(logits, targets)
    M, V = logits.shape
    mx = torch.empty(M, dtype=torch.float32, device=logits.device)
    sm = torch.empty_like(mx)
    tg = torch.empty_like(mx)
    t = targets.to(torch.int64).contiguous()
    rc = _lib.lib().ksd8_ce_partials(logits.data_ptr(), _lib.dtype_code(logits), M, V,
                                     logits.stride(0) if M > 1 else V, t.data_ptr(), vstart,
                                     mx.data_ptr(), sm.data_ptr(), tg.data_ptr(), None,
                                     _lib.stream_ptr(logits.device))
    _lib.check(rc, "ce_partials")
    return mx, sm, tg


def ce_grad(logits: torch.Tensor, targets: torch.Tensor, vstart: int, gmax: torch.Tensor,
            gsum: torch.Tensor, scale: float) -> torch.Tensor:
    """(softmax - onehot) * scale over one logits shard (fp32)."""
    _lib.require_cuda(logits, targets)
    M, V = logits.shape
    d = torch.empty(M, V, dtype=torch.float32, device=logits.device)
    t = targets.to(torch.int64).contiguous()
    rc = _lib.lib().ksd8_ce_grad(logits.data_ptr(), _lib.dtype_code(logits), M, V,
                                 logits.stride(0) if M > 1 else V, t.data_ptr(), vstart,
                                 gmax.contiguous().data_ptr(), gsum.contiguous().data_ptr(),
                                 float(scale), d.data_ptr(), V, None,
                                 _lib.stream_ptr(logits.device))
    _lib.check(rc, "ce_grad")
    return d


def ce_grad_quant(logits: torch.Tensor, targets: torch.Tensor, vstart: int, gmax: torch.Tensor,
                  gsum: torch.Tensor, scale: float):
    """The shard's dlogits ((softmax - onehot) * scale) quantised along the
    vocabulary (M, Vp) and along the tokens (V_local, Mp), both zero-padded to
    multiples of 128 for the backward GEMMs; the codes equal quantize_last_dim /
    quantize_cols of ce_grad's fp32 output."""
    _lib.require_cuda(logits, targets)
    M, V = logits.shape
    Vp, Mp = -(-V // GROUP_SIZE) * GROUP_SIZE, -(-M // GROUP_SIZE) * GROUP_SIZE
    dev = logits.device
    dq = torch.empty(M, Vp, dtype=torch.int8, device=dev)
    dqs = torch.empty(M, Vp // GROUP_SIZE, dtype=torch.float16, device=dev)
    dqt = torch.empty(V, Mp, dtype=torch.int8, device=dev)
    dqts = torch.empty(V, Mp // GROUP_SIZE, dtype=torch.float16, device=dev)
    t = targets.to(torch.int64).contiguous()
    rc = _lib.lib().ksd8_ce_grad_quant(
        logits.data_ptr(), _lib.dtype_code(logits), M, V, logits.stride(0) if M > 1 else V,
        t.data_ptr(), vstart, gmax.contiguous().data_ptr(), gsum.contiguous().data_ptr(),
        float(scale), dq.data_ptr(), Vp, dqs.data_ptr(), dqt.data_ptr(), Mp, dqts.data_ptr(),
        None, _lib.stream_ptr(dev))
    _lib.check(rc, "ce_grad_quant")
    return dq, dqs, dqt, dqts


def topk_rows(vals: torch.Tensor, k: int, offset: int = 0, ids: torch.Tensor | None = None):
    """Per-row top-k of a (M, C) tensor: (values fp32 (M, k), ids int64 (M, k)),
    descending, ties to the smaller id; ids = offset + column or ids[row, col]."""
    _lib.require_cuda(vals)
    M, C = vals.shape
    if vals.stride(-1) != 1:
        vals = vals.contiguous()
    if ids is not None:
        ids = ids.to(torch.int64).contiguous()
        if ids.shape != vals.shape or vals.stride(0) != C:
            vals = vals.contiguous()
    ov = torch.empty(M, k, dtype=torch.float32, device=vals.device)
    oi = torch.empty(M, k, dtype=torch.int64, device=vals.device)
    rc = _lib.lib().ksd8_topk_rows(vals.data_ptr(), _lib.dtype_code(vals), _lib.ptr(ids), M, C,
                                   vals.stride(0) if M > 1 else C, k, offset, ov.data_ptr(),
                                   oi.data_ptr(), None, _lib.stream_ptr(vals.device))
    _lib.check(rc, "topk_rows")
    return ov, oi


def gather_topk(v: torch.Tensor, i: torch.Tensor, k: int, group=None, select=topk_rows):
    """Merge every rank's (M, k) top-k candidates into the global top-k: one
    all-gather of values and ids, then `select` (the top-k kernel) over the
    world * k candidates per row."""
    _, world = _world(group)
    if world == 1:
        return v, i
    vs = [torch.empty_like(v) for _ in range(world)]
    is_ = [torch.empty_like(i) for _ in range(world)]
    dist.all_gather(vs, v.contiguous(), group=group)
    dist.all_gather(is_, i.contiguous(), group=group)
    return select(torch.cat(vs, 1), k, ids=torch.cat(is_, 1))


def _pad_k(t: torch.Tensor) -> torch.Tensor:
    pad = -t.shape[-1] % GROUP_SIZE
    return torch.nn.functional.pad(t, (0, pad)) if pad else t


def check_targets(targets: torch.Tensor, vocab: int) -> None:
    """Targets must index the vocabulary: F.cross_entropy raises on anything
    else.  Its ignore_index (-100) is rejected too: the reference trainer never
    produces such targets (ksdraft/train/__init__.py:75-77), and a silent
    mean over fewer rows would differ from what this head computes.  One host
    read of the min and max."""
    if targets.numel() == 0:
        return
    lo, hi = int(targets.min()), int(targets.max())
    if lo < 0 or hi >= vocab:
        raise ValueError(f"targets must lie in [0, {vocab}); got [{lo}, {hi}]"
                         + (" (ignore_index targets are not supported)" if lo == -100 else ""))


class _HeadCE(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, weight, targets, head):
        x2 = x.reshape(-1, x.shape[-1])
        wq, ws = head.weight_codes()
        xq, xs = quantize_last_dim(x2)
        logits = gemm_out(_pad_k(xq), xs, _pad_k(wq), ws)       # (M, V_local) fp32
        mx, sm, tg = ce_partials(logits, targets.reshape(-1), head.vstart)
        gmax, gsum, loss_rows = combine_ce_partials(mx, sm, tg, head.group)
        ctx.head = head
        ctx.x_shape, ctx.x_dtype = x.shape, x.dtype
        ctx.save_for_backward(x2, logits, targets.reshape(-1), gmax, gsum)
        return loss_rows.mean()

    @staticmethod
    def backward(ctx, grad_loss):
        head = ctx.head
        x2, logits, targets, gmax, gsum = ctx.saved_tensors
        M = logits.shape[0]
        # d(mean)/d(logit) = (softmax - onehot) / M, times the upstream scalar
        scale = float(grad_loss) / M
        # q(dl) along the vocabulary and along the tokens, straight from the
        # logits (dl itself is never written)
        dq, dsc, dlT_q, dlT_s = ce_grad_quant(logits, targets, head.vstart, gmax, gsum, scale)
        wT_q, wT_s = head.weight_codes_t()                       # (d, Vp) along V
        # dx = q(dl) @ q(W^T)^T over this shard's vocabulary, summed over ranks
        dx = gemm_out(dq, dsc, wT_q, wT_s)
        _, world = _world(head.group)
        if world > 1:
            dist.all_reduce(dx, group=head.group)
        # dW_shard = q(dl^T) @ q(x^T)^T, contracted over the tokens
        xT_q, xT_s = quantize_cols(x2)                           # (d, M)
        if head.tied is not None:
            # tied to the full embedding master: its gradient rows of this shard
            dw = torch.zeros_like(head.tied)
            gemm_out(dlT_q, dlT_s, _pad_k(xT_q), xT_s,
                     out=dw[head.vstart:head.vstart + head.v_local])
        else:
            dw = gemm_out(dlT_q, dlT_s, _pad_k(xT_q), xT_s)
        return dx.reshape(ctx.x_shape).to(ctx.x_dtype), dw, None, None


class VocabParallelHead(torch.nn.Module):
    """One rank's vocab shard of a W8A8 GS128 LM head.

    weight: either the tied embedding master itself -- a (vocab, d) fp32
    nn.Parameter, as the reference ties head and embedding (draft.py:51) -- in
    which case the head reads its rows [vstart, vstart + V_local) in place and
    its weight gradient lands in those rows of the embedding's gradient (zero
    elsewhere), so embedding and head stay one tensor; or a plain tensor (the
    full master, or this rank's (V_local, d) shard with `vstart` given), copied
    into an untied fp32 parameter of the shard.  Codes are re-quantised when
    the master's version changes (in-place torch updates); code that updates it
    outside torch calls invalidate()."""

    def __init__(self, weight: torch.Tensor, vocab: int | None = None, group=None,
                 vstart: int | None = None):
        super().__init__()
        rank, world = _world(group)
        self.group = group
        self.vocab = int(vocab if vocab is not None else weight.shape[0])
        tie = isinstance(weight, torch.nn.Parameter) and vstart is None and \
            weight.dtype == torch.float32 and weight.shape[0] == self.vocab
        if vstart is None:
            start, size = vocab_shard(self.vocab, rank, world)
        else:
            start, size = int(vstart), weight.shape[0]
        self.vstart = start
        self._size = size
        if tie:
            self.tied = weight                  # not registered again: the embedding owns it
            self._own = None
        else:
            self.tied = None
            shard = weight[start:start + size] if vstart is None else weight
            self._own = torch.nn.Parameter(shard.detach().float().clone())
        self._codes = None
        self._codes_t = None
        self._version = None

    @property
    def weight(self) -> torch.Tensor:
        """This rank's (V_local, d) fp32 rows (a view of the tied embedding)."""
        if self.tied is not None:
            return self.tied[self.vstart:self.vstart + self._size]
        return self._own

    @property
    def v_local(self) -> int:
        return self._size

    def invalidate(self) -> None:
        self._codes = None
        self._codes_t = None

    def weight_codes(self):
        """Per-row GS128 codes of the shard, re-quantised when the master changes."""
        src = self.tied if self.tied is not None else self._own
        v = src._version
        if self._codes is None or self._version != v:
            self._codes = quantize_last_dim(self.weight.detach())
            self._codes_t = None
            self._version = v
        return self._codes

    def weight_codes_t(self):
        """Codes of W^T (d, Vp) quantised along the vocabulary (zero-padded to a
        multiple of 128), cached with the row codes they are derived from."""
        wq, ws = self.weight_codes()
        if self._codes_t is None:
            tq, ts = quantize_cols(wq, x_scales=ws)
            self._codes_t = (_pad_k(tq), ts)
        return self._codes_t

    def logits(self, x: torch.Tensor) -> torch.Tensor:
        """This shard's logits (M, V_local) fp32 for x (..., d)."""
        x2 = x.reshape(-1, x.shape[-1])
        xq, xs = quantize_last_dim(x2)
        wq, ws = self.weight_codes()
        return gemm_out(_pad_k(xq), xs, _pad_k(wq), ws)

    def cross_entropy(self, x: torch.Tensor, targets: torch.Tensor) -> torch.Tensor:
        """Mean cross-entropy over the whole vocabulary (all ranks' shards)."""
        check_targets(targets, self.vocab)
        master = self.tied if self.tied is not None else self._own
        return _HeadCE.apply(x, master, targets, self)

    def topk(self, x: torch.Tensor, k: int):
        """Global top-k (values, vocab ids) per row over every rank's shard."""
        v, i = topk_rows(self.logits(x), k, offset=self.vstart)
        return gather_topk(v, i, k, self.group)
