"""Data-parallel training step for INT8 KS3 layers (one process per GPU).

Every rank runs the same INT8 layer forward/backward on its own tokens; the
gradients of the fp32 masters land in one flat, bucket-aligned buffer (the
`.grad` of every master is a view into it), which is averaged across ranks
with a single NCCL all-reduce, then the ksd8 AdamW kernel updates the masters.
There is no other exchange: the path shards by tokens (weak scaling).

The host-side pieces (flat views, averaging, the failure check before the
collective) are plain torch and run on CPU `gloo` ranks in the tests.
"""

from __future__ import annotations

import datetime
import os

import torch
import torch.distributed as dist

from .. import _lib


class FlatGrads:
    """Points each parameter's .grad at a slice of one contiguous fp32 buffer."""

    def __init__(self, params: list[torch.nn.Parameter], align: int = 64):
        self.params = list(params)
        self.offsets = []
        off = 0
        for p in self.params:
            self.offsets.append(off)
            off += (p.numel() + align - 1) // align * align
        self.numel = off
        dev = self.params[0].device
        self.buffer = torch.zeros(off, dtype=torch.float32, device=dev)
        self.attach()

    def attach(self) -> None:
        for p, off in zip(self.params, self.offsets):
            p.grad = self.buffer[off:off + p.numel()].view_as(p)

    def zero_(self) -> None:
        self.buffer.zero_()
        self.attach()

    def views(self):
        for p, off in zip(self.params, self.offsets):
            yield p, self.buffer[off:off + p.numel()]

    def span(self, params) -> torch.Tensor:
        """The contiguous slice of the buffer covering `params` (and the zero
        padding between them)."""
        idx = [i for i, p in enumerate(self.params) if any(p is q for q in params)]
        lo = self.offsets[min(idx)]
        hi = self.offsets[max(idx)] + self.params[max(idx)].numel()
        return self.buffer[lo:hi]


def allreduce_mean_(buffer: torch.Tensor, group=None) -> None:
    """Average a flat gradient buffer over the ranks of `group` (no-op alone)."""
    if not dist.is_available() or not dist.is_initialized():
        return
    world = dist.get_world_size(group)
    if world == 1:
        return
    dist.all_reduce(buffer, op=dist.ReduceOp.SUM, group=group)
    buffer.div_(world)


def allreduce_mean_async(t: torch.Tensor, group=None):
    """Start averaging `t` over the ranks; returns a list of pending works whose
    wait() completes the mean in place (NCCL averages in the collective, gloo
    sums and the caller's wait_all divides).  Empty when running alone."""
    if not dist.is_available() or not dist.is_initialized():
        return []
    world = dist.get_world_size(group)
    if world == 1:
        return []
    if dist.get_backend(group) == "nccl":
        return [(dist.all_reduce(t, op=dist.ReduceOp.AVG, group=group, async_op=True), None)]
    return [(dist.all_reduce(t, op=dist.ReduceOp.SUM, group=group, async_op=True), (t, world))]


def wait_all(pending) -> None:
    for work, post in pending:
        work.wait()
        if post is not None:
            post[0].div_(post[1])


def check_finite_across_ranks(buffer: torch.Tensor, group=None) -> bool:
    """True when every rank's gradients are finite (one small all-reduce of a flag)."""
    ok = torch.isfinite(buffer).all().to(torch.int32).reshape(1)
    if dist.is_available() and dist.is_initialized() and dist.get_world_size(group) > 1:
        dist.all_reduce(ok, op=dist.ReduceOp.MIN, group=group)
    return bool(ok.item())


class AdamW:
    """torch.optim.AdamW semantics over fp32 params, one ksd8 kernel launch per tensor."""

    def __init__(self, params, lr=3e-4, betas=(0.9, 0.999), eps=1e-8, weight_decay=0.01):
        self.params = list(params)
        self.lr, self.betas, self.eps, self.wd = lr, betas, eps, weight_decay
        self.state = [(torch.zeros_like(p), torch.zeros_like(p)) for p in self.params]
        self.step_count = 0

    @torch.no_grad()
    def step(self) -> None:
        self.begin_step()
        for i in range(len(self.params)):
            self.update(i)

    def begin_step(self) -> None:
        """Advance the step count (bias correction) once; then update() each tensor."""
        self.step_count += 1

    @torch.no_grad()
    def update(self, index: int, grad_scale: torch.Tensor | None = None) -> None:
        """AdamW on one parameter tensor for the current step (a data-parallel
        step updates each tensor as soon as its gradient's mean is complete).
        `grad_scale`: a one-element fp32 device tensor the gradient is
        multiplied by first (the clip coefficient of clip_grad_norm)."""
        lib = _lib.lib()
        p = self.params[index]
        m, v = self.state[index]
        g = p.grad
        if g is not None:
            g = g.contiguous()
            args = (p.data_ptr(), g.data_ptr(), _lib.dtype_code(g), m.data_ptr(), v.data_ptr(),
                    p.numel(), self.lr, self.betas[0], self.betas[1], self.eps, self.wd,
                    self.step_count)
            if grad_scale is None:
                rc = lib.ksd8_adamw_step(*args, None, _lib.stream_ptr(p.device))
            else:
                rc = lib.ksd8_adamw_step_scaled(*args, grad_scale.data_ptr(), None,
                                                _lib.stream_ptr(p.device))
            _lib.check(rc, "adamw_step")


    @torch.no_grad()
    def update_all(self, grad_scale: torch.Tensor | None = None) -> None:
        """update() of every tensor with a gradient, in one kernel launch
        (tensors sharing one gradient dtype, at most 8)."""
        import ctypes as C
        items = [(p, self.state[i], p.grad.contiguous()) for i, p in enumerate(self.params)
                 if p.grad is not None]
        if not items:
            return
        dt = {_lib.dtype_code(g) for _, _, g in items}
        if len(items) > 8 or len(dt) != 1:
            for i in range(len(self.params)):
                self.update(i, grad_scale)
            return
        n = len(items)
        ptrs = lambda ts: (C.c_void_p * n)(*[t.data_ptr() for t in ts])  # noqa: E731
        numels = (C.c_int64 * n)(*[p.numel() for p, _, _ in items])
        rc = _lib.lib().ksd8_adamw_multi(
            n, ptrs([p for p, _, _ in items]), ptrs([g for _, _, g in items]), dt.pop(),
            ptrs([s[0] for _, s, _ in items]), ptrs([s[1] for _, s, _ in items]), numels,
            self.lr, self.betas[0], self.betas[1], self.eps, self.wd, self.step_count,
            grad_scale.data_ptr() if grad_scale is not None else None, None,
            _lib.stream_ptr(items[0][0].device))
        _lib.check(rc, "adamw_multi")


def clip_grad_norm(flat: torch.Tensor, max_norm: float, scratch: torch.Tensor,
                   out: torch.Tensor) -> torch.Tensor:
    """torch.nn.utils.clip_grad_norm_ over one flat fp32 gradient buffer, on the
    device: out[0] = total L2 norm, out[1] = min(1, max_norm / (norm + 1e-6)),
    the factor AdamW applies (ksdraft/train/__init__.py:165).  Nothing waits
    for the GPU; returns out."""
    rc = _lib.lib().ksd8_grad_clip_coef(flat.data_ptr(), flat.numel(), float(max_norm),
                                        scratch.data_ptr(), out.data_ptr(), None,
                                        _lib.stream_ptr(flat.device))
    _lib.check(rc, "grad_clip_coef")
    return out


# SMs per GPU left to NCCL while gradient reductions overlap the backward.
# On 8 B200s a 1536 x 5888 layer step scaled 0.86 with 16 and 0.82 with 10
# (10 gives the weight-gradient GEMMs whole waves but starves the all-reduce).
SM_RESERVE = int(os.environ.get("KSD8_SM_RESERVE", "16"))


def init_distributed(timeout_s: float = 120.0,
                     nccl_max_ctas: int | None = None) -> tuple[int, int, int]:
    """(rank, world, local_rank) from the torchrun environment; NCCL on GPUs,
    limited to nccl_max_ctas CTAs (default: the SM reserve of the persistent
    kernels)."""
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1 and not dist.is_initialized():
        backend = "nccl" if torch.cuda.is_available() else "gloo"
        if backend == "nccl":
            torch.cuda.set_device(local)
            # NCCL's kernels then fit in the SMs the persistent kernels leave
            # free while a gradient reduction overlaps the backward
            os.environ.setdefault("NCCL_MAX_CTAS", str(nccl_max_ctas or SM_RESERVE))
        dist.init_process_group(backend, timeout=datetime.timedelta(seconds=timeout_s))
    return rank, world, local


class KS3DataParallelStep:
    """fwd + bwd + gradient all-reduce + AdamW for one trainable KS3Int8Cell."""

    def __init__(self, cell, lr: float = 3e-4, group=None, grad_clip: float | None = 1.0):
        self.cell = cell
        self.params = [cell.master_down, cell.master_up, cell.master_coefficients,
                       cell.master_raw_scale, cell.master_raw_shift]
        self.grads = FlatGrads(self.params)
        names = ("down", "up", "coefficients", "raw_scale", "raw_shift")
        self.named = dict(zip(names, self.params))
        self.index = {n: i for i, n in enumerate(names)}
        self.grad_views = {name: p.grad for name, p in self.named.items()}
        self.group = group
        self.opt = AdamW(self.params, lr=lr)
        # the reference trainer clips the global gradient norm to 1.0 before
        # AdamW (ksdraft/train/__init__.py:39,165); None disables it
        self.grad_clip = grad_clip
        dev = self.grads.buffer.device
        self._clip_scratch = torch.empty(_lib.GRAD_CLIP_SCRATCH, device=dev)
        self._clip_out = torch.zeros(2, device=dev)
        self._copy_stream = torch.cuda.Stream(device=dev) if dev.type == "cuda" else None
        self._dev_bufs: dict[str, torch.Tensor] = {}

    @property
    def last_grad_norm(self) -> torch.Tensor:
        """The total gradient norm of the last step (device tensor, no sync)."""
        return self._clip_out[0]

    def _to_device(self, t: torch.Tensor, name: str, stream=None) -> torch.Tensor:
        """A host tensor copied into this step's device buffer `name` (allocated
        on first use), on `stream` or the current stream; device tensors pass."""
        if t.is_cuda:
            return t
        dev = self.grads.buffer.device
        buf = self._dev_bufs.get(name)
        if buf is None or buf.shape != t.shape or buf.dtype != t.dtype:
            buf = torch.empty(t.shape, dtype=t.dtype, device=dev)
            self._dev_bufs[name] = buf
        with torch.cuda.stream(stream or torch.cuda.current_stream(dev)):
            buf.copy_(t, non_blocking=True)
        return buf

    def __call__(self, x: torch.Tensor, grad_out: torch.Tensor,
                 y_out: torch.Tensor | None = None) -> torch.Tensor:
        """One step.  The backward writes every parameter gradient straight into
        the flat fp32 buffer (as the reference's autograd would leave it after
        the FP16 handoff and the cast to fp32), so no zeroing, casting or
        accumulation pass runs and nothing waits for the GPU.

        x and grad_out may be host tensors (pinned for asynchronous copies):
        x is copied before the forward, grad_out on a copy stream while the
        forward runs.  With `y_out` (a pinned host tensor) the forward output is
        copied back on the copy stream while the backward runs; the current
        stream waits for both copies before the step returns, so anything timed
        or ordered after the call includes them."""
        from ..kernels.ks3_int8 import ks3_backward, ks3_train_forward
        dev = self.grads.buffer.device
        main = torch.cuda.current_stream(dev)
        copy = self._copy_stream
        host_io = not grad_out.is_cuda or y_out is not None
        if host_io:
            copy.wait_stream(main)  # the previous step is done with the device buffers
        x = self._to_device(x, "x")
        g_ready = None
        if not grad_out.is_cuda:
            grad_out = self._to_device(grad_out, "grad_out", copy)
            g_ready = torch.cuda.Event()
            g_ready.record(copy)
        y, saved = ks3_train_forward(self.cell, x.detach())
        if y_out is not None:
            y_done = torch.cuda.Event()
            y_done.record(main)
            copy.wait_event(y_done)
            with torch.cuda.stream(copy):
                y_out.copy_(y.detach(), non_blocking=True)
            y.record_stream(copy)
        if g_ready is not None:
            main.wait_event(g_ready)
        lib = _lib.lib()
        pending = []          # (parameter indices, works) in launch order
        overlapping = [False]

        def on_grad(names):   # each gradient's mean over the ranks starts as soon as it exists
            params = [self.named[n] for n in names]
            works = allreduce_mean_async(self.grads.span(params), self.group)
            if works and not overlapping[0]:
                # from here on the persistent kernels share the GPU with NCCL
                _lib.check(lib.ksd8_set_sm_reserve(SM_RESERVE), "set_sm_reserve")
                overlapping[0] = True
            pending.append(([self.index[n] for n in names], works))
        try:
            ks3_backward(self.cell, grad_out, *saved, x.shape, grads_into=self.grad_views,
                         on_grad=on_grad)
            self.opt.begin_step()
            if self.grad_clip:
                # clip-norm over all reduced gradients, then AdamW on every tensor
                for _, works in pending:
                    wait_all(works)
                clip_grad_norm(self.grads.buffer, self.grad_clip, self._clip_scratch,
                               self._clip_out)
                self.opt.update_all(grad_scale=self._clip_out[1:2])
            else:
                for indices, works in pending:  # update each tensor once its mean is complete
                    wait_all(works)
                    for i in indices:
                        self.opt.update(i)
        finally:
            if overlapping[0]:
                lib.ksd8_set_sm_reserve(0)
        if host_io:
            main.wait_stream(copy)
        return y
