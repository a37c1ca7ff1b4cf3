"""GPU: the data-parallel step's direct-to-buffer backward equals the
reference-shaped autograd path (ks3_int8.py:326-429 + the FP16 handoff
:75-84 + the cast into fp32 masters), including the fp32 overflow fallback."""

import pytest
import torch

pytestmark = pytest.mark.gpu


def _cell(d, C, seed):
    from ksdraft_b200.kernels.ks3_int8 import KS3Int8Cell, init_ks3_weights
    cell = init_ks3_weights(d, C, generator=torch.Generator().manual_seed(seed), device="cuda")
    return KS3Int8Cell(cell, nonlinear="int8", trainable=True)


def _autograd_grads(q, x, g):
    for p in (q.master_down, q.master_up, q.master_coefficients, q.master_raw_scale,
              q.master_raw_shift):
        p.grad = None
    xr = x.detach().requires_grad_(True)
    y = q(xr)
    y.backward(g)
    return y.detach(), xr.grad, [p.grad.float().clone() for p in (
        q.master_down, q.master_up, q.master_coefficients, q.master_raw_scale,
        q.master_raw_shift)]


def _direct_grads(q, x, g):
    from ksdraft_b200.kernels.ks3_int8 import ks3_backward, ks3_train_forward
    views = {n: torch.full_like(p, float("nan"), dtype=torch.float32) for n, p in zip(
        ("down", "up", "coefficients", "raw_scale", "raw_shift"),
        (q.master_down, q.master_up, q.master_coefficients, q.master_raw_scale,
         q.master_raw_shift))}
    y, saved = ks3_train_forward(q, x)
    dx = ks3_backward(q, g, *saved, x.shape, grads_into=views)
    torch.cuda.synchronize()
    return y, dx, [views[n] for n in ("down", "up", "coefficients", "raw_scale", "raw_shift")]


@pytest.mark.parametrize("g_scale", [1e-2, 3e3])   # 3e3 overflows fp16 in the wgrads
def test_direct_backward_equals_autograd(g_scale):
    q = _cell(256, 384, 5)
    gen = torch.Generator(device="cuda").manual_seed(7)
    x = torch.randn(300, 256, device="cuda", generator=gen).to(torch.bfloat16)
    g = (torch.randn(300, 256, device="cuda", generator=gen) * g_scale).to(torch.bfloat16)
    y_a, dx_a, ga = _autograd_grads(q, x, g)
    y_d, dx_d, gd = _direct_grads(q, x, g)
    assert torch.equal(y_a, y_d)
    assert torch.equal(dx_a, dx_d)
    for name, a, b in zip(("down", "up", "coefficients", "raw_scale", "raw_shift"), ga, gd):
        a = a.reshape(b.shape)
        same = (a == b) | (torch.isnan(a) & torch.isnan(b))
        assert bool(same.all()), name
    if g_scale > 1:   # the fallback path ran: some wgrad is beyond fp16 range
        assert max(float(ga[0].abs().max()), float(ga[1].abs().max())) > 65504


def test_data_parallel_step_runs_and_updates():
    from ksdraft_b200.train.dp import KS3DataParallelStep
    q = _cell(256, 384, 6)
    gen = torch.Generator(device="cuda").manual_seed(8)
    x = torch.randn(256, 256, device="cuda", generator=gen).to(torch.bfloat16)
    g = (torch.randn(256, 256, device="cuda", generator=gen) * 1e-2).to(torch.bfloat16)
    _, _, ga = _autograd_grads(q, x, g)      # reference-shaped grads, before any update
    step = KS3DataParallelStep(q)            # attaches the flat fp32 grad buffer
    before = q.master_down.detach().clone()
    step(x, g)
    torch.cuda.synchronize()
    assert torch.equal(step.grad_views["down"].reshape(ga[0].shape), ga[0])
    assert torch.equal(step.grad_views["up"].reshape(ga[1].shape), ga[1])
    assert not torch.equal(before, q.master_down.detach())


@pytest.mark.parametrize("scale", [1e-2, 30.0])
def test_data_parallel_step_clips_like_torch(scale):
    """clip_grad_norm_(1.0) + AdamW of the reference trainer (train/__init__.py:
    165-166) against torch on the same gradients: the norm is computed and
    applied on the device; with small gradients the coefficient is 1."""
    from ksdraft_b200.train.dp import KS3DataParallelStep
    q = _cell(256, 384, 6)
    gen = torch.Generator(device="cuda").manual_seed(9)
    x = torch.randn(256, 256, device="cuda", generator=gen).to(torch.bfloat16)
    g = (torch.randn(256, 256, device="cuda", generator=gen) * scale).to(torch.bfloat16)
    step = KS3DataParallelStep(q, grad_clip=1.0)
    params = step.params
    before = [p.detach().clone() for p in params]
    step(x, g)
    torch.cuda.synchronize()
    grads = [p.grad.detach().clone() for p in params]
    norm = torch.linalg.vector_norm(torch.cat([t.reshape(-1) for t in grads]))
    torch.testing.assert_close(step.last_grad_norm, norm, rtol=1e-5, atol=0)
    coef = torch.clamp(1.0 / (norm + 1e-6), max=1.0)
    ref = [b.clone().requires_grad_(True) for b in before]
    for r, gr in zip(ref, grads):
        r.grad = gr * coef
    opt = torch.optim.AdamW(ref, lr=3e-4, betas=(0.9, 0.999), eps=1e-8, weight_decay=0.01)
    opt.step()
    for p, r in zip(params, ref):
        torch.testing.assert_close(p.detach(), r.detach(), rtol=1e-6, atol=1e-7)
    if scale > 1:
        assert float(coef) < 1.0


@pytest.mark.parametrize("tokens", [256, 1024])
def test_data_parallel_step_host_io_matches_device_io(tokens):
    """Host inputs and a host output buffer (copies overlapped with the step on
    a copy stream; with 1024 tokens x arrives in 4 row chunks that are
    quantised and projected as they land) give the same output and the same
    update as device tensors."""
    from ksdraft_b200.train.dp import KS3DataParallelStep
    gen = torch.Generator(device="cuda").manual_seed(10)
    x = torch.randn(tokens, 256, device="cuda", generator=gen).to(torch.bfloat16)
    g = (torch.randn(tokens, 256, device="cuda", generator=gen) * 1e-2).to(torch.bfloat16)
    steps = [KS3DataParallelStep(_cell(256, 384, 6)) for _ in range(2)]
    x_h, g_h = x.cpu().pin_memory(), g.cpu().pin_memory()
    y_h = torch.empty(tokens, 256, dtype=torch.bfloat16).pin_memory()
    for _ in range(2):  # two steps: the reused device buffers and copy stream
        y_dev = steps[0](x, g)
        y_ret = steps[1](x_h, g_h, y_out=y_h)
        torch.cuda.synchronize()
        assert torch.equal(y_dev.cpu(), y_h)
        assert torch.equal(y_ret.cpu(), y_h)
    for p0, p1 in zip(steps[0].params, steps[1].params):
        assert torch.equal(p0.detach(), p1.detach())
