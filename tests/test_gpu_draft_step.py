"""GPU: the full KSDraft INT8 training step (model of ksdraft/model/draft.py,
trainer step of ksdraft/train/__init__.py:145-166) against the reference's own
int8-tier run of the same small model (tests/golden/draft_step.npz, made by
tests/golden/make_golden.py from the reference package on its CPU tier).

Where the two differ by design: the reference's int8 tier keeps the tied LM
head in fp32 (ksdraft/model/int8_convert.py:8-12) while this step runs it W8A8
(logits, dgrad and wgrad), and fp32 GEMM summation order moves a few KS3
coordinates across fp16 roundings.  The tolerances below bound both; the
component tests pin each kernel to 1e-3 or bit-exactness."""

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

SMALL = dict(vocab=512, layers=2, d_model=128, streams=128, charts=256, teacher_dim=64)


def _rel(a, b):
    a, b = np.asarray(a, np.float64), np.asarray(b, np.float64)
    return np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30)


def _step(golden, act=torch.float32, grad_clip=1.0, head_mode="w8a8"):
    from ksdraft_b200.train.draft_step import DraftShape, DraftTrainStep
    g = golden("draft_step")
    st = DraftTrainStep(DraftShape(**SMALL), "cuda", act_dtype=act, grad_clip=grad_clip,
                        head_mode=head_mode)
    st.load_state_dict({k[2:]: torch.from_numpy(v) for k, v in g.items() if k.startswith("w.")})
    return g, st


def _compare(g, st, loss):
    ce, tr = float(st.last["ce"]), float(st.last["transfer"])
    print(f"loss {float(loss):.6f} vs {float(g['loss']):.6f}; ce {ce:.6f} vs {float(g['ce']):.6f};"
          f" transfer {tr:.6f} vs {float(g['transfer']):.6f}")
    assert abs(tr - float(g["transfer"])) < 1e-5 * max(1.0, abs(float(g["transfer"])))
    assert abs(ce - float(g["ce"])) < 2e-3 * abs(float(g["ce"]))
    names = sorted(k[5:] for k in g if k.startswith("grad."))
    params = st.parameter_dict()
    worst = {}
    for n in names:
        got = st.flat.g(n).cpu().numpy() if n in st.flat.offsets else None
        assert got is not None, f"no gradient for {n}"
        r = _rel(got.reshape(-1), g["grad." + n].reshape(-1))
        worst[n] = r
        print(f"grad {n}: rel-L2 {r:.2e}")
    # every parameter the reference trains is trained here, and only those
    assert set(names) == set(st.flat.names)
    assert set(params) - set(names) == set(st.frozen)
    return ce, tr, worst


def test_draft_step_matches_reference_int8_tier(golden):
    """With the reference int8 tier's own float head (int8_convert.py:8-12) the
    full step's loss matches to 1e-5 and the gradients to 1e-3 rel-L2 (median
    over parameters); the KS3 weight and ln_ffn gradients reach 1.6e-3 after two
    blocks: the reference's fp32 matmul of the dequantised operands rounds a few
    fp16 KS3 coordinates the other way (0.13% at the single-layer test), which
    moves the LUT index of those elements."""
    g, st = _step(golden, head_mode="float")
    loss = st.forward_backward(torch.from_numpy(g["tokens"]), torch.from_numpy(g["states"]))
    ce, tr, worst = _compare(g, st, loss)
    assert abs(ce - float(g["ce"])) < 1e-5 * abs(float(g["ce"]))
    assert np.median(list(worst.values())) < 1e-3
    bad = {n: r for n, r in worst.items() if r >= 2e-3}
    assert not bad, bad
    coord_path = {n: r for n, r in worst.items() if r >= 1e-3}
    assert all(".ffn." in n or ".ln_ffn." in n for n in coord_path), coord_path


def test_draft_step_w8a8_head_vs_reference(golden):
    """With the north-star W8A8 head (logits, dgrad, wgrad on int8 operands) the
    step differs from the reference's float head by the head's quantisation:
    the loss within 2e-3, gradients within 0.15 rel-L2 (sums over tokens such as
    output_norm.bias the loosest), the median within 5%."""
    g, st = _step(golden)
    loss = st.forward_backward(torch.from_numpy(g["tokens"]), torch.from_numpy(g["states"]))
    ce, tr, worst = _compare(g, st, loss)
    assert abs(ce - float(g["ce"])) < 2e-3 * abs(float(g["ce"]))
    assert max(worst.values()) < 0.15, max(worst.items(), key=lambda kv: kv[1])
    assert np.median(list(worst.values())) < 5e-2


def test_draft_step_trains_and_bf16_agrees(golden):
    """Three steps on one batch lower the loss; the bf16-activation step (the
    benchmark's) agrees with the fp32 one on the first loss."""
    g, st = _step(golden)
    tokens = torch.from_numpy(g["tokens"])
    states = torch.from_numpy(g["states"])
    losses = [float(st(tokens, states)) for _ in range(3)]
    assert all(np.isfinite(losses)) and losses[-1] < losses[0], losses
    assert torch.isfinite(st.flat.data).all()
    _, sb = _step(golden, act=torch.bfloat16)
    lb = float(sb(tokens.cuda(), states.cuda().to(torch.bfloat16)))
    assert abs(lb - losses[0]) < 2e-2 * abs(losses[0]), (lb, losses[0])


def test_draft_step_cuda_graph_replay_matches_eager(golden):
    """The captured step (one CUDA graph for forward + backward, AdamW eager)
    gives the eager step's loss and gradients, and keeps doing so on new inputs
    copied into its static buffers."""
    g, eager = _step(golden)
    _, graphed = _step(golden)
    tokens = torch.from_numpy(g["tokens"])
    states = torch.from_numpy(g["states"])
    graphed.capture(tokens, states)
    for shift in (0, 7):
        tk = (tokens + shift) % SMALL["vocab"]
        le = eager.forward_backward(tk, states)
        lg = graphed.replay(tk, states, update=False)
        torch.cuda.synchronize()
        assert abs(float(le) - float(lg)) <= 1e-6 * abs(float(le))
        ge, gg = eager.flat.grad, graphed.flat.grad
        assert float((ge - gg).norm() / ge.norm()) < 1e-6
    # a replay with the update equals an eager step with the update
    le = eager(tokens, states)
    lg = graphed.replay(tokens, states)
    torch.cuda.synchronize()
    assert float((eager.flat.data - graphed.flat.data).norm() / eager.flat.data.norm()) < 1e-6
