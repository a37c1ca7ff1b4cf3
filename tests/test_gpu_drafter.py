"""GPU: drafting (benchmark config 5 path, ksdraft_b200/model/drafter.py).

Appending blocks to prefilled contexts must give what a whole-sequence int8
forward of the extended contexts gives (KSDraftModel.forward semantics,
ksdraft/model/draft.py:58-82): the Rosa matches of every layer at the appended
positions (bit-exact where the layer's inputs are bit-exact, i.e. layer 0),
and the head's top-k candidates and logits at the last appended position."""

import pytest
import torch

pytestmark = pytest.mark.gpu

SMALL = dict(vocab=512, layers=3, d_model=128, streams=128, charts=256, teacher_dim=64)


def _model(seed=0):
    from ksdraft_b200.train.draft_step import DraftShape, init_draft_params
    shape = DraftShape(**SMALL)
    flat, frozen = init_draft_params(shape, "cuda", seed=seed)
    state = {n: flat.p(n) for n in flat.names}
    state.update(frozen)
    g = torch.Generator(device="cuda").manual_seed(seed + 1)
    with torch.no_grad():   # a "woken" model: the zero-init paths carry signal
        for l in range(shape.layers):
            state[f"blocks.{l}.rosa.out_proj.weight"].normal_(0, 0.3, generator=g)
            state[f"blocks.{l}.injection.inject.up.weight"].normal_(0, 0.3, generator=g)
            state[f"blocks.{l}.injection.gate_q.up.weight"].normal_(0, 0.3, generator=g)
        state["embedding.weight"].normal_(0, 1.0, generator=g)
    return shape, state


def _inputs(C, T, seed=3):
    g = torch.Generator().manual_seed(seed)
    # a small vocabulary slice with repeats so that Rosa finds long matches
    tokens = torch.randint(0, 40, (C, T), generator=g)
    states = torch.randn(C, T, SMALL["teacher_dim"], generator=g)
    return tokens, states


@pytest.mark.parametrize("act", [torch.float32, torch.bfloat16])
def test_propose_equals_whole_sequence_forward(act):
    from ksdraft_b200.model.drafter import KSDraftDrafter
    shape, state = _model()
    C, T0, n = 4, 96, 8
    tokens, states = _inputs(C, T0 + 2 * n)
    st = states.to(act)
    inc = KSDraftDrafter(state, shape, "cuda", contexts=C, capacity=256, act_dtype=act)
    inc.prefill(tokens[:, :T0], st[:, :T0])
    probes = []
    outs = []
    for b in range(2):
        pr = {}
        sl = slice(T0 + b * n, T0 + (b + 1) * n)
        outs.append(inc.propose(st[:, sl], tokens[:, sl], topk=5, probe=pr))
        probes.append(pr)
    assert inc.length == T0 + 2 * n
    tol = 1e-4 if act == torch.float32 else 3e-2
    for b in range(2):
        T = T0 + (b + 1) * n
        whole = KSDraftDrafter(state, shape, "cuda", contexts=C, capacity=256, act_dtype=act)
        pw = {}
        ids_w, vals_w = whole.prefill(tokens[:, :T], st[:, :T], topk=5, probe=pw)
        ids_i, vals_i, refined = outs[b]
        assert refined is None and ids_i.shape == (C, n, 5)
        # layer 0 sees identical inputs: its matches are bit-identical
        ml_w, me_w, _ = pw[0]
        ml_i, me_i, _ = probes[b][0]
        assert torch.equal(ml_i, ml_w[:, T - n:T]) and torch.equal(me_i, me_w[:, T - n:T])
        # deeper layers: the same up to summation-order effects on near-zero projections
        for l in range(1, shape.layers):
            same = (probes[b][l][1] == pw[l][1][:, T - n:T]).float().mean().item()
            assert same > 0.99, (l, same)
        # last appended position vs the whole-sequence forward's last position
        rel = ((vals_i[:, -1] - vals_w).norm() / vals_w.norm()).item()
        print(f"block {b} act {act}: top-5 logits rel {rel:.2e}, "
              f"ids equal {(ids_i[:, -1] == ids_w).float().mean().item():.3f}")
        assert rel < tol
        assert (ids_i[:, -1, 0] == ids_w[:, 0]).all()


def test_drafter_argument_checks():
    from ksdraft_b200.model.drafter import KSDraftDrafter
    shape, state = _model()
    d = KSDraftDrafter(state, shape, "cuda", contexts=2, capacity=128)
    tokens, states = _inputs(2, 100)
    with pytest.raises(RuntimeError):
        d.propose(None, tokens[:, :4])
    with pytest.raises(ValueError):
        d.prefill(tokens[:, :40])                       # shorter than the Rosa cap
    with pytest.raises(ValueError):
        d.prefill(tokens[:, :100] + 600)                # outside the vocabulary
    d.prefill(tokens[:, :100], states[:, :100].to(torch.bfloat16))
    with pytest.raises(ValueError):
        d.propose(None, tokens[:, :33])                 # a block holds at most 32 positions


def test_drafter_matches_reference_int8_eval(golden):
    """The reference's own int8-tier evaluation forward (to_int8, float head) of
    the draft_step model on 120 positions (tests/golden/draft_eval.npz): a
    prefill of 96 positions and three appended blocks of 8 give, at every
    appended position, the reference's top-5 candidates and their logits.
    The fixture's inputs keep every Rosa projection at least 1e-5 of its mean
    magnitude away from zero: a sign decided by fp32 summation order (the
    reference dequantises and runs an fp32 matmul, the GEMM here sums exact
    int32 groups; they agree to 2.2e-6 of the mean) would flip one bit and
    every later match of its stream."""
    from ksdraft_b200.model.drafter import KSDraftDrafter
    from ksdraft_b200.train.draft_step import DraftShape
    g = golden("draft_eval")
    w = golden("draft_step")
    state = {k[2:]: torch.from_numpy(v) for k, v in w.items() if k.startswith("w.")}
    shape = DraftShape(vocab=512, layers=2, d_model=128, streams=128, charts=256,
                       teacher_dim=64)
    d = KSDraftDrafter(state, shape, "cuda", contexts=2, capacity=128,
                       act_dtype=torch.float32, head_mode="float")
    tokens = torch.from_numpy(g["tokens"])
    states = torch.from_numpy(g["states"])
    ref = torch.from_numpy(g["logits_tail"]).cuda()          # positions 96 .. 119
    d.prefill(tokens[:, :96], states[:, :96])
    worst, agree = 0.0, []
    for b in range(3):
        sl = slice(96 + 8 * b, 104 + 8 * b)
        ids, vals, _ = d.propose(states[:, sl], tokens[:, sl], topk=5)
        r = ref[:, 8 * b:8 * b + 8]
        rv = torch.gather(r, 2, ids)                           # reference logits at our ids
        worst = max(worst, ((vals - rv).norm() / rv.norm()).item())
        agree.append((ids == r.topk(5, dim=-1).indices).float().mean().item())
    print(f"drafter vs reference int8 eval: top-5 logits rel-L2 {worst:.2e}, "
          f"top-5 ids agree {min(agree):.3f}")
    assert worst < 2e-3
    assert min(agree) > 0.95


def test_graph_replay_equals_eager_across_rebuilds():
    """propose() replayed from one recorded CUDA graph gives the eager result at
    every block, including blocks after a main-run rebuild (taken outside the
    graph, the position read from device memory)."""
    from ksdraft_b200.model.drafter import KSDraftDrafter
    shape, state = _model()
    C, T0, n, blocks = 2, 96, 8, 280
    tokens, states = _inputs(C, T0 + n * (blocks + 1), seed=5)
    st = states.to(torch.bfloat16)
    cap = T0 + n * (blocks + 1)
    eager = KSDraftDrafter(state, shape, "cuda", contexts=C, capacity=cap)
    graphed = KSDraftDrafter(state, shape, "cuda", contexts=C, capacity=cap)
    for d in (eager, graphed):
        d.prefill(tokens[:, :T0], st[:, :T0])
    graphed.capture(n, topk=4)
    n_main0 = graphed.states[0].n_main
    worst, agree = 0.0, 1.0
    for b in range(blocks):
        sl = slice(T0 + b * n, T0 + (b + 1) * n)
        ie, ve, _ = eager.propose(st[:, sl], tokens[:, sl], topk=4)
        ig, vg, _ = graphed.propose(st[:, sl], tokens[:, sl], topk=4)
        worst = max(worst, ((ve - vg).norm() / ve.norm()).item())
        agree = min(agree, (ie[..., 0] == ig[..., 0]).float().mean().item())
    print(f"graph vs eager over {blocks} blocks: top-4 logits rel {worst:.2e}, "
          f"top-1 agree {agree:.3f}")
    # the same kernels in the same order (cuBLAS may pick another algorithm for
    # the low-rank bf16 GEMMs under capture: bf16 rounding level at most)
    assert worst < 2e-2 and agree >= 0.95
    assert graphed.states[0].n_main > n_main0      # at least one rebuild happened
    graphed.release()
