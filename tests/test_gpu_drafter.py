"""GPU: drafting (BASELINE config 5 path, ksdraft_b200/model/drafter.py).

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
