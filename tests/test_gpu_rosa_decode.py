"""GPU: incremental Rosa matching (ksd8_rosa_decode_step / _build) against the
whole-sequence matcher (itself pinned to the reference's _match_payload_sign,
ksdraft/model/rosa.py:40-98, by the oracle tests): a context prefilled by the
sequence matcher, then blocks of positions appended, must give the same match
length, latest endpoint and sign at every appended position as matching the
whole extended sequence at once -- bit for bit, on fair bits and on long-run
bits (the deep-layer statistics), across main-run rebuilds."""

import pytest
import torch

pytestmark = pytest.mark.gpu

S = 64


def _bits(kind, B, T, gen):
    if kind == "fair":
        return (torch.rand(B, T, S, generator=gen) > 0.5).to(torch.int8)
    if kind == "runs":
        flips = (torch.rand(B, T, S, generator=gen) < 0.1).to(torch.int32)
        return (torch.cumsum(flips, 1) & 1).to(torch.int8)
    # periodic with rare noise: many equal windows
    base = (torch.arange(T)[None, :, None] % 3 == 0).to(torch.int8).expand(B, T, S)
    noise = (torch.rand(B, T, S, generator=gen) < 0.01).to(torch.int8)
    return (base ^ noise).contiguous()


def _full(bits3, B, T):
    from ksdraft_b200.model.rosa import match_words, pack_bits
    dev = bits3[0].device
    words = [pack_bits(b, B, T, S, T * S, S, 1) for b in bits3]
    out = torch.empty(B, T, S, dtype=torch.float32, device=dev)
    ml, me = match_words(*words, B, S, T, min(62, T - 1), out=out, strides=(T * S, S, 1),
                         with_indices=True)
    return ml, me, out


@pytest.mark.parametrize("kind", ["fair", "runs", "periodic"])
@pytest.mark.parametrize("k_new", [1, 8, 12, 32])
def test_decode_matches_whole_sequence(kind, k_new):
    from ksdraft_b200.model.drafter import RosaDecodeState
    from ksdraft_b200.model.rosa import match_words, pack_bits
    gen = torch.Generator().manual_seed(sum(map(ord, kind)) * 100 + k_new)
    B, T0 = 3, 100
    steps = 2600 // k_new if k_new > 1 else 150   # k_new > 1 passes a main-run rebuild
    T = T0 + steps * k_new
    bits3 = [_bits(kind, B, T, gen).cuda() for _ in range(3)]
    ml_ref, me_ref, out_ref = _full(bits3, B, T)

    cap = (T + 63) // 64 * 64
    st = RosaDecodeState(B, S, cap, "cuda")
    words = [pack_bits(b[:, :T0].contiguous(), B, T0, S, T0 * S, S, 1) for b in bits3]
    st.load_words(words, T0)
    st.build(T0)
    payload = torch.ones(S, device="cuda")
    builds = 0
    for i in range(steps):
        t0 = T0 + i * k_new
        # projections whose sign is the bit (proj > 0), layout (contexts, k_new, streams)
        projs = [(b[:, t0:t0 + k_new].float() * 2 - 1).contiguous() for b in bits3]
        out = torch.empty(B, k_new, S, device="cuda")
        ml = torch.empty(B * S, k_new, dtype=torch.int32, device="cuda")
        me = torch.empty_like(ml)
        n_before = st.n_main
        st.step(projs, t0, payload, out, ml, me)
        builds += st.n_main != n_before
        assert torch.equal(ml, ml_ref[:, t0:t0 + k_new]), (kind, k_new, t0)
        assert torch.equal(me, me_ref[:, t0:t0 + k_new]), (kind, k_new, t0)
        assert torch.equal(out, out_ref[:, t0:t0 + k_new]), (kind, k_new, t0)
    if k_new > 1:
        assert builds >= 1    # the delta outgrew the step kernel's window at least once


def test_decode_rollback_overwrites_appended_bits():
    """A step at an earlier t0 (>= the main run) replaces the positions it covers."""
    from ksdraft_b200.model.drafter import RosaDecodeState
    from ksdraft_b200.model.rosa import pack_bits
    gen = torch.Generator().manual_seed(7)
    B, T0, k = 2, 128, 8
    T = T0 + 3 * k
    bits3 = [_bits("runs", B, T, gen).cuda() for _ in range(3)]
    ml_ref, me_ref, _ = _full(bits3, B, T)
    st = RosaDecodeState(B, S, 256, "cuda")
    st.load_words([pack_bits(b[:, :T0].contiguous(), B, T0, S, T0 * S, S, 1) for b in bits3],
                  T0)
    st.build(T0)
    pay = torch.ones(S, device="cuda")
    out = torch.empty(B, k, S, device="cuda")
    junk = [torch.randn(B, k, S, generator=gen).cuda() for _ in range(3)]
    st.step(junk, T0, pay, out)                       # a block that gets rejected
    for t0 in (T0, T0 + k, T0 + 2 * k):
        projs = [(b[:, t0:t0 + k].float() * 2 - 1).contiguous() for b in bits3]
        ml = torch.empty(B * S, k, dtype=torch.int32, device="cuda")
        me = torch.empty_like(ml)
        st.step(projs, t0, pay, out, ml, me)
        assert torch.equal(ml, ml_ref[:, t0:t0 + k]) and torch.equal(me, me_ref[:, t0:t0 + k])


@pytest.mark.parametrize("kind", ["fair", "runs"])
def test_match_context_equals_sequence_matcher(kind):
    """The drafter's prefill path: a whole context matched 32 positions at a time
    through the decode kernels (a full main-run build and a merge included)."""
    from ksdraft_b200.model.drafter import RosaDecodeState
    from ksdraft_b200.model.rosa import pack_bits
    gen = torch.Generator().manual_seed(11 + len(kind))
    B, T = 2, 5000       # one full build, then one merge of the appended keys
    bits3 = [_bits(kind, B, T, gen).cuda() for _ in range(3)]
    ml_ref, me_ref, out_ref = _full(bits3, B, T)
    st = RosaDecodeState(B, S, 5056, "cuda")
    st.load_words([pack_bits(b, B, T, S, T * S, S, 1) for b in bits3], T)
    out = torch.empty(B, T, S, device="cuda")
    ml = torch.empty(B * S, T, dtype=torch.int32, device="cuda")
    me = torch.empty_like(ml)
    st.match_context(T, torch.ones(S, device="cuda"), out, ml, me)
    assert torch.equal(ml, ml_ref) and torch.equal(me, me_ref) and torch.equal(out, out_ref)


def test_decode_rejects_bad_arguments():
    from ksdraft_b200 import _lib
    lib = _lib.lib()
    # k_new outside 1..32, n_main beyond t0: shape errors before any launch
    rc = lib.ksd8_rosa_decode_step(None, None, None, 0, 1, 1, 33, 0, 0, 62, None, None, None, 1,
                                   None, None, None, None, 64, None, None, 33, 0, None, None, 33,
                                   None, None, None)
    assert rc == 1
    rc = lib.ksd8_rosa_decode_step(None, None, None, 0, 1, 1, 8, 10, 11, 62, None, None, None, 1,
                                   None, None, None, None, 64, None, None, 8, 0, None, None, 8,
                                   None, None, None)
    assert rc == 1
