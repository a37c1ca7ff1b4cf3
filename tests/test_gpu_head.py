"""GPU: LM head kernels and the vocab-sharded W8A8 head vs the oracle
(oracle.lm_head_ce: Int8Linear-semantics logits, float64 cross-entropy)."""

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def _rel(a, b):
    a, b = np.asarray(a, np.float64), np.asarray(b, np.float64)
    return np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30)


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_ce_partials_and_grad_vs_numpy(dtype):
    from ksdraft_b200.model.head import ce_grad, ce_partials
    g = torch.Generator().manual_seed(1)
    M, V, vstart = 37, 1003, 512
    logits = (torch.randn(M, V, generator=g) * 4).to(dtype)
    t = torch.randint(0, 2000, (M,), generator=g)          # some targets outside the shard
    t[:5] = vstart + torch.arange(5)                         # and some inside
    mx, sm, tg = ce_partials(logits.cuda(), t.cuda(), vstart)
    l = logits.float().double().numpy()
    np.testing.assert_array_equal(mx.cpu().numpy(), l.max(1).astype(np.float32))
    ref_s = np.exp(l - l.max(1, keepdims=True)).sum(1)
    np.testing.assert_allclose(sm.cpu().numpy(), ref_s, rtol=2e-5)
    loc = (t.numpy() >= vstart) & (t.numpy() < vstart + V)
    ref_t = np.where(loc, l[np.arange(M), np.clip(t.numpy() - vstart, 0, V - 1)], 0.0)
    np.testing.assert_array_equal(tg.cpu().numpy(), ref_t.astype(np.float32))
    # gradient with these as the global statistics, scale 1/M
    d = ce_grad(logits.cuda(), t.cuda(), vstart, mx, sm, 1.0 / M).cpu().numpy()
    p = np.exp(l - l.max(1, keepdims=True)) / ref_s[:, None]
    cols = t.numpy() - vstart
    p[np.arange(M)[loc], cols[loc]] -= 1.0
    np.testing.assert_allclose(d, p / M, rtol=2e-5, atol=1e-9)


@pytest.mark.parametrize("k", [1, 8, 32])
def test_topk_rows_exact_with_ties(k):
    from ksdraft_b200.model.head import topk_rows
    g = torch.Generator().manual_seed(2)
    M, C = 9, 3001
    v = torch.randn(M, C, generator=g)
    v[0] = 0.5                                               # all ties: smallest ids win
    v[1, 100:140] = 9.0                                      # a block of equal maxima
    ov, oi = topk_rows(v.cuda(), k, offset=1000)
    order = np.lexsort((np.broadcast_to(np.arange(C), (M, C)), -v.numpy()), axis=1)[:, :k]
    np.testing.assert_array_equal(oi.cpu().numpy(), order + 1000)
    np.testing.assert_array_equal(ov.cpu().numpy(), np.take_along_axis(v.numpy(), order, 1))
    # merging candidates given with explicit ids (the all-gather path)
    ids = torch.from_numpy(np.stack([np.random.default_rng(r).permutation(C) for r in range(M)]))
    mv, mi = topk_rows(v.cuda(), k, ids=ids.cuda())
    order2 = np.lexsort((ids.numpy(), -v.numpy()), axis=1)[:, :k]
    np.testing.assert_array_equal(mi.cpu().numpy(), np.take_along_axis(ids.numpy(), order2, 1))


@pytest.mark.parametrize("M,V", [(300, 1003), (256, 2048), (1, 130)])
def test_ce_grad_quant_equals_quantised_ce_grad(M, V):
    """The fused kernel's codes == quantize_last_dim / quantize_cols of ce_grad."""
    from ksdraft_b200.kernels.quant import quantize_cols, quantize_last_dim
    from ksdraft_b200.model.head import ce_grad, ce_grad_quant, ce_partials
    g = torch.Generator().manual_seed(M + V)
    logits = (torch.randn(M, V, generator=g) * 4).cuda()
    t = torch.randint(0, V + 300, (M,), generator=g).cuda()
    mx, sm, _ = ce_partials(logits, t, 0)
    dl = ce_grad(logits, t, 0, mx, sm, 1.0 / M)
    dq, dqs, dqt, dqts = ce_grad_quant(logits, t, 0, mx, sm, 1.0 / M)
    rq, rs = quantize_last_dim(dl)
    tq, ts = quantize_cols(dl)
    assert torch.equal(dq[:, :V], rq) and not dq[:, V:].any()
    assert torch.equal(dqs.view(torch.int16), rs.view(torch.int16))
    assert torch.equal(dqt[:, :M], tq) and not dqt[:, M:].any()
    assert torch.equal(dqts.view(torch.int16), ts.view(torch.int16))


def _head_case(M=256, d=256, V=2048, seed=4):
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(M, d, generator=g).to(torch.bfloat16)
    w = torch.randn(V, d, generator=g) * 0.02
    t = torch.randint(0, V, (M,), generator=g)
    return x, w, t


def test_head_loss_and_grads_vs_oracle(oracle):
    from ksdraft_b200.model.head import VocabParallelHead
    x, w, t = _head_case()
    head = VocabParallelHead(w.cuda())
    xd = x.cuda().requires_grad_(True)
    loss = head.cross_entropy(xd, t.cuda())
    loss.backward()
    ref_loss, ref_logits, ref_dx, ref_dw = oracle.lm_head_ce(x.float().numpy(), w.numpy(),
                                                             t.numpy())
    np.testing.assert_array_equal(head.logits(x.cuda()).cpu().numpy(), ref_logits)
    assert abs(float(loss.detach()) - ref_loss) <= 1e-5 * abs(ref_loss)
    dx_ref = torch.from_numpy(ref_dx).to(torch.bfloat16).float().numpy()
    assert xd.grad.dtype == torch.bfloat16
    assert _rel(xd.grad.float().cpu().numpy(), dx_ref) < 1e-3
    assert _rel(head.weight.grad.cpu().numpy(), ref_dw) < 1e-3


def test_two_vocab_shards_match_the_whole_head():
    from ksdraft_b200.model.head import VocabParallelHead, ce_partials, topk_rows
    x, w, t = _head_case(M=128, V=1920)
    xd, td = x.cuda(), t.cuda()
    full = VocabParallelHead(w.cuda())
    shards = [VocabParallelHead(w[:1024].cuda(), vocab=1920, vstart=0),
              VocabParallelHead(w[1024:].cuda(), vocab=1920, vstart=1024)]
    # loss: combine the shard partials as the all-reduces would
    parts = [ce_partials(s.logits(xd), td, s.vstart) for s in shards]
    gmax = torch.maximum(parts[0][0], parts[1][0])
    gsum = sum(p[1] * torch.exp(p[0] - gmax) for p in parts)
    loss = (torch.log(gsum) + gmax - (parts[0][2] + parts[1][2])).mean()
    ref = full.cross_entropy(xd, td)
    assert abs(float(loss) - float(ref)) <= 1e-6 * abs(float(ref))
    # top-k: per-shard candidates merged by id == top-k of the whole head
    k = 8
    cands = [topk_rows(s.logits(xd), k, offset=s.vstart) for s in shards]
    mv, mi = topk_rows(torch.cat([c[0] for c in cands], 1), k,
                       ids=torch.cat([c[1] for c in cands], 1))
    fv, fi = full.topk(xd, k)
    assert torch.equal(mi, fi) and torch.equal(mv, fv)


def test_head_at_config_shape_tied_vs_oracle(oracle):
    """The LM head at the model's shape (d 1536, vocab 150144) on a few hundred
    tokens, tied to an embedding parameter (draft.py:51): logits bit-exact, loss
    within 1e-5, dx within 1e-3 and the weight gradient within 1e-3, landing in
    the embedding's own gradient."""
    from ksdraft_b200.model.head import VocabParallelHead
    M, d, V = 160, 1536, 150144
    x, w, t = _head_case(M=M, d=d, V=V, seed=11)
    emb = torch.nn.Parameter(w.cuda())
    head = VocabParallelHead(emb)
    assert head.tied is emb and head.weight.data_ptr() == emb.data_ptr()
    xd = x.cuda().requires_grad_(True)
    loss = head.cross_entropy(xd, t.cuda())
    loss.backward()
    ref_loss, ref_logits, ref_dx, ref_dw = oracle.lm_head_ce(x.float().numpy(), w.numpy(),
                                                             t.numpy())
    np.testing.assert_array_equal(head.logits(x.cuda()).cpu().numpy(), ref_logits)
    assert abs(float(loss.detach()) - ref_loss) <= 1e-5 * abs(ref_loss)
    dx_ref = torch.from_numpy(ref_dx).to(torch.bfloat16).float().numpy()
    assert _rel(xd.grad.float().cpu().numpy(), dx_ref) < 1e-3
    assert emb.grad is not None and emb.grad.shape == (V, d)
    assert _rel(emb.grad.cpu().numpy(), ref_dw) < 1e-3


def test_head_rejects_out_of_range_targets():
    from ksdraft_b200.model.head import VocabParallelHead
    x, w, t = _head_case(M=8, V=256)
    head = VocabParallelHead(w.cuda())
    for bad in (256, -100, -1):
        tb = t.clone()
        tb[3] = bad
        with pytest.raises(ValueError):
            head.cross_entropy(x.cuda(), tb.cuda())
