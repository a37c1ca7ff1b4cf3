"""Multi-rank host logic on CPU (gloo, world size 2, 127.0.0.1): data-parallel
gradient averaging and finiteness agreement (ksdraft_b200/train/dp.py), the
vocab-parallel cross-entropy combine and top-k merge of the LM head
(ksdraft_b200/model/head.py), and failure detection when a rank dies before a
collective.  Each rank is a spawned child process; results come back through
files under tmp_path."""

import json
import os
import socket
import sys
import time
from pathlib import Path

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

ROOT = Path(__file__).resolve().parents[1]


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _init(rank, world, port, timeout_s=30):
    import datetime
    sys.path.insert(0, str(ROOT))
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank,
                            world_size=world, timeout=datetime.timedelta(seconds=timeout_s))


def _run(fn, world, tmp_path, *args):
    port = _free_port()
    ctx = mp.get_context("spawn")
    procs = [ctx.Process(target=fn, args=(r, world, port, str(tmp_path), *args))
             for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
    for p in procs:
        if p.is_alive():
            p.kill()
            p.join()
    return [p.exitcode for p in procs]


# ---------------------------------------------------------------- data parallel

def _dp_worker(rank, world, port, out):
    _init(rank, world, port)
    from ksdraft_b200.train.dp import (FlatGrads, allreduce_mean_, allreduce_mean_async,
                                       check_finite_across_ranks, wait_all)
    torch.manual_seed(0)
    params = [torch.nn.Parameter(torch.zeros(5, 3)), torch.nn.Parameter(torch.zeros(7))]
    fg = FlatGrads(params)
    for i, (p, view) in enumerate(fg.views()):
        view.copy_(torch.arange(view.numel(), dtype=torch.float32) * (rank + 1) + i)
    allreduce_mean_(fg.buffer)
    res = {"grads": [p.grad.reshape(-1).tolist() for p in params]}
    # the overlapped form: start the mean of one parameter's span, then wait
    params[1].grad.fill_(10.0 * (rank + 1))
    pending = allreduce_mean_async(fg.span([params[1]]), dist.group.WORLD)
    wait_all(pending)
    res["span_mean"] = params[1].grad.tolist()
    res["span_len"] = fg.span(params).numel()
    res["finite_all"] = check_finite_across_ranks(fg.buffer)
    if rank == 1:
        fg.buffer[3] = float("nan")
    res["finite_one_bad"] = check_finite_across_ranks(fg.buffer)
    Path(out, f"dp{rank}.json").write_text(json.dumps(res))
    dist.destroy_process_group()


def test_dp_allreduce_mean_and_finite_flags(tmp_path):
    assert _run(_dp_worker, 2, tmp_path) == [0, 0]
    for r in range(2):
        res = json.loads(Path(tmp_path, f"dp{r}.json").read_text())
        for i, g in enumerate(res["grads"]):
            base = np.arange(len(g), dtype=np.float64)
            np.testing.assert_allclose(g, (base * 1 + i + base * 2 + i) / 2, rtol=1e-6)
        assert res["span_mean"] == [15.0] * 7
        assert res["span_len"] == 64 + 7          # first param padded to 64, then the second
        assert res["finite_all"] is True
        assert res["finite_one_bad"] is False     # every rank sees rank 1's NaN


# ---------------------------------------------------------------- vocab-parallel head

def _logits(M, V, seed=3):
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(M, V, generator=g) * 3
    t = torch.randint(0, V, (M,), generator=g)
    x[0, :] = 1.25             # a row of ties for the top-k
    return x, t


def _head_worker(rank, world, port, out, V, M, k):
    _init(rank, world, port)
    from ksdraft_b200.model.head import combine_ce_partials, gather_topk, vocab_shard
    logits, t = _logits(M, V)
    start, size = vocab_shard(V, rank, world)
    shard = logits[:, start:start + size]
    # this rank's partials, computed on the host as the kernel defines them
    mx = shard.max(1).values
    sm = torch.exp(shard - mx[:, None]).sum(1)
    local = (t >= start) & (t < start + size)
    tg = torch.where(local, shard[torch.arange(M), (t - start).clamp(0, size - 1)],
                     torch.zeros(M))
    _, _, loss_rows = combine_ce_partials(mx, sm, tg, group=dist.group.WORLD)

    def select(vals, kk, offset=0, ids=None):   # host stand-in for the top-k kernel
        order = np.lexsort((ids.numpy(), -vals.numpy()), axis=1)[:, :kk]
        return (torch.from_numpy(np.take_along_axis(vals.numpy(), order, 1)),
                torch.from_numpy(np.take_along_axis(ids.numpy(), order, 1)))

    ids = torch.arange(start, start + size).expand(M, size)
    lv, li = select(shard, k, ids=ids)
    gv, gi = gather_topk(lv, li, k, group=dist.group.WORLD, select=select)
    Path(out, f"head{rank}.json").write_text(json.dumps({
        "loss_rows": loss_rows.tolist(), "topv": gv.tolist(), "topi": gi.tolist(),
        "shard": [start, size]}))
    dist.destroy_process_group()


def test_vocab_parallel_ce_and_topk_merge(tmp_path):
    V, M, k = 1000, 6, 5           # 8 groups of 128 (last partial): shards 512 + 488
    assert _run(_head_worker, 2, tmp_path, V, M, k) == [0, 0]
    logits, t = _logits(M, V)
    l64 = logits.double()
    full = torch.logsumexp(l64, 1) - l64[torch.arange(M), t]
    order = np.lexsort((np.broadcast_to(np.arange(V), (M, V)), -logits.numpy()), axis=1)[:, :k]
    shards = []
    for r in range(2):
        res = json.loads(Path(tmp_path, f"head{r}.json").read_text())
        np.testing.assert_allclose(res["loss_rows"], full.numpy(), rtol=1e-5, atol=1e-5)
        np.testing.assert_array_equal(np.array(res["topi"]), order)
        np.testing.assert_allclose(res["topv"], np.take_along_axis(logits.numpy(), order, 1))
        shards.append(res["shard"])
    assert shards == [[0, 512], [512, 488]]


def test_vocab_shard_boundaries():
    from ksdraft_b200.model.head import vocab_shard
    for V in (150144, 1000, 128, 300):
        for world in (1, 2, 3, 4, 8):
            parts = [vocab_shard(V, r, world) for r in range(world)]
            assert parts[0][0] == 0
            assert sum(s for _, s in parts) == V
            for (a, s), (b, _) in zip(parts, parts[1:]):
                assert a + s == b and a % 128 == 0 and b % 128 == 0
    assert vocab_shard(150144, 1, 2) == (75008, 75136)   # 586 + 587 groups


# ---------------------------------------------------------------- failure detection

def _fail_worker(rank, world, port, out):
    _init(rank, world, port, timeout_s=5)
    if rank == 1:
        os._exit(3)                  # dies between steps, before the collective
    t0 = time.time()
    err = None
    try:
        x = torch.ones(4)
        dist.all_reduce(x)
    except Exception as e:           # noqa: BLE001 - any error ends the wait
        err = type(e).__name__
    Path(out, "fail0.json").write_text(json.dumps({"error": err, "seconds": time.time() - t0}))
    os._exit(0)


def test_peer_death_ends_collective_with_error(tmp_path):
    codes = _run(_fail_worker, 2, tmp_path)
    assert codes[1] == 3
    res = json.loads(Path(tmp_path, "fail0.json").read_text())
    assert res["error"] is not None                 # detected, not hung
    assert res["seconds"] < 60


# ---------------------------------------------------------------- full-model step

def _sparse_rows_worker(rank, world, port, out):
    _init(rank, world, port)
    from ksdraft_b200.train.dp import allreduce_mean_async, wait_all
    from ksdraft_b200.train.draft_step import gather_sparse_rows
    V, d = 10, 4
    g = torch.Generator().manual_seed(rank)
    dense = torch.randn(V, d, generator=g)
    ids = torch.randint(0, V, (6,), generator=g)
    rows = torch.randn(6, d, generator=g)
    # the step's order: dense head gradient averaged asynchronously, sparse rows
    # gathered afterwards and added once the mean is complete
    grad = dense.clone()
    pending = allreduce_mean_async(grad, dist.group.WORLD)
    all_ids, all_rows = gather_sparse_rows(ids, rows, world, dist.group.WORLD)
    wait_all(pending)
    grad.index_add_(0, all_ids, all_rows)
    full = dense.clone()
    full.index_add_(0, ids, rows)                    # this rank's whole gradient
    Path(out, f"sp{rank}.json").write_text(json.dumps({"grad": grad.tolist(),
                                                      "full": full.tolist()}))
    dist.destroy_process_group()


def test_embedding_sparse_rows_mean_over_ranks(tmp_path):
    """The tied embedding's gradient (dense head part + sparse gathered rows) equals
    the mean over ranks of each rank's full dense gradient."""
    assert _run(_sparse_rows_worker, 2, tmp_path) == [0, 0]
    r = [json.loads(Path(tmp_path, f"sp{i}.json").read_text()) for i in range(2)]
    want = (np.array(r[0]["full"]) + np.array(r[1]["full"])) / 2
    for i in range(2):
        np.testing.assert_allclose(np.array(r[i]["grad"]), want, rtol=1e-6, atol=1e-6)


def test_draft_param_layout_and_token_check():
    """Flat layout of the full step: reference state-dict names, every block one
    contiguous span in backward order, 64-element alignment; token range check."""
    from ksdraft_b200.train.draft_step import (DraftShape, FlatParams, _frozen_shapes,
                                               check_tokens)
    s = DraftShape(vocab=300, layers=3, d_model=128, streams=128, charts=256, teacher_dim=64)
    f = FlatParams(s, "cpu")
    assert f.names[0] == "embedding.weight" and f.names[-1] == "input_norm.bias"
    assert all(off % 64 == 0 for off in f.offsets.values())
    spans = [f.block_span[layer] for layer in reversed(range(3))]
    assert [a for a, _ in spans] == sorted(a for a, _ in spans)
    for layer in range(3):
        a, b = f.block_span[layer]
        assert all(n.startswith(f"blocks.{layer}.") for n in f.names[a:b])
        assert f.block_grad_span(layer).numel() >= sum(
            int(np.prod(f.shapes[n])) for n in f.names[a:b])
    assert "blocks.0.ffn.down.weight" in f.names and "blocks.0.rosa.payload" in f.names
    assert not any(n.endswith(k) for n in f.names for k, _ in _frozen_shapes(s))
    check_tokens(torch.tensor([[0, 299]]), 300)
    for bad in (torch.tensor([[0, 300]]), torch.tensor([[-100, 2]])):
        with pytest.raises(ValueError):
            check_tokens(bad, 300)
