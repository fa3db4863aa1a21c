"""Expert-parallel host logic on CPU ranks (gloo, world size 2): placement,
replicated routing, zero rows for remote experts, sum over ranks, ordered
combine -- the same composition the GPU layer runs with NCCL -- must equal
the single-process layer.  The expert math here is the oracle (torch CPU)."""

from __future__ import annotations

import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from voom_b200.runtime.moe import place_experts, route_rows, zipf_popularity


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _make(E=12, H=64, I=32, seed=3):
    g = torch.Generator().manual_seed(seed)
    ex = [tuple((torch.randn(sh, generator=g) * 0.05).to(torch.bfloat16) for sh in ((I, H), (I, H), (H, I)))
          for _ in range(E)]
    wr = torch.randn((E, H), generator=g).to(torch.bfloat16)
    x = torch.randn((5, H), generator=g).to(torch.bfloat16)
    return ex, wr, x


def _ep_forward(rank: int, world: int, ex, wr, x, k: int):
    from oracle import moe as om

    owned = place_experts(np.ones(len(ex)), world)[rank]
    h = x
    idx, pw = om.route(h, wr, k, True)
    order, ntok, uoff, upair, tok_order = route_rows(idx.numpy())
    y = torch.zeros((x.shape[0] * k, x.shape[1]), dtype=torch.float32)
    for u, e in enumerate(order):
        if e in owned:
            rows = list(range(uoff[u], uoff[u + 1]))
            y[rows] = om.swiglu(h[[upair[q] for q in rows]], *ex[e]).float()
    dist.all_reduce(y)  # exact: one nonzero contributor per row
    wrow = torch.zeros(len(upair))
    for t in range(x.shape[0]):
        for j in range(k):
            e = int(idx[t, j])
            u = order.index(e)
            q = next(q for q in range(uoff[u], uoff[u + 1]) if upair[q] == t)
            wrow[q] = float(pw[t, j])
    out = torch.zeros_like(x)
    for t in range(x.shape[0]):
        for q in tok_order[t]:
            contrib = (y[q].to(torch.bfloat16).float() * wrow[q].to(torch.bfloat16).float()).to(torch.bfloat16)
            out[t] = (out[t].float() + contrib.float()).to(torch.bfloat16)
    return (x.float() + out.float()).to(torch.bfloat16)


def _worker(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        ex, wr, x = _make()
        got = _ep_forward(rank, world, ex, wr, x, 3)
        q.put((rank, got.view(torch.int16).numpy().tobytes()))
    finally:
        dist.destroy_process_group()


def test_expert_parallel_matches_single_process():
    from oracle import moe as om

    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=120) for _ in range(2))
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    ex, wr, x = _make()
    ref = om.moe_layer(x, wr, None, ex, 3, True)
    for r in range(2):
        assert res[r] == ref.view(torch.int16).numpy().tobytes(), r


def test_lpt_placement_balances_zipf_load():
    p = zipf_popularity(160, 1.1, seed=0)
    for world in (2, 4, 8):
        bins = place_experts(p, world)
        assert sorted(e for b in bins for e in b) == list(range(160))
        loads = [p[b].sum() for b in bins]
        assert max(loads) <= (1 / world) * 1.6 + p.max()


def test_route_rows_matches_reference_order():
    idx = np.array([[3, 1], [1, 2], [0, 3]])
    order, ntok, uoff, upair, tok_order = route_rows(idx)
    assert order == [3, 1, 2, 0] and ntok == [2, 2, 1, 1]
    assert list(uoff) == [0, 2, 4, 5, 6] and upair == [0, 2, 0, 1, 1, 2]
    assert tok_order == [[0, 2], [3, 4], [1, 5]]
