"""Expert-parallel MoE combine on CPU, world-size-2 and 4 gloo ranks: each rank combines the
slots of the experts it owns (e % world == rank) in slot order, the partials are all-gathered
and added in rank order, and the result must equal the oracle's expert-parallel combine.  The
restatement itself is pinned to the C oracle's single-rank combine (lfm2_moe.cpp:2300-2318),
and for two ranks it is the reference's even / odd die split with the dies' sums added after
(lfm2_moe.cpp:2190-2432)."""
from __future__ import annotations

import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from oracle import oracle as O

T, K_TOP, S, E, H = 6, 3, 2, 16, 96
SLOTS = K_TOP + S


def _problem():
    rng = np.random.default_rng(4)
    idx = np.stack([rng.choice(E, K_TOP, replace=False) for _ in range(T)]).astype(np.int32)
    w = rng.random((T, K_TOP)).astype(np.float32)
    yq = rng.integers(-127, 128, (T * SLOTS, H)).astype(np.int32)
    osc = (rng.random((E + S, H)) * 0.01).astype(np.float32)
    return yq, idx, w, osc


def test_restatement_equals_single_rank_combine():
    yq, idx, w, osc = _problem()
    assert np.array_equal(O.moe_combine_ep(yq, idx, w, osc, E, SLOTS, 1),
                          O.moe_combine(yq, idx, w, osc, E, SLOTS))


def test_two_ranks_are_the_even_odd_die_split():
    yq, idx, w, osc = _problem()
    dies = []
    for parity in (0, 1):
        acc = np.zeros((T, H), np.float32)
        for t in range(T):
            for j in range(SLOTS):
                e = int(idx[t, j]) if j < K_TOP else E + (j - K_TOP)
                if e % 2 != parity:
                    continue
                wj = w[t, j] if j < K_TOP else np.float32(1)
                acc[t] = acc[t] + yq[t * SLOTS + j].astype(np.float32) * (np.float32(wj) * osc[e])
        dies.append(acc)
    want = (np.zeros((T, H), np.float32) + dies[0]) + dies[1]
    assert np.array_equal(O.moe_combine_ep(yq, idx, w, osc, E, SLOTS, 2), want)


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank: int, world: int, port: int, q) -> None:
    import sys
    from pathlib import Path
    sys.path.insert(0, str(Path(__file__).resolve().parent.parent))
    from oracle import oracle as O2

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        yq, idx, w, osc = _problem()
        # this rank's partial: its own slots only (the other ranks' yq rows zeroed out would
        # change nothing; the owner test below is what the device combine applies)
        part = np.zeros((T, H), np.float32)
        for t in range(T):
            for j in range(SLOTS):
                e = int(idx[t, j]) if j < K_TOP else E + (j - K_TOP)
                if e % world != rank:
                    continue
                wj = w[t, j] if j < K_TOP else np.float32(1)
                part[t] = part[t] + yq[t * SLOTS + j].astype(np.float32) * (np.float32(wj) * osc[e])
        gathered = [torch.empty((T, H), dtype=torch.float32) for _ in range(world)]
        dist.all_gather(gathered, torch.from_numpy(part))
        out = np.zeros((T, H), np.float32)
        for g in gathered:
            out = out + g.numpy()
        q.put((rank, bool(np.array_equal(out, O2.moe_combine_ep(yq, idx, w, osc, E, SLOTS, world)))))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 4])
def test_gloo_ranks_reproduce_the_expert_parallel_combine(world):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = [q.get(timeout=120) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
    assert all(ok for _, ok in res), res
