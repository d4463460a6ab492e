"""Multi-rank LM-head exchange on CPU: world-size-2 (and 4) gloo ranks run the exact host logic
of the sharded LM head (contiguous vocab split, [2, T_all, k] candidate blocks, all-gather,
per-rank token views) with the shard top-k and the merge computed by the CPU oracle, and must
reproduce the unsharded top-k / greedy argmax."""
from __future__ import annotations

import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from romanaccio_b200.lmhead import (candidate_buffers, exchange_candidates, shard_range,
                                    token_candidates)

V, K, T, KTOP = 5000, 64, 3, 40


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _problem():
    rng = np.random.default_rng(0)
    wq = rng.integers(-127, 128, size=(V, K)).astype(np.int8)
    acc_step = (rng.random(V) * 1e-3 + 1e-6).astype(np.float32)
    return wq, acc_step


def _worker(rank: int, world: int, port: int, q) -> None:
    import sys
    from pathlib import Path
    sys.path.insert(0, str(Path(__file__).resolve().parent.parent))
    from oracle import oracle as O

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        wq, acc_step = _problem()
        # every rank decodes its own T tokens; hidden states are all-gathered
        h_local = torch.from_numpy(np.random.default_rng(100 + rank).standard_normal((T, K)).astype(np.float32))
        h_all = torch.empty((world * T, K), dtype=torch.float32)
        dist.all_gather_into_tensor(h_all, h_local)
        lo, hi = shard_range(V, world, rank)
        x = h_all.numpy()
        lg = O.dequant_acc(O.gemm_i32(O.pack_static(x, 0.04), wq[lo:hi]), acc_step[lo:hi])
        val, idx = O.topk(lg, KTOP, id_offset=lo)
        local, gathered = candidate_buffers(world * T, KTOP, world, "cpu")
        local[0].copy_(torch.from_numpy(val).view(torch.int32))
        local[1].copy_(torch.from_numpy(idx))
        exchange_candidates(local, gathered)
        vals, ids = token_candidates(gathered, world, rank * T, T)
        assert vals.shape == (T, world, KTOP)
        merged = []
        for t in range(T):
            v = vals[t].reshape(-1).numpy()
            i = ids[t].reshape(-1).numpy()
            order = sorted(range(len(v)), key=lambda j: (-v[j], i[j]))[:KTOP]
            merged.append(i[order])
        # unsharded reference for this rank's tokens
        full = O.dequant_acc(O.gemm_i32(O.pack_static(h_local.numpy(), 0.04), wq), acc_step)
        _, want = O.topk(full, KTOP)
        ok = all(np.array_equal(merged[t], want[t]) for t in range(T))
        ok = ok and all(merged[t][0] == O.argmax(full[t]) for t in range(T))
        q.put((rank, ok))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 4])
def test_sharded_lm_head_exchange_gloo(world):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = dict(q.get(timeout=300) for _ in range(world))
    for p in procs:
        p.join(timeout=60)
    assert all(p.exitcode == 0 for p in procs)
    assert all(results[r] for r in range(world)), results


def test_shard_range_is_contiguous_halves():
    """dual_die_splitter.py:63-147: die 0 gets [0, V//2), die 1 the rest."""
    for V_ in (49152, 151936, 102400, 262144, 7):
        assert shard_range(V_, 2, 0) == (0, V_ // 2)
        assert shard_range(V_, 2, 1) == (V_ // 2, V_)
        for n in (1, 2, 4, 8):
            rngs = [shard_range(V_, n, r) for r in range(n)]
            assert rngs[0][0] == 0 and rngs[-1][1] == V_
            assert all(a[1] == b[0] for a, b in zip(rngs, rngs[1:]))
