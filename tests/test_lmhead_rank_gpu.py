"""The LM head vocab-sharded over ranks (w8a8_lmhead_rank_*, one rank per GPU): every rank's
merged top-k for its own tokens must equal the oracle's top-k over the whole vocabulary
(identical ids, bit-exact values), for several forwards in a row, driven eagerly and from a
CUDA graph.  Ranks never share a GPU (their kernels wait on one another), so the multi-rank
cases need as many GPUs as ranks and are skipped otherwise."""
from __future__ import annotations

import os
import socket

import numpy as np
import pytest
import torch

from oracle import oracle as O
import romanaccio_b200 as rb
from romanaccio_b200 import synth

pytestmark = pytest.mark.gpu


def _head(V, K, seed):
    rng = np.random.default_rng(seed)
    wq = rng.integers(-127, 128, size=(V, K)).astype(np.int8)
    w_step = rng.random(V) * 0.02 / 127 + 1e-5
    return wq, w_step


def _oracle(x, wq, in_step, acc_step, k):
    lg = O.dequant_acc(O.gemm_i32(O.pack_static(x, in_step), wq), acc_step)
    return O.topk(lg, k)


def test_single_rank(ctx):
    V, K, T, k = 49152, 576, 3, 40
    wq, w_step = _head(V, K, 1)
    in_step = 0.03
    acc = (in_step * w_step).astype(np.float32)
    head = rb.RankLmHead(ctx, 0, 1, wq, acc, in_step, V, max_tokens=8, k_max=64)
    handles = [head.export()]
    head.connect(handles)
    for it in range(3):
        x = synth.activations(T, K, seed=it).numpy()
        v, i, a = head.forward(torch.from_numpy(x).cuda(), k)
        wv, wi = _oracle(x, wq, in_step, acc, k)
        assert np.array_equal(i.cpu().numpy(), wi)
        assert np.array_equal(v.cpu().numpy(), wv)
        assert np.array_equal(a.cpu().numpy(), wi[:, 0])
    ctx.check()


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2,
                    reason="needs one GPU per rank")
@pytest.mark.parametrize("T", [1, 3])
def test_ranks_of_one_process_on_separate_gpus(T):
    n = min(torch.cuda.device_count(), 8)
    V, K, k = 151936, 1536, 40
    wq, w_step = _head(V, K, 2)
    in_step = 0.03
    acc = (in_step * w_step).astype(np.float32)
    ctxs = [rb.Context(d) for d in range(n)]
    heads = []
    for r in range(n):
        lo, hi = rb.shard_range(V, n, r)
        heads.append(rb.RankLmHead(ctxs[r], r, n, wq[lo:hi], acc[lo:hi], in_step, V,
                                   max_tokens=T, k_max=64))
    rb.RankLmHead.connect_local(heads)
    for it in range(3):
        xs = [synth.activations(T, K, seed=10 * it + r).numpy() for r in range(n)]
        outs = []
        for r in range(n):
            with torch.cuda.device(r):
                outs.append(heads[r].forward(torch.from_numpy(xs[r]).cuda(r), k))
        for r in range(n):
            torch.cuda.synchronize(r)
            wv, wi = _oracle(xs[r], wq, in_step, acc, k)
            v, i, a = outs[r]
            assert np.array_equal(i.cpu().numpy(), wi), f"rank {r} forward {it}: ids"
            assert np.array_equal(v.cpu().numpy(), wv), f"rank {r} forward {it}: values"
            assert np.array_equal(a.cpu().numpy(), wi[:, 0])
    for c in ctxs:
        c.check()


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank, world, port, result_q):
    import datetime
    import torch.distributed as dist
    try:
        torch.cuda.set_device(rank)
        dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank,
                                world_size=world, timeout=datetime.timedelta(seconds=60))
        V, K, T, k = 151936, 1536, 2, 40
        wq, w_step = _head(V, K, 3)
        in_step = 0.03
        acc = (in_step * w_step).astype(np.float32)
        ctx = rb.Context(rank)
        lo, hi = rb.shard_range(V, world, rank)
        head = rb.RankLmHead(ctx, rank, world, wq[lo:hi], acc[lo:hi], in_step, V,
                             max_tokens=T, k_max=64)
        handles = [None] * world
        dist.all_gather_object(handles, head.export())
        head.connect(handles)
        ok = True
        # eager forwards, then the same forward replayed from a CUDA graph
        h = torch.empty((T, K), dtype=torch.float32, device=f"cuda:{rank}")
        val = torch.empty((T, k), dtype=torch.float32, device=f"cuda:{rank}")
        idx = torch.empty((T, k), dtype=torch.int32, device=f"cuda:{rank}")
        am = torch.empty((T,), dtype=torch.int32, device=f"cuda:{rank}")
        for it in range(2):
            x = synth.activations(T, K, seed=100 * it + rank).numpy()
            h.copy_(torch.from_numpy(x))
            head.forward(h, k, val, idx, am)
            torch.cuda.synchronize()
            wv, wi = _oracle(x, wq, in_step, acc, k)
            ok &= bool(np.array_equal(idx.cpu().numpy(), wi) and
                       np.array_equal(val.cpu().numpy(), wv))
        g = torch.cuda.CUDAGraph()
        s = torch.cuda.Stream()
        with torch.cuda.graph(g, stream=s):
            head.forward(h, k, val, idx, am)
        for it in range(3):
            x = synth.activations(T, K, seed=1000 + 100 * it + rank).numpy()
            h.copy_(torch.from_numpy(x))
            torch.cuda.synchronize()
            dist.barrier()
            g.replay()
            torch.cuda.synchronize()
            wv, wi = _oracle(x, wq, in_step, acc, k)
            ok &= bool(np.array_equal(idx.cpu().numpy(), wi) and
                       np.array_equal(val.cpu().numpy(), wv) and
                       np.array_equal(am.cpu().numpy(), wi[:, 0]))
        ctx.check()
        del g
        dist.barrier()
        head.close()
        dist.destroy_process_group()
        result_q.put((rank, ok, ""))
    except Exception as e:  # reported to the parent
        result_q.put((rank, False, f"{type(e).__name__}: {e}"))


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2,
                    reason="needs one GPU per rank")
def test_ranks_as_processes():
    """One process per GPU, handles exchanged over a gloo group (set-up only); eager and
    graph-replayed forwards."""
    import torch.multiprocessing as mp
    world = min(torch.cuda.device_count(), 4)
    ctxm = mp.get_context("spawn")
    q = ctxm.Queue()
    port = _free_port()
    procs = [ctxm.Process(target=_rank_main, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = [q.get(timeout=300) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
    for rank, ok, msg in sorted(results):
        assert ok, f"rank {rank}: {msg or 'differs from the oracle'}"
