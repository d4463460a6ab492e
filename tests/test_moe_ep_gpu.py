"""Expert-parallel MoE layer (w8a8_moe_ep_*): every rank's output must equal the oracle's
expert-parallel combine of the ranks' requantised expert outputs (each rank contributing its own
experts, e % world == rank), bit for bit, with routing identical to the oracle's and each owned
expert stage bit-exact; several forwards in a row (the exchange's double buffer alternates).
Ranks never share a GPU (their kernels wait on one another): multi-rank cases need one GPU per
rank and are skipped otherwise."""
from __future__ import annotations

import socket

import numpy as np
import pytest
import torch

from oracle import oracle as O
import romanaccio_b200 as rb
from romanaccio_b200 import synth
from romanaccio_b200.moe import ExpertParallelMoE, MoELayer, make_moe_params

pytestmark = pytest.mark.gpu

H, I, E, S, K_TOP = 2048, 1408, 64, 2, 6


def _owned_stage_ok(layer, p, x, v, world, rank, sample=8):
    """Bit-exact gate|up and down stages of a sample of this rank's own pairs."""
    slots = K_TOP + S
    T = x.shape[0]
    owned = []
    for pi in range(T * slots):
        t, j = divmod(pi, slots)
        e = int(v["idx"][t, j]) if j < K_TOP else E + (j - K_TOP)
        if e % world == rank:
            owned.append((pi, t, e))
    for pi, t, e in owned[:sample]:
        gu, dn = p.gu[e], p.dn[e]
        q, r = O.pack_dyntok(x[t:t + 1], gu.in_thresh, gu.in_inv_smooth)
        yq = O.requant(O.gemm_i32(q, gu.wq), gu.quant_m, gu.trunc, 127)
        if not np.array_equal(v["gate_up"][pi:pi + 1], O.unpack(yq, 0.0, gu.out_step_chan, r)):
            return False
        q2 = O.pack_static(v["act"][pi:pi + 1], dn.in_step, dn.in_inv_smooth)
        want = O.requant(O.gemm_i32(q2, dn.wq), dn.quant_m, dn.trunc, 127)
        if not np.array_equal(v["down_q"][pi:pi + 1].astype(np.int32), want):
            return False
    return True


def _assemble_yq(views, world):
    """The requantised expert outputs of every pair, each taken from the rank that owns it."""
    slots = K_TOP + S
    idx = views[0]["idx"]
    T = idx.shape[0]
    yq = np.zeros_like(views[0]["down_q"]).astype(np.int32)
    for pi in range(T * slots):
        t, j = divmod(pi, slots)
        e = int(idx[t, j]) if j < K_TOP else E + (j - K_TOP)
        yq[pi] = views[e % world]["down_q"][pi]
    return yq


def test_single_rank_equals_whole_layer(ctx):
    p = make_moe_params(H=H, I=I, E=E, S=S, k=K_TOP, seed=3, device="cuda")
    layer = MoELayer(ctx, p, max_tokens=64)
    ep = ExpertParallelMoE(layer, 0, 1)
    ep.connect([ep.export()])
    for it, T in enumerate((1, 8, 64)):
        x = synth.activations(T, H, seed=200 + it).numpy()
        out = ep.forward(torch.from_numpy(x).cuda()).cpu().numpy()
        v = {k: t.cpu().numpy() for k, t in layer.views(T).items()}
        idx, _ = O.moe_route(x, p.gate_w, K_TOP)
        assert np.array_equal(v["idx"], idx)
        osc = np.stack([q.out_step_chan for q in p.dn])
        want = O.moe_combine_ep(v["down_q"], v["idx"], v["w"], osc, E, K_TOP + S, 1)
        assert np.array_equal(out, want)
        assert _owned_stage_ok(layer, p, x, v, 1, 0)
    ctx.check()


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2,
                    reason="needs one GPU per rank")
def test_ranks_of_one_process_on_separate_gpus():
    n = min(torch.cuda.device_count(), 8)
    ctxs = [rb.Context(d) for d in range(n)]
    layers, eps, ps = [], [], []
    for r in range(n):
        with torch.cuda.device(r):
            p = make_moe_params(H=H, I=I, E=E, S=S, k=K_TOP, seed=3, device=f"cuda:{r}")
            ps.append(p)
            layers.append(MoELayer(ctxs[r], p, max_tokens=64))
            eps.append(ExpertParallelMoE(layers[r], r, n))
    ExpertParallelMoE.connect_local(eps)
    osc = np.stack([q.out_step_chan for q in ps[0].dn])
    for it, T in enumerate((1, 64, 1)):
        x = synth.activations(T, H, seed=300 + it).numpy()
        outs = []
        for r in range(n):
            with torch.cuda.device(r):
                outs.append(eps[r].forward(torch.from_numpy(x).cuda(r)))
        for r in range(n):
            torch.cuda.synchronize(r)
        views = [{k: t.cpu().numpy() for k, t in layers[r].views(T).items()} for r in range(n)]
        idx, _ = O.moe_route(x, ps[0].gate_w, K_TOP)
        want = O.moe_combine_ep(_assemble_yq(views, n), views[0]["idx"], views[0]["w"], osc, E,
                                K_TOP + S, n)
        for r in range(n):
            assert np.array_equal(views[r]["idx"], idx), f"rank {r}: routing"
            assert np.array_equal(outs[r].cpu().numpy(), want), f"rank {r} forward {it}: output"
            assert _owned_stage_ok(layers[r], ps[r], x, views[r], n, r, sample=4)
    for c in ctxs:
        c.check()


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank, world, port, q):
    import datetime
    import torch.distributed as dist
    try:
        torch.cuda.set_device(rank)
        dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank,
                                world_size=world, timeout=datetime.timedelta(seconds=60))
        ctx = rb.Context(rank)
        p = make_moe_params(H=H, I=I, E=E, S=S, k=K_TOP, seed=3, device=f"cuda:{rank}")
        layer = MoELayer(ctx, p, max_tokens=64)
        ep = ExpertParallelMoE(layer, rank, world)
        handles = [None] * world
        dist.all_gather_object(handles, ep.export())
        ep.connect(handles)
        osc = np.stack([qq.out_step_chan for qq in p.dn])
        ok = True
        for it, T in enumerate((1, 64, 8)):
            x = synth.activations(T, H, seed=400 + it).numpy()
            out = ep.forward(torch.from_numpy(x).cuda()).cpu().numpy()
            v = {k: t.cpu().numpy() for k, t in layer.views(T).items()}
            parts = [None] * world
            dist.all_gather_object(parts, v)
            want = O.moe_combine_ep(_assemble_yq(parts, world), v["idx"], v["w"], osc, E,
                                    K_TOP + S, world)
            ok &= bool(np.array_equal(out, want))
            ok &= _owned_stage_ok(layer, p, x, v, world, rank, sample=4)
        ctx.check()
        dist.barrier()
        ep.close()
        dist.destroy_process_group()
        q.put((rank, ok, ""))
    except Exception as e:
        q.put((rank, False, f"{type(e).__name__}: {e}"))


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2,
                    reason="needs one GPU per rank")
def test_ranks_as_processes():
    import torch.multiprocessing as mp
    world = min(torch.cuda.device_count(), 4)
    c = mp.get_context("spawn")
    q = c.Queue()
    port = _free_port()
    procs = [c.Process(target=_rank_main, args=(r, world, port, q)) for r in range(world)]
    for pr in procs:
        pr.start()
    res = [q.get(timeout=300) for _ in range(world)]
    for pr in procs:
        pr.join(timeout=60)
    for rank, ok, msg in sorted(res):
        assert ok, f"rank {rank}: {msg or 'differs from the oracle'}"
