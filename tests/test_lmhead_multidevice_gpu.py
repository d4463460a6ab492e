"""The single-process, multi-device LM head (w8a8_lmhead_*): shards on one device (every shard
count) and, when the box has them, on several devices; the merged top-k and argmax must equal
the oracle's top-k over the full vocabulary (bit-exact values, identical ids)."""
from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import oracle as O
import romanaccio_b200 as rb
from romanaccio_b200 import synth

from test_lmhead_gpu import lm_params, oracle_logits

pytestmark = pytest.mark.gpu


def _check(lm, x, wq, in_step, acc_step, k):
    val, idx, am = lm.forward(torch.from_numpy(x).cuda(lm.device), k)
    torch.cuda.synchronize()
    lg = oracle_logits(x, wq, in_step, acc_step)
    wv, wi = O.topk(lg, k)
    assert np.array_equal(idx.cpu().numpy(), wi)
    assert np.array_equal(val.cpu().numpy(), wv)
    assert np.array_equal(am.cpu().numpy(), wi[:, 0])


@pytest.mark.parametrize("n,V,K,T,k", [
    (1, 49152, 576, 1, 40), (2, 49152, 576, 1, 40), (3, 20000, 1536, 2, 40),
    (4, 151936, 1536, 1, 40), (8, 151936, 1536, 3, 64), (2, 1000, 64, 5, 7),
])
def test_shards_on_one_device(ctx, n, V, K, T, k):
    wq, w_step = lm_params(V, K, seed=V + n)
    in_step = 0.031
    acc_step = (in_step * w_step).astype(np.float32)
    lm = rb.MultiDeviceLmHead([ctx] * n, wq, acc_step, in_step, max_tokens=8, k_max=64)
    assert lm.shards == n
    x = synth.activations(T, K, seed=n + T).numpy()
    _check(lm, x, wq, in_step, acc_step, k)
    # repeated calls reuse the gather buffers and streams
    _check(lm, synth.activations(T, K, seed=99).numpy(), wq, in_step, acc_step, k)


def test_graph_capture(ctx):
    """With every shard on device 0 the whole forward is ordered on one stream: capturable."""
    V, K, T, k, n = 65536, 1536, 1, 40, 4
    wq, w_step = lm_params(V, K, seed=5)
    in_step = 0.02
    acc_step = (in_step * w_step).astype(np.float32)
    lm = rb.MultiDeviceLmHead([ctx] * n, wq, acc_step, in_step, max_tokens=4, k_max=40)
    x = torch.from_numpy(synth.activations(T, K, seed=7).numpy()).cuda()
    val = torch.empty((T, k), dtype=torch.float32, device="cuda")
    idx = torch.empty((T, k), dtype=torch.int32, device="cuda")
    am = torch.empty((T,), dtype=torch.int32, device="cuda")
    s = torch.cuda.Stream()
    with torch.cuda.stream(s):
        lm.forward(x, k, val, idx, am)
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        lm.forward(x, k, val, idx, am)
    val.zero_()
    idx.zero_()
    g.replay()
    torch.cuda.synchronize()
    lg = oracle_logits(x.cpu().numpy(), wq, in_step, acc_step)
    wv, wi = O.topk(lg, k)
    assert np.array_equal(idx.cpu().numpy(), wi)
    assert np.array_equal(val.cpu().numpy(), wv)


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 or more GPUs")
def test_shards_on_several_devices():
    n = min(torch.cuda.device_count(), 8)
    before = torch.cuda.current_device()
    ctxs = [rb.Context(d) for d in range(n)]
    # Creating contexts on other devices leaves the caller's current device alone.
    assert torch.cuda.current_device() == before
    V, K, k = 151936, 1536, 40
    wq, w_step = lm_params(V, K, seed=11)
    in_step = 0.031
    acc_step = (in_step * w_step).astype(np.float32)
    lm = rb.MultiDeviceLmHead(ctxs, wq, acc_step, in_step, max_tokens=8, k_max=64)
    # consecutive forwards advance the cross-device counters; token counts vary
    for i, T in enumerate((2, 1, 8, 3, 1)):
        x = synth.activations(T, K, seed=12 + i).numpy()
        _check(lm, x, wq, in_step, acc_step, k if i != 3 else 64)
    for c in ctxs:
        c.check()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 or more GPUs")
def test_mixed_local_and_remote_shards():
    """Shards 0 and 1 on device 0 (stream-ordered), shards 2 and 3 on device 1 (counters)."""
    c0, c1 = rb.Context(0), rb.Context(1)
    V, K, k = 40000, 1024, 40
    wq, w_step = lm_params(V, K, seed=21)
    in_step = 0.027
    acc_step = (in_step * w_step).astype(np.float32)
    lm = rb.MultiDeviceLmHead([c0, c0, c1, c1], wq, acc_step, in_step, max_tokens=4, k_max=40)
    for i in range(3):
        x = synth.activations(1 + i, K, seed=30 + i).numpy()
        _check(lm, x, wq, in_step, acc_step, k)
    c0.check()
    c1.check()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 or more GPUs")
def test_remote_shards_refuse_graph_capture():
    c0, c1 = rb.Context(0), rb.Context(1)
    V, K, T, k = 8192, 512, 1, 16
    wq, w_step = lm_params(V, K, seed=3)
    acc_step = (0.02 * w_step).astype(np.float32)
    lm = rb.MultiDeviceLmHead([c0, c1], wq, acc_step, 0.02, max_tokens=2, k_max=16)
    x = torch.from_numpy(synth.activations(T, K, seed=4).numpy()).cuda(0)
    val = torch.empty((T, k), dtype=torch.float32, device="cuda:0")
    idx = torch.empty((T, k), dtype=torch.int32, device="cuda:0")
    g = torch.cuda.CUDAGraph()
    with pytest.raises(RuntimeError, match="graph-captured"):
        with torch.cuda.graph(g):
            lm.forward(x, k, val, idx)
    del g
    torch.cuda.synchronize()
    # the head still works outside capture
    _check(lm, synth.activations(T, K, seed=5).numpy(), wq, 0.02, acc_step, k)
    c0.check()
    c1.check()
    with pytest.raises(RuntimeError, match="max_tokens"):
        rb.MultiDeviceLmHead([c0, c1], wq, acc_step, 0.02, max_tokens=9, k_max=16)


_BIG = {}


def _device_head(V: int, K: int, seed: int):
    """Seeded int8 rows generated on the GPU (a 1 GB head would take minutes in numpy)."""
    key = (V, K, seed)
    if key not in _BIG:
        g = torch.Generator(device="cuda").manual_seed(seed)
        wq = torch.randint(-127, 128, (V, K), generator=g, device="cuda", dtype=torch.int32)
        w_step = torch.rand((V,), generator=g, device="cuda", dtype=torch.float64) * 0.02 / 127 + 1e-5
        _BIG.clear()
        _BIG[key] = (wq.to(torch.int8).cpu().numpy(), w_step.cpu().numpy())
    return _BIG[key]


@pytest.mark.parametrize("V,K,n", [
    (102400, 2048, 2), (102400, 2048, 4), (102400, 2048, 8),
    (262144, 3840, 2), (262144, 3840, 4), (262144, 3840, 8),
])
def test_config_heads_sharded_on_one_device(ctx, V, K, n):
    """The DeepSeek-V2-Lite (102400 x 2048) and Gemma-12B-class (262144 x 3840) LM heads in 2, 4
    and 8 contiguous vocab shards, merged: the oracle's top-40 over the whole vocabulary."""
    wq, w_step = _device_head(V, K, seed=V)
    in_step = 0.027
    acc_step = (in_step * w_step).astype(np.float32)
    lm = rb.MultiDeviceLmHead([ctx] * n, wq, acc_step, in_step, max_tokens=8, k_max=64)
    assert lm.shards == n
    _check(lm, synth.activations(1, K, seed=n).numpy(), wq, in_step, acc_step, 40)
    ctx.check()
