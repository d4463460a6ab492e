"""Failure detection on the device without a GPU fault: a bounded in-kernel wait that runs out
must end its kernel and be reported by w8a8_ctx_check as W8A8_ERR_PEER_TIMEOUT, leaving the
context usable.  Two ranks of an LM head vocab-sharded over ranks are connected on one GPU and
only rank 0 ever runs a forward: its shard GEMV waits for rank 1's activations and its merge for
rank 1's candidates, flags that nothing sets.  Rank 1 launches nothing, so no two waiting kernels
share the GPU; every wait gives up after 1 to 2 s (no trap, no fault)."""
from __future__ import annotations

import time

import numpy as np
import pytest
import torch

from oracle import oracle as O
import romanaccio_b200 as rb
from romanaccio_b200 import _lib, synth

pytestmark = pytest.mark.gpu


def test_peer_wait_runs_out_and_is_reported():
    ctx = rb.Context(0)  # its own error word, apart from the session's context
    V, K, T, k = 4096, 256, 1, 8
    rng = np.random.default_rng(9)
    wq = rng.integers(-127, 128, size=(V, K)).astype(np.int8)
    in_step = 0.03
    acc = ((rng.random(V) * 1e-3 + 1e-5) * in_step).astype(np.float32)
    heads = []
    for r in range(2):
        lo, hi = rb.shard_range(V, 2, r)
        heads.append(rb.RankLmHead(ctx, r, 2, wq[lo:hi], acc[lo:hi], in_step, V, max_tokens=1,
                                   k_max=8))
    rb.RankLmHead.connect_local(heads)
    x = torch.from_numpy(synth.activations(T, K, seed=1).numpy()).cuda()
    t0 = time.time()
    heads[0].forward(x, k)  # rank 1 never publishes
    with pytest.raises(rb.W8A8Error) as e:
        ctx.check()
    elapsed = time.time() - t0
    assert e.value.status == _lib.ERR_PEER_TIMEOUT
    assert elapsed < 30, f"the kernels took {elapsed:.1f} s to give up"
    for h in heads:
        h.close()
    # the error was consumed and the context still works: a single-rank head on it is exact
    ctx.check()
    head = rb.RankLmHead(ctx, 0, 1, wq, acc, in_step, V, max_tokens=1, k_max=8)
    head.connect([head.export()])
    v, i, a = head.forward(x, k)
    lg = O.dequant_acc(O.gemm_i32(O.pack_static(x.cpu().numpy(), in_step), wq), acc)
    wv, wi = O.topk(lg, k)
    assert np.array_equal(i.cpu().numpy(), wi) and np.array_equal(v.cpu().numpy(), wv)
    ctx.check()
    head.close()
    ctx.close()
