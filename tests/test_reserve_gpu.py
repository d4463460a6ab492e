"""w8a8_linear_reserve: after one set-up call, forwards of up to the reserved token count (GEMV
and tensor-core paths, split-K planes, 16+ token top-k scratch) allocate and synchronise nothing.
Checked by capturing them in a CUDA graph (any cudaMalloc or synchronous cudaMemset inside a
capture fails it) and comparing the replayed outputs with the oracle."""
from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import oracle as O
import romanaccio_b200 as rb
from romanaccio_b200 import synth

pytestmark = pytest.mark.gpu


def test_reserved_forwards_capture_and_match_oracle(ctx):
    K, N = 1536, 2048
    p = synth.make_linear(K, N, seed=11)
    scale = rb.SubgraphScaleInfo(in_dtype=rb.DTYPE_INT8, out_dtype=rb.DTYPE_INT8,
                                 in_thresh=p.in_thresh, in_step=p.in_step,
                                 in_inv_smooth=p.in_inv_smooth, out_step_chan=p.out_step_chan)
    lin = rb.W8A8Linear(ctx, p.wq, scale, quant_m=p.quant_m, trunc=p.trunc, acc_step=p.acc_step)
    V, Kh, Th, k, in_step = 30000, 1024, 32, 40, 0.029
    rng = np.random.default_rng(5)
    wh = rng.integers(-127, 128, size=(V, Kh)).astype(np.int8)
    acc_h = (rng.random(V) * 1e-4 + 1e-6).astype(np.float32)
    shard = rb.LmHeadShard(ctx, wh, acc_h, in_step, row_offset=3)

    lin.reserve(64)
    shard.linear.reserve(Th, k)
    torch.cuda.synchronize()

    Ts = (1, 8, 16, 64)
    xs = {T: torch.from_numpy(synth.activations(T, K, seed=T).numpy()).cuda() for T in Ts}
    ys = {T: torch.empty((T, N), dtype=torch.float32, device="cuda") for T in Ts}
    xh = torch.from_numpy(synth.activations(Th, Kh, seed=9).numpy()).cuda()
    vh = torch.empty((Th, k), dtype=torch.float32, device="cuda")
    ih = torch.empty((Th, k), dtype=torch.int32, device="cuda")

    def step():
        for T in Ts:
            lin.forward(xs[T], rb.OUT_F32, dyntok=True, out=ys[T])
        shard.forward(xh, k, val=vh, idx=ih)

    # one eager pass loads the kernels; the capture then fails if any call allocates
    step()
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        step()
    for T in Ts:
        ys[T].zero_()
    vh.zero_()
    ih.zero_()
    g.replay()
    torch.cuda.synchronize()

    for T in Ts:
        *_, y_ref = O.linear(xs[T].cpu().numpy(), p.wq, p.quant_m, p.trunc, p.out_step_chan,
                             p.in_inv_smooth, in_thresh=p.in_thresh)
        assert np.array_equal(ys[T].cpu().numpy(), y_ref), f"T={T}: output differs from the oracle"
    lg = O.dequant_acc(O.gemm_i32(O.pack_static(xh.cpu().numpy(), in_step, None), wh), acc_h)
    wv, wi = O.topk(lg, k, id_offset=3)
    assert np.array_equal(ih.cpu().numpy(), wi)
    assert np.array_equal(vh.cpu().numpy(), wv)
    del g
    ctx.check()


def test_reserve_rejects_bad_limits(ctx):
    p = synth.make_linear(64, 32, seed=2)
    scale = rb.SubgraphScaleInfo(in_dtype=rb.DTYPE_INT8, out_dtype=rb.DTYPE_INT8,
                                 in_thresh=p.in_thresh, in_step=p.in_step,
                                 in_inv_smooth=p.in_inv_smooth, out_step_chan=p.out_step_chan)
    lin = rb.W8A8Linear(ctx, p.wq, scale, quant_m=p.quant_m, trunc=p.trunc, acc_step=p.acc_step)
    with pytest.raises(rb.W8A8Error, match="max_tokens"):
        lin.reserve(0)
    with pytest.raises(rb.W8A8Error, match="max_k"):
        lin.reserve(4, rb.TOPK_MAX + 1)
