"""Parity of the CUDA W8A8 linear (through the C ABI) with the CPU oracle: bit-exact int8
activations, int32 accumulators, int8/int16 requantised outputs, and fp32 unpacked outputs,
every boundary stage separately and fused, over decode shapes, ragged shapes and full-size
layers of the decode workloads."""
from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import oracle as O
import romanaccio_b200 as rb
from romanaccio_b200 import synth

pytestmark = pytest.mark.gpu


def random_params(K: int, N: int, seed: int, out_i16: bool = False):
    rng = np.random.default_rng(seed)
    wq = rng.integers(-127, 128, size=(N, K)).astype(np.int8)
    qm = rng.integers(1, 32768, size=N).astype(np.int16)
    osc = (rng.random(N) * 0.01 + 1e-5).astype(np.float32)
    inv = (rng.random(K) * 3 + 0.05).astype(np.float32)
    acc_step = (rng.random(N) * 1e-4 + 1e-7).astype(np.float32)
    # trunc chosen so outputs spread over the int8 range with some saturation
    trunc = 14 if out_i16 else 22
    return dict(wq=wq, quant_m=qm, out_step_chan=osc, inv_smooth=inv, acc_step=acc_step, trunc=trunc)


def make_linear(ctx, p, in_thresh=3.0, in_step=0.05, out_i16=False, smooth=True, chan=True):
    scale = rb.SubgraphScaleInfo(in_dtype=rb.DTYPE_INT8,
                                 out_dtype=rb.DTYPE_INT16 if out_i16 else rb.DTYPE_INT8,
                                 in_thresh=in_thresh, in_step=in_step, out_step=0.0123,
                                 in_inv_smooth=p["inv_smooth"] if smooth else None,
                                 out_step_chan=p["out_step_chan"] if chan else None)
    return rb.W8A8Linear(ctx, p["wq"], scale, quant_m=p["quant_m"], trunc=p["trunc"],
                         acc_step=p["acc_step"])


def inputs(T, K, seed):
    return synth.activations(T, K, seed).numpy()


SHAPES = [
    (1, 576, 576), (1, 576, 192), (1, 1536, 256), (1, 1536, 2048), (2, 576, 1536),
    (3, 1536, 1536), (4, 96, 40), (8, 8960, 1536), (7, 100, 37), (1, 16, 8), (5, 1408, 2048),
    (12, 576, 1536), (1, 3840, 4096),
]


@pytest.mark.parametrize("T,K,N", SHAPES)
@pytest.mark.parametrize("dyntok", [True, False])
def test_boundary_stages_bit_exact(ctx, T, K, N, dyntok):
    p = random_params(K, N, seed=T * 7919 + K * 31 + N)
    lin = make_linear(ctx, p)
    x = inputs(T, K, seed=K + N)
    xd = torch.from_numpy(x).cuda()
    ratio_d = torch.zeros(T, dtype=torch.float32, device="cuda") if dyntok else None

    qd = lin.pack_npu_input(xd, dyntok_ratios=ratio_d)
    if dyntok:
        q, r = O.pack_dyntok(x, 3.0, p["inv_smooth"])
    else:
        q, r = O.pack_static(x, 0.05, p["inv_smooth"]), None
    torch.cuda.synchronize()
    assert np.array_equal(qd.cpu().numpy(), q)
    if dyntok:
        assert np.array_equal(ratio_d.cpu().numpy(), r)

    acc = O.gemm_i32(q, p["wq"])
    assert np.array_equal(lin.submit(qd, rb.OUT_ACC_I32).cpu().numpy(), acc)
    yq = O.requant(acc, p["quant_m"], p["trunc"], 127)
    yqd = lin.submit(qd, rb.OUT_QUANT)
    assert np.array_equal(yqd.cpu().numpy().astype(np.int32), yq)
    y = O.unpack(yq, 0.0123, p["out_step_chan"], r)
    assert np.array_equal(lin.unpack_npu_output(yqd, dyntok_ratios=ratio_d).cpu().numpy(), y)
    assert np.array_equal(lin.submit(qd, rb.OUT_F32, dyntok_ratios=ratio_d).cpu().numpy(), y)
    ya = O.dequant_acc(acc, p["acc_step"], r)
    assert np.array_equal(lin.submit(qd, rb.OUT_F32_ACC, dyntok_ratios=ratio_d).cpu().numpy(), ya)


@pytest.mark.parametrize("T,K,N", SHAPES)
@pytest.mark.parametrize("out_mode", [rb.OUT_ACC_I32, rb.OUT_QUANT, rb.OUT_F32, rb.OUT_F32_ACC])
def test_fused_forward_bit_exact(ctx, T, K, N, out_mode):
    p = random_params(K, N, seed=N * 13 + K)
    lin = make_linear(ctx, p)
    x = inputs(T, K, seed=T + K + N)
    q, r, acc, yq, y = O.linear(x, p["wq"], p["quant_m"], p["trunc"], p["out_step_chan"],
                                p["inv_smooth"], in_thresh=3.0)
    ratio_d = torch.empty(T, dtype=torch.float32, device="cuda")
    got = lin.forward(torch.from_numpy(x).cuda(), out_mode=out_mode, dyntok=True, ratios_out=ratio_d)
    got = got.cpu().numpy()
    want = {rb.OUT_ACC_I32: acc, rb.OUT_QUANT: yq.astype(np.int8), rb.OUT_F32: y,
            rb.OUT_F32_ACC: O.dequant_acc(acc, p["acc_step"], r)}[out_mode]
    assert np.array_equal(got, want)
    assert np.array_equal(ratio_d.cpu().numpy(), r)


@pytest.mark.parametrize("T,K,N", [(1, 1536, 1536), (6, 576, 200), (9, 1408, 64)])
def test_int16_requant_and_static_modes(ctx, T, K, N):
    p = random_params(K, N, seed=5, out_i16=True)
    lin = make_linear(ctx, p, out_i16=True, smooth=False, chan=False)
    x = inputs(T, K, seed=9)
    q = O.pack_static(x, 0.05, None)
    acc = O.gemm_i32(q, p["wq"])
    yq = O.requant(acc, p["quant_m"], p["trunc"], 32767)
    got = lin.forward(torch.from_numpy(x).cuda(), out_mode=rb.OUT_QUANT, dyntok=False)
    assert got.dtype == torch.int16
    assert np.array_equal(got.cpu().numpy().astype(np.int32), yq)
    y = O.unpack(yq, 0.0123, None, None)
    got = lin.forward(torch.from_numpy(x).cuda(), out_mode=rb.OUT_F32, dyntok=False)
    assert np.array_equal(got.cpu().numpy(), y)


def test_strided_and_unaligned_inputs(ctx):
    T, K, N = 3, 1000, 300
    p = random_params(K, N, seed=77)
    lin = make_linear(ctx, p)
    big = inputs(T, K + 24, seed=3)
    xd = torch.from_numpy(big).cuda()[:, 8:8 + K]  # row stride K+24, offset 32 bytes
    x = big[:, 8:8 + K]
    q, r, acc, yq, y = O.linear(x, p["wq"], p["quant_m"], p["trunc"], p["out_step_chan"],
                                p["inv_smooth"], in_thresh=3.0)
    got = lin.forward(xd, out_mode=rb.OUT_F32, dyntok=True)
    assert np.array_equal(got.cpu().numpy(), y)
    # int8 input at an odd address / stride goes through the staging copy
    qbuf = torch.zeros((T, K + 5), dtype=torch.int8, device="cuda")
    qbuf[:, 1:1 + K] = torch.from_numpy(q).cuda()
    got = lin.submit(qbuf[:, 1:1 + K], rb.OUT_ACC_I32)
    assert np.array_equal(got.cpu().numpy(), acc)


def test_extreme_values_and_saturation(ctx):
    """Max-magnitude weights/activations (int32 extremes of acc x QuantM 32767), NaN/inf inputs."""
    K, N, T = 4096, 64, 2
    wq = np.full((N, K), 127, np.int8)
    wq[1::2] = -127
    qm = np.full(N, 32767, np.int16)
    qm[:8] = np.arange(1, 9)
    p = dict(wq=wq, quant_m=qm, out_step_chan=np.full(N, 0.5, np.float32),
             inv_smooth=np.ones(K, np.float32), acc_step=np.full(N, 1e-3, np.float32), trunc=28)
    lin = make_linear(ctx, p)
    x = np.full((T, K), 1000.0, np.float32)
    x[1, ::3] = -1e30
    x[1, 5] = np.inf
    x[1, 7] = np.nan
    for dyn in (True, False):
        if dyn:
            q, r = O.pack_dyntok(x, 3.0, p["inv_smooth"])
        else:
            q, r = O.pack_static(x, 0.05, p["inv_smooth"]), None
        acc = O.gemm_i32(q, wq)
        yq = O.requant(acc, qm, 28, 127)
        y = O.unpack(yq, 0.0123, p["out_step_chan"], r)
        xd = torch.from_numpy(x).cuda()
        assert np.array_equal(lin.forward(xd, rb.OUT_ACC_I32, dyntok=dyn).cpu().numpy(), acc)
        got = lin.forward(xd, rb.OUT_F32, dyntok=dyn).cpu().numpy()
        np.testing.assert_array_equal(got, y)


@pytest.mark.parametrize("shape", [synth.QWEN25_15B, synth.SMOLLM_135M, synth.GEMMA_12B])
def test_full_size_decode_layer(ctx, shape):
    """Every subgraph of one decode layer at full size (T=1 and T=8), quantised with the
    reference's SmoothQuant/QuantM synthesis; bit-exact against the oracle."""
    for i, (name, K, N, trunc) in enumerate(shape.subgraphs()):
        p = synth.make_linear(K, N, seed=100 + i, trunc=trunc)
        scale = rb.SubgraphScaleInfo(in_dtype=rb.DTYPE_INT8, out_dtype=rb.DTYPE_INT8,
                                     in_thresh=p.in_thresh, in_step=p.in_step,
                                     in_inv_smooth=p.in_inv_smooth, out_step_chan=p.out_step_chan)
        lin = rb.W8A8Linear(ctx, p.wq, scale, quant_m=p.quant_m, trunc=p.trunc, acc_step=p.acc_step)
        for T in (1, 8):
            x = inputs(T, K, seed=i + T)
            *_, yq, y = O.linear(x, p.wq, p.quant_m, p.trunc, p.out_step_chan, p.in_inv_smooth,
                                 in_thresh=p.in_thresh)
            got = lin.forward(torch.from_numpy(x).cuda(), rb.OUT_F32, dyntok=True)
            assert np.array_equal(got.cpu().numpy(), y), (name, T)
        lin.close()


def test_repeated_calls_and_errors(ctx):
    p = random_params(256, 128, seed=1)
    lin = make_linear(ctx, p)
    x = torch.from_numpy(inputs(1, 256, seed=1)).cuda()
    first = lin.forward(x, rb.OUT_F32).cpu()
    for _ in range(50):
        assert torch.equal(lin.forward(x, rb.OUT_F32).cpu(), first)
    with pytest.raises(ValueError):
        lin.forward(x[:, :100], rb.OUT_F32)  # K mismatch
    nolin = rb.W8A8Linear(ctx, p["wq"], rb.SubgraphScaleInfo(), quant_m=None)
    with pytest.raises(rb.W8A8Error):
        nolin.forward(x, rb.OUT_QUANT)
    ctx.check()


@pytest.mark.parametrize("n", [2, 3, 4])
def test_column_split_tensor_parallel(ctx, n):
    """Column-split TP (output-channel shards sharing the input side): the shards' outputs,
    concatenated, equal the unsplit linear's and the oracle's, for every output mode."""
    from romanaccio_b200.quantize import split_columns
    T, K, N = 5, 1536, 2304
    p = synth.make_linear(K, N, seed=40 + n)
    full = rb.W8A8Linear.from_params(ctx, p)
    shards = [rb.W8A8Linear.from_params(ctx, s) for s in split_columns(p, n)]
    x = synth.activations(T, K, seed=n).cuda()
    for mode in (rb.OUT_ACC_I32, rb.OUT_QUANT, rb.OUT_F32, rb.OUT_F32_ACC):
        want = full.forward(x, out_mode=mode, dyntok=True).cpu()
        got = torch.cat([s.forward(x, out_mode=mode, dyntok=True).cpu() for s in shards], dim=1)
        assert torch.equal(got, want)
    q, r = O.pack_dyntok(x.cpu().numpy(), p.in_thresh, p.in_inv_smooth)
    yq = O.requant(O.gemm_i32(q, p.wq), p.quant_m, p.trunc, 127)
    got = torch.cat([s.forward(x, out_mode=rb.OUT_QUANT, dyntok=True).cpu() for s in shards], dim=1)
    assert np.array_equal(got.numpy().astype(np.int32), yq)
