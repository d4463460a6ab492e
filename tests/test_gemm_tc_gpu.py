"""Parity of the tensor-core (tcgen05 kind::i8) contraction with the CPU oracle and with the GEMV
path: int32 accumulators, int8/int16 requant and fp32 outputs bit-exact, over batched-decode and
prefill shapes (ragged token / channel / K tails, split-K and multi-token-block plans), and the
prefill sweep at full size through sampled rows checked against the oracle."""
from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import oracle as O
import romanaccio_b200 as rb
from romanaccio_b200 import synth
from romanaccio_b200._lib import PATH_GEMV, PATH_TENSOR, PATH_TENSOR_PAIR

from test_linear_gpu import inputs, make_linear, random_params

pytestmark = pytest.mark.gpu


def _oracle_outputs(p, q, r):
    acc = O.gemm_i32(q, p["wq"])
    yq = O.requant(acc, p["quant_m"], p["trunc"], 127)
    return acc, yq, O.unpack(yq, 0.0123, p["out_step_chan"], r), O.dequant_acc(acc, p["acc_step"], r)


# (T, K, N): ragged channels and K, one and several token blocks, split and unsplit K.
SHAPES = [
    (16, 576, 576), (17, 100, 37), (32, 1536, 1536), (33, 1536, 256), (64, 8960, 1536),
    (128, 2048, 2048), (200, 1408, 2048), (256, 576, 1536), (300, 576, 1536), (513, 160, 136),
    (40, 16, 8),
]


@pytest.mark.parametrize("T,K,N", SHAPES)
@pytest.mark.parametrize("dyntok", [True, False])
def test_tensor_path_bit_exact(ctx, T, K, N, dyntok):
    p = random_params(K, N, seed=T * 131 + K * 7 + N)
    lin = make_linear(ctx, p)
    lin.set_path(PATH_TENSOR)
    x = inputs(T, K, seed=T + K + N)
    xd = torch.from_numpy(x).cuda()
    ratio_d = torch.zeros(T, dtype=torch.float32, device="cuda") if dyntok else None
    qd = lin.pack_npu_input(xd, dyntok_ratios=ratio_d)
    if dyntok:
        q, r = O.pack_dyntok(x, 3.0, p["inv_smooth"])
    else:
        q, r = O.pack_static(x, 0.05, p["inv_smooth"]), None
    acc, yq, y, ya = _oracle_outputs(p, q, r)
    torch.cuda.synchronize()
    assert np.array_equal(qd.cpu().numpy(), q)
    assert np.array_equal(lin.submit(qd, rb.OUT_ACC_I32).cpu().numpy(), acc)
    assert np.array_equal(lin.submit(qd, rb.OUT_QUANT).cpu().numpy().astype(np.int32), yq)
    assert np.array_equal(lin.submit(qd, rb.OUT_F32, dyntok_ratios=ratio_d).cpu().numpy(), y)
    assert np.array_equal(lin.submit(qd, rb.OUT_F32_ACC, dyntok_ratios=ratio_d).cpu().numpy(), ya)
    # fused forward (act quant + contraction + epilogue)
    yf = lin.forward(xd, out_mode=rb.OUT_F32, dyntok=dyntok)
    assert np.array_equal(yf.cpu().numpy(), y)


# CTA-pair plans (clusters of two, cta_group::2 MMAs over 256-channel tiles) forced at small and
# ragged sizes: an odd count of 128-channel blocks (the pair's second half past N), token tiles
# not a multiple of the pair's halves, K tails, several token blocks and several units per pair.
PAIR_SHAPES = [(32, 576, 576), (17, 160, 300), (256, 1024, 384), (300, 1536, 1536),
               (513, 160, 136), (64, 8960, 1536), (96, 2048, 2304)]


@pytest.mark.parametrize("T,K,N", PAIR_SHAPES)
@pytest.mark.parametrize("dyntok", [True, False])
def test_tensor_pair_path_bit_exact(ctx, T, K, N, dyntok):
    p = random_params(K, N, seed=T * 137 + K * 5 + N)
    lin = make_linear(ctx, p)
    lin.set_path(PATH_TENSOR_PAIR)
    x = inputs(T, K, seed=T + 2 * K + N)
    xd = torch.from_numpy(x).cuda()
    ratio_d = torch.zeros(T, dtype=torch.float32, device="cuda") if dyntok else None
    qd = lin.pack_npu_input(xd, dyntok_ratios=ratio_d)
    if dyntok:
        q, r = O.pack_dyntok(x, 3.0, p["inv_smooth"])
    else:
        q, r = O.pack_static(x, 0.05, p["inv_smooth"]), None
    acc, yq, y, ya = _oracle_outputs(p, q, r)
    torch.cuda.synchronize()
    assert np.array_equal(lin.submit(qd, rb.OUT_ACC_I32).cpu().numpy(), acc)
    assert np.array_equal(lin.submit(qd, rb.OUT_QUANT).cpu().numpy().astype(np.int32), yq)
    assert np.array_equal(lin.submit(qd, rb.OUT_F32, dyntok_ratios=ratio_d).cpu().numpy(), y)
    assert np.array_equal(lin.submit(qd, rb.OUT_F32_ACC, dyntok_ratios=ratio_d).cpu().numpy(), ya)
    ctx.check()


@pytest.mark.parametrize("T", [9, 16, 24, 48, 64])
def test_tensor_matches_gemv(ctx, T):
    K, N = 1536, 2304
    p = random_params(K, N, seed=T)
    lin = make_linear(ctx, p)
    xd = synth.activations(T, K, seed=T).cuda()
    outs = {}
    for path in (PATH_GEMV, PATH_TENSOR):
        lin.set_path(path)
        outs[path] = [lin.forward(xd, out_mode=m, dyntok=True).cpu()
                      for m in (rb.OUT_ACC_I32, rb.OUT_QUANT, rb.OUT_F32, rb.OUT_F32_ACC)]
    for a, b in zip(outs[PATH_GEMV], outs[PATH_TENSOR]):
        assert torch.equal(a, b)


def test_tensor_int16_output(ctx):
    T, K, N = 48, 1536, 640
    p = random_params(K, N, seed=5, out_i16=True)
    lin = make_linear(ctx, p, out_i16=True)
    lin.set_path(PATH_TENSOR)
    x = inputs(T, K, seed=9)
    q, r = O.pack_dyntok(x, 3.0, p["inv_smooth"])
    qd = torch.from_numpy(q).cuda()
    acc = O.gemm_i32(q, p["wq"])
    yq = O.requant(acc, p["quant_m"], p["trunc"], 32767)
    out = lin.submit(qd, rb.OUT_QUANT)
    assert out.dtype == torch.int16
    assert np.array_equal(out.cpu().numpy().astype(np.int32), yq)


def test_tensor_split_k_workspace_stays_clean(ctx):
    """Split-K plans leave the workspace zeroed: repeated and interleaved calls agree."""
    T, K, N = 32, 8960, 256      # 2 channel tiles -> many K splits
    p = random_params(K, N, seed=77)
    lin = make_linear(ctx, p)
    lin.set_path(PATH_TENSOR)
    x = inputs(T, K, seed=78)
    q, _ = O.pack_dyntok(x, 3.0, p["inv_smooth"])
    acc = O.gemm_i32(q, p["wq"])
    qd = torch.from_numpy(q).cuda()
    for _ in range(3):
        assert np.array_equal(lin.submit(qd, rb.OUT_ACC_I32).cpu().numpy(), acc)
    # a smaller T in between (different tile count / split plan) and back
    assert np.array_equal(lin.submit(qd[:20], rb.OUT_ACC_I32).cpu().numpy(), acc[:20])
    assert np.array_equal(lin.submit(qd, rb.OUT_ACC_I32).cpu().numpy(), acc)


def test_tensor_strided_and_unaligned_q(ctx):
    T, K, N = 40, 200, 300
    p = random_params(K, N, seed=3)
    lin = make_linear(ctx, p)
    lin.set_path(PATH_TENSOR)
    x = inputs(T, K, seed=4)
    q, _ = O.pack_dyntok(x, 3.0, p["inv_smooth"])
    acc = O.gemm_i32(q, p["wq"])
    # aligned strided view (ld 256) and an unaligned one (ld 203, offset 1) -> copy/pad path
    for ld, off in ((256, 0), (203, 1)):
        buf = torch.zeros(T * ld + 64, dtype=torch.int8, device="cuda")
        view = buf[off:off + T * ld].view(T, ld)[:, :K]
        view.copy_(torch.from_numpy(q).cuda())
        assert np.array_equal(lin.submit(view, rb.OUT_ACC_I32).cpu().numpy(), acc)


PREFILL = [(m, k, n) for m in (128, 512, 2048)
           for (k, n) in ((2048, 2048), (8192, 8192), (2048, 8192), (8192, 2048))]


@pytest.mark.parametrize("M,K,N", PREFILL)
def test_prefill_sweep_sampled_rows(ctx, M, K, N):
    """Full-size prefill GEMMs (SmoothQuant linear, seeded Gaussians with outlier channels):
    every int8 output of 16 sampled tokens equals the oracle's; the whole output equals the
    F32 dequant of the requantised int8 output (an identity that holds for every element)."""
    lp = synth.make_linear(K, N, seed=M + K + N)
    lin = rb.W8A8Linear.from_params(ctx, lp)
    x = synth.activations(M, K, seed=M * 3 + 1)
    xd = x.cuda()
    ratio = torch.zeros(M, dtype=torch.float32, device="cuda")
    yq = lin.forward(xd, out_mode=rb.OUT_QUANT, dyntok=True, ratios_out=ratio).cpu().numpy()
    yf = lin.forward(xd, out_mode=rb.OUT_F32, dyntok=True).cpu().numpy()
    rng = np.random.default_rng(M + N)
    sel = np.sort(rng.choice(M, size=16, replace=False))
    q, r = O.pack_dyntok(x.numpy()[sel], lp.in_thresh, lp.in_inv_smooth)
    acc = O.gemm_i32(q, lp.wq)
    want = O.requant(acc, lp.quant_m, lp.trunc, 127)
    assert np.array_equal(yq[sel].astype(np.int32), want)
    assert np.array_equal(ratio.cpu().numpy()[sel], r)
    full = O.unpack(yq.astype(np.int32), lp.in_step, lp.out_step_chan, ratio.cpu().numpy())
    assert np.array_equal(yf, full)
