"""Parity of the fused LM-head shard (GEMV + on-chip top-k) and the cross-shard merge with the
CPU oracle: identical token ids and values (bit-exact: the logits are a deterministic function
of int32 accumulators), including int8-saturated logits where ties are decided by the lowest
vocab id, as Sampler::sample's greedy rule does."""
from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import oracle as O
import romanaccio_b200 as rb
from romanaccio_b200 import synth

pytestmark = pytest.mark.gpu


def lm_params(V: int, K: int, seed: int):
    rng = np.random.default_rng(seed)
    wq = rng.integers(-127, 128, size=(V, K)).astype(np.int8)
    w_step = (rng.random(V) * 0.02 / 127 + 1e-5).astype(np.float64)
    return wq, w_step


def oracle_logits(x, wq, in_step, acc_step):
    q = O.pack_static(x, in_step, None)
    return O.dequant_acc(O.gemm_i32(q, wq), acc_step)


@pytest.mark.parametrize("V,K,T,k", [
    (49152, 576, 1, 40), (24576, 576, 1, 1), (18992, 1536, 1, 40), (151936, 1536, 1, 40),
    (151936, 1536, 3, 64), (12800, 2048, 8, 40), (32768, 3840, 2, 17), (1000, 64, 5, 64),
    (40, 32, 1, 40), (200, 100, 11, 7),
    # 16+ tokens: tensor-core GEMM into the logits, per-CTA row lists, per-token selection
    (151936, 1536, 16, 40), (49152, 576, 64, 64), (12800, 2048, 20, 1), (4097, 128, 33, 33),
    (1000, 64, 17, 64), (200, 100, 40, 7),
])
def test_shard_topk_matches_oracle(ctx, V, K, T, k):
    wq, w_step = lm_params(V, K, seed=V + K)
    in_step = 0.031
    acc_step = (in_step * w_step).astype(np.float32)
    x = synth.activations(T, K, seed=T).numpy()
    off = 1000
    shard = rb.LmHeadShard(ctx, wq, acc_step, in_step, row_offset=off)
    logits_d = torch.empty((T, V), dtype=torch.float32, device="cuda")
    val, idx = shard.forward(torch.from_numpy(x).cuda(), k, logits=logits_d)
    lg = oracle_logits(x, wq, in_step, acc_step)
    wv, wi = O.topk(lg, k, id_offset=off)
    assert np.array_equal(logits_d.cpu().numpy(), lg)
    assert np.array_equal(idx.cpu().numpy(), wi)
    assert np.array_equal(val.cpu().numpy(), wv)
    for t in range(T):
        assert idx[t, 0].item() == O.argmax(lg[t]) + off


@pytest.mark.parametrize("T,k", [(1, 64), (3, 40), (16, 64), (24, 32)])
def test_top_keys_concentrated_in_one_cta(ctx, T, k):
    """The whole top-k inside one CTA's rows, with exact ties: one per-CTA list holds every
    winner, so the final selection walks that list far past its head (and breaks the ties by
    the lowest vocab id)."""
    V, K = 151936, 1536
    wq, w_step = lm_params(V, K, seed=77)
    in_step = 0.031
    x = synth.activations(T, K, seed=78).numpy()
    q = O.pack_static(x, in_step, None)
    # rows 5000..5099: 127 * sign(q[0]) -> the largest accumulators for token 0; pairs of equal rows
    hot = np.arange(5000, 5100)
    sign = np.where(q[0] >= 0, 127, -127).astype(np.int8)
    wq[hot] = sign
    wq[hot[1::2], :8] = 0  # every other row slightly smaller; duplicates below tie exactly
    w_step[hot] = 1e-3
    acc_step = (in_step * w_step).astype(np.float32)
    shard = rb.LmHeadShard(ctx, wq, acc_step, in_step, row_offset=0)
    val, idx = shard.forward(torch.from_numpy(x).cuda(), k)
    lg = oracle_logits(x, wq, in_step, acc_step)
    wv, wi = O.topk(lg, k)
    assert np.isin(wi[0], hot).all()
    assert np.array_equal(idx.cpu().numpy(), wi)
    assert np.array_equal(val.cpu().numpy(), wv)


@pytest.mark.parametrize("T", [2, 16])
def test_saturated_int8_logits_tie_rule(ctx, T):
    """LFM3's INT8 LM head requantises logits to int8 (static out_step), so the largest logits
    saturate at +127 and tie; the lowest vocab id must win (FINDINGS.md:2476-2498 case)."""
    V, K, k = 64000, 512, 40
    rng = np.random.default_rng(0)
    wq = rng.integers(-127, 128, size=(V, K)).astype(np.int8)
    qm = np.full(V, 32767, np.int16)
    scale = rb.SubgraphScaleInfo(in_dtype=rb.DTYPE_INT8, out_dtype=rb.DTYPE_INT8, in_step=0.02,
                                 out_step=0.21785)
    lin = rb.W8A8Linear(ctx, wq, scale, quant_m=qm, trunc=22)
    x = synth.activations(T, K, seed=5).numpy()
    q = O.pack_static(x, 0.02, None)
    yq = O.requant(O.gemm_i32(q, wq), qm, 22, 127)
    assert (yq == 127).sum(axis=1).min() > k  # many ties at the top
    lg = O.unpack(yq, 0.21785, None, None)
    wv, wi = O.topk(lg, k, id_offset=16000)
    val, idx = lin.forward_topk(torch.from_numpy(x).cuda(), k, row_offset=16000, out_mode=rb.OUT_F32)
    assert np.array_equal(idx.cpu().numpy(), wi)
    assert np.array_equal(val.cpu().numpy(), wv)
    for t in range(T):
        assert idx[t, 0].item() == 16000 + O.ref_greedy(lg[t]) if O.ref_available() else True


@pytest.mark.parametrize("n_shards", [2, 4, 8])
def test_sharded_merge_equals_unsharded(ctx, n_shards):
    """Contiguous vocab shards (one GPU here, one per rank in deployment) + merge == full top-k."""
    V, K, T, k = 151936, 1536, 2, 40
    wq, w_step = lm_params(V, K, seed=9)
    in_step = 0.027
    acc_step = (in_step * w_step).astype(np.float32)
    x = synth.activations(T, K, seed=11).numpy()
    xd = torch.from_numpy(x).cuda()
    vals, ids = [], []
    for r in range(n_shards):
        lo, hi = rb.shard_range(V, n_shards, r)
        sh = rb.LmHeadShard(ctx, wq[lo:hi], acc_step[lo:hi], in_step, row_offset=lo)
        v, i = sh.forward(xd, k)
        vals.append(v)
        ids.append(i)
    gv = torch.stack(vals, dim=1)  # [T, n, k]
    gi = torch.stack(ids, dim=1)
    mv, mi, am = rb.topk_merge(ctx, gv, gi, k)
    lg = oracle_logits(x, wq, in_step, acc_step)
    wv, wi = O.topk(lg, k)
    assert np.array_equal(mi.cpu().numpy(), wi)
    assert np.array_equal(mv.cpu().numpy(), wv)
    assert np.array_equal(am.cpu().numpy(), wi[:, 0])
    # rank-major layout straight out of an all-gather ([n, T, k] permuted to [T, n, k])
    gv2 = torch.stack(vals, dim=0).permute(1, 0, 2)
    gi2 = torch.stack(ids, dim=0).permute(1, 0, 2)
    mv2, mi2, _ = rb.topk_merge(ctx, gv2, gi2, k)
    assert torch.equal(mi2, mi) and torch.equal(mv2, mv)


def test_repeated_topk_calls_reset_scratch(ctx):
    V, K = 30000, 256
    wq, w_step = lm_params(V, K, seed=1)
    acc_step = (0.03 * w_step).astype(np.float32)
    shard = rb.LmHeadShard(ctx, wq, acc_step, 0.03, row_offset=0)
    x = torch.from_numpy(synth.activations(1, K, seed=2).numpy()).cuda()
    v0, i0 = shard.forward(x, 40)
    for _ in range(30):
        v, i = shard.forward(x, 40)
        assert torch.equal(i, i0) and torch.equal(v, v0)
    ctx.check()


@pytest.mark.parametrize("T,k", [(16, 40), (32, 64)])
def test_tensor_topk_equals_gemv_topk(ctx, T, k):
    """16+ tokens: the tensor-core top-k (one GEMM into the logits, then row lists) and the GEMV
    top-k forced on the same linear select the same (value, id) pairs, in the same order."""
    V, K = 60000, 1024
    wq, w_step = lm_params(V, K, seed=T)
    acc_step = (0.029 * w_step).astype(np.float32)
    shard = rb.LmHeadShard(ctx, wq, acc_step, 0.029, row_offset=7)
    x = torch.from_numpy(synth.activations(T, K, seed=3).numpy()).cuda()
    v_tc, i_tc = shard.forward(x, k)
    shard.linear.set_path(rb.PATH_GEMV)
    v_gv, i_gv = shard.forward(x, k)
    assert torch.equal(i_tc, i_gv) and torch.equal(v_tc, v_gv)
    ctx.check()


def test_tensor_topk_equal_logits(ctx):
    """Every logit equal (zero weights): the order is by vocab id alone, so each CTA's threshold
    keeps exactly its lowest ids and the selection returns ids row_offset .. row_offset + k - 1."""
    V, K, T, k = 20000, 256, 16, 64
    wq = np.zeros((V, K), np.int8)
    acc_step = np.full(V, 1e-3, np.float32)
    shard = rb.LmHeadShard(ctx, wq, acc_step, 0.03, row_offset=100)
    x = torch.from_numpy(synth.activations(T, K, seed=4).numpy()).cuda()
    v, i = shard.forward(x, k)
    want = np.broadcast_to(np.arange(100, 100 + k, dtype=np.int32), (T, k))
    assert np.array_equal(i.cpu().numpy(), want)
    assert (v.cpu().numpy() == 0).all()
