"""The GPU norm + quantisation steps (w8a8_rmsnorm_pack_dyntok, w8a8_post_op_ffn_pack) against
the C restatement pinned to the reference: bit-identical int8 rows, ratios, normalised rows and
residual rows, for several token counts and row widths (including tails and the widest row)."""
from __future__ import annotations

import numpy as np
import pytest
import torch

from pathlib import Path

from oracle import oracle as O
import romanaccio_b200 as rb
from romanaccio_b200 import synth
from romanaccio_b200.norm import post_op_ffn_pack, rmsnorm_pack_dyntok

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("T,C", [(1, 1536), (1, 576), (3, 1537), (8, 2048), (2, 8960),
                                 (1, 12288), (5, 3)])
def test_rmsnorm_pack_matches_oracle(ctx, T, C):
    rng = np.random.default_rng(T * 100 + C)
    h = (rng.standard_normal((T, C)) * rng.uniform(0.1, 30)).astype(np.float32)
    h[0, : min(C, 4)] *= 50  # an outlier channel
    norm = (rng.standard_normal(C) * 0.4 + 1).astype(np.float32)
    smooth = (rng.random(C) * 3 + 0.02).astype(np.float32)
    q, ratio, u = rmsnorm_pack_dyntok(ctx, torch.from_numpy(h).cuda(),
                                      torch.from_numpy(smooth).cuda(), 6.0,
                                      norm=torch.from_numpy(norm).cuda())
    wq, wr, wu = O.rmsnorm_pack_dyntok(h, norm, smooth, 6.0)
    assert np.array_equal(q.cpu().numpy(), wq)
    assert np.array_equal(ratio.cpu().numpy(), wr)
    assert np.array_equal(u.cpu().numpy(), wu)
    # without the normalised-row output
    q2, r2, u2 = rmsnorm_pack_dyntok(ctx, torch.from_numpy(h).cuda(),
                                     torch.from_numpy(smooth).cuda(), 6.0)
    assert u2 is None and np.array_equal(q2.cpu().numpy(), wq)
    ctx.check()


@pytest.mark.parametrize("T,C", [(1, 1536), (4, 2049), (2, 8960)])
def test_post_op_ffn_pack_matches_oracle(ctx, T, C):
    rng = np.random.default_rng(C + T)
    op = (rng.standard_normal((T, C)) * 6).astype(np.float32)
    post = (rng.standard_normal(C) * 0.3 + 1).astype(np.float32)
    h = (rng.standard_normal((T, C)) * 3).astype(np.float32)
    ffn = (rng.random(C) * 30).astype(np.float32)
    m, q = post_op_ffn_pack(ctx, *(torch.from_numpy(a).cuda() for a in (op, post, h, ffn)))
    wm, wq = O.post_op_ffn_pack(op, post, h, ffn)
    assert np.array_equal(m.cpu().numpy(), wm)
    assert np.array_equal(q.cpu().numpy(), wq)
    ctx.check()


EMB_GOLDEN = Path(__file__).resolve().parent / "golden" / "emb_norm_pack.npz"


@pytest.mark.parametrize("tag", ["c1536", "c2048", "c3840", "c578"])
def test_emb_norm_pack_matches_reference_fixture(ctx, tag):
    """The LM head's input step on the GPU, against rows the reference produced."""
    g = np.load(EMB_GOLDEN)
    h = torch.from_numpy(np.ascontiguousarray(g[f"{tag}_h"][None])).cuda()
    emb = torch.from_numpy(g[f"{tag}_emb"]).cuda()
    q = rb.emb_norm_pack(ctx, h, emb, float(g["eps"]))
    assert np.array_equal(q.cpu().numpy()[0], g[f"{tag}_q"])


@pytest.mark.parametrize("n", [1, 4])
def test_lm_heads_with_fused_input_norm(ctx, n):
    """The input RMSNorm fused into the LM heads' quantisation step: the merged top-k equals
    the oracle's LM head over the oracle's normalised, packed input."""
    V, K, T, k = 49152, 1536, 3, 40
    rng = np.random.default_rng(n)
    wq = rng.integers(-127, 128, size=(V, K)).astype(np.int8)
    in_step = 0.031
    acc = ((rng.random(V) * 0.02 / 127 + 1e-5) * in_step).astype(np.float32)
    emb = rb.emb_norm_scaled((rng.standard_normal(K) * 0.3 + 1).astype(np.float32), in_step)
    emb_d = torch.from_numpy(emb).cuda()
    h = (synth.activations(T, K, seed=n).numpy() * 3).astype(np.float32)
    q = O.emb_norm_pack(h, emb)
    wv, wi = O.topk(O.dequant_acc(O.gemm_i32(q, wq), acc), k)
    multi = rb.MultiDeviceLmHead([ctx] * n, wq, acc, in_step, max_tokens=8, k_max=64)
    multi.set_input_norm(emb_d)
    v, i, a = multi.forward(torch.from_numpy(h).cuda(), k)
    assert np.array_equal(i.cpu().numpy(), wi) and np.array_equal(v.cpu().numpy(), wv)
    rank = rb.RankLmHead(ctx, 0, 1, wq, acc, in_step, V, max_tokens=8, k_max=64)
    rank.connect([rank.export()])
    rank.set_input_norm(emb_d)
    v, i, a = rank.forward(torch.from_numpy(h).cuda(), k)
    assert np.array_equal(i.cpu().numpy(), wi) and np.array_equal(v.cpu().numpy(), wv)
    assert np.array_equal(a.cpu().numpy(), wi[:, 0])
    ctx.check()
