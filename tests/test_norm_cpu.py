"""The C restatements of the reference's fused norm + quantisation steps (oracle/w8a8_oracle.c)
pinned to the reference: to the committed fixture the reference produced
(tests/golden/norm_pack.npz) and, where the reference is built here, to it directly on seeded
rows of every width class (multiple of 4, tails of 1..3)."""
from __future__ import annotations

from pathlib import Path

import numpy as np
import pytest

from oracle import oracle as O

GOLDEN = Path(__file__).resolve().parent / "golden" / "norm_pack.npz"


@pytest.mark.parametrize("tag", ["c1536", "c579"])
def test_restatement_matches_reference_fixture(tag):
    g = np.load(GOLDEN)
    q, ratio, u = O.rmsnorm_pack_dyntok(g[f"{tag}_h"][None], g[f"{tag}_norm"], g[f"{tag}_smooth"],
                                        float(g["in_thresh"]))
    assert np.array_equal(q[0], g[f"{tag}_q"])
    assert ratio[0] == g[f"{tag}_ratio"]
    assert np.array_equal(u[0], g[f"{tag}_u"])
    m, q2 = O.post_op_ffn_pack(g[f"{tag}_op"][None], g[f"{tag}_post"], g[f"{tag}_h"][None],
                               g[f"{tag}_ffn"])
    assert np.array_equal(m[0], g[f"{tag}_hmid"])
    assert np.array_equal(q2[0], g[f"{tag}_q2"])


@pytest.mark.skipif(not O.ref_available(), reason="reference not built here")
@pytest.mark.parametrize("C", [576, 1536, 1537, 1538, 1539, 2048, 4096])
def test_restatement_matches_reference(C):
    rng = np.random.default_rng(C)
    for _ in range(4):
        h = (rng.standard_normal(C) * rng.uniform(0.05, 40)).astype(np.float32)
        norm = (rng.standard_normal(C) * 0.5 + 1).astype(np.float32)
        smooth = (rng.random(C) * 3 + 0.01).astype(np.float32)
        thr = float(rng.uniform(0.5, 30))
        q, r, u = O.rmsnorm_pack_dyntok(h[None], norm, smooth, thr)
        rq, rr, ru = O.ref_rmsnorm_pack_dyntok(h, norm, smooth, thr)
        assert np.array_equal(q[0], rq) and r[0] == rr and np.array_equal(u[0], ru)
        op = (rng.standard_normal(C) * 8).astype(np.float32)
        post = (rng.standard_normal(C) * 0.3 + 1).astype(np.float32)
        ffn = (rng.random(C) * 30).astype(np.float32)
        m, q2 = O.post_op_ffn_pack(op[None], post, h[None], ffn)
        rm, rq2 = O.ref_post_op_ffn_pack(op, post, h, ffn)
        assert np.array_equal(m[0], rm) and np.array_equal(q2[0], rq2)


EMB_GOLDEN = Path(__file__).resolve().parent / "golden" / "emb_norm_pack.npz"


@pytest.mark.parametrize("tag", ["c1536", "c2048", "c3840", "c578"])
def test_emb_norm_pack_matches_reference_fixture(tag):
    """The LM head's input step (fused_emb_norm_broadcast_t1) against rows the reference
    produced."""
    g = np.load(EMB_GOLDEN)
    q = O.emb_norm_pack(g[f"{tag}_h"][None], g[f"{tag}_emb"], float(g["eps"]))
    assert np.array_equal(q[0], g[f"{tag}_q"])


@pytest.mark.skipif(not O.ref_available(), reason="reference C++ not built here")
@pytest.mark.parametrize("C", [1536, 3840, 577, 64])
def test_emb_norm_pack_matches_reference_cpp(C):
    rng = np.random.default_rng(C + 5)
    for _ in range(4):
        h = (rng.standard_normal(C) * rng.uniform(0.05, 40)).astype(np.float32)
        emb = ((rng.standard_normal(C) * 0.4 + 1) * rng.uniform(5, 60)).astype(np.float32)
        assert np.array_equal(O.emb_norm_pack(h[None], emb)[0], O.ref_emb_norm_pack(h, emb))
