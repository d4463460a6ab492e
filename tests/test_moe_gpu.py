"""Parity of the device MoE layer (router -> W8A8 experts -> combine) with the oracle.

The router's logits are a warp-parallel fp32 sum, so routing is checked as identical expert ids
and weights within float rounding (on the reference's own fixture and on seeded layers); each
expert stage is then checked bit-exactly against the oracle fed with the device's upstream
values, and the combine bit-exactly against lfm2_moe.cpp's accumulation order."""
from __future__ import annotations

from pathlib import Path

import numpy as np
import pytest
import torch

from oracle import oracle as O
from romanaccio_b200 import DTYPE_INT8, DTYPE_INT16, synth
from romanaccio_b200.moe import MoELayer, MoEParams, make_moe_params

pytestmark = pytest.mark.gpu

GOLDEN = Path(__file__).resolve().parent / "golden" / "moe_route.npz"


def test_router_matches_reference_fixture(ctx):
    g = np.load(GOLDEN)
    k = int(g["k"])
    E, H = g["gate_w"].shape
    base = make_moe_params(H, 16, 1, 0, 1, seed=5)
    for kw, key in (({}, "raw"), ({"norm_topk_prob": True, "routed_scaling": 2.5}, "norm"),
                    ({"gate_bias": g["bias"]}, "bias")):
        p = MoEParams(gate_w=g["gate_w"], gate_bias=kw.get("gate_bias"),
                      gu=[base.gu[0]] * E, dn=[base.dn[0]] * E, top_k=k,
                      norm_topk_prob=kw.get("norm_topk_prob", False),
                      routed_scaling=kw.get("routed_scaling", 1.0))
        layer = MoELayer(ctx, p, max_tokens=8)
        idx, w = layer.route(torch.from_numpy(g["hidden"]).cuda())
        assert np.array_equal(idx.cpu().numpy(), g[f"idx_{key}"])
        np.testing.assert_allclose(w.cpu().numpy(), g[f"w_{key}"], rtol=2e-6, atol=0)


def _check_layer(layer: MoELayer, x: np.ndarray, sample_pairs=None):
    p = layer.p
    T = x.shape[0]
    out = layer.forward(torch.from_numpy(x).cuda()).cpu().numpy()
    v = {k: t.cpu().numpy() for k, t in layer.views(T).items()}
    idx, w = O.moe_route(x, p.gate_w, p.top_k, bias=p.gate_bias, norm_topk=p.norm_topk_prob,
                         scaling=p.routed_scaling)
    assert np.array_equal(v["idx"], idx)
    # different fp32 summation order of the logits: weights agree to float rounding (1e-4 rel)
    np.testing.assert_allclose(v["w"], w, rtol=1e-4, atol=0)
    slots, E, I = layer.slots, p.n_routed, p.inter
    pairs = range(T * slots) if sample_pairs is None else sample_pairs
    qmax = 32767 if p.dn_out_dtype == DTYPE_INT16 else 127
    for pi in pairs:
        t, j = divmod(pi, slots)
        e = int(v["idx"][t, j]) if j < p.top_k else E + (j - p.top_k)
        gu, dn = p.gu[e], p.dn[e]
        # gate|up: dyntok pack with the expert's smoothing, int32 GEMM, requant, unpack
        q, r = O.pack_dyntok(x[t:t + 1], gu.in_thresh, gu.in_inv_smooth)
        yq = O.requant(O.gemm_i32(q, gu.wq), gu.quant_m, gu.trunc, 127)
        assert np.array_equal(v["gate_up"][pi:pi + 1], O.unpack(yq, 0.0, gu.out_step_chan, r)), \
            f"gate_up pair {pi}"
        # silu(gate) * up in float (the device uses expf): within a few ulp
        g_, u_ = v["gate_up"][pi, :I], v["gate_up"][pi, I:]
        want_h = (g_ / (np.float32(1) + np.exp(-g_))) * u_
        np.testing.assert_allclose(v["act"][pi], want_h, rtol=2e-6, atol=1e-30)
        # down: static pack of the device activations, GEMM, requant to int8/int16
        q2 = O.pack_static(v["act"][pi:pi + 1], dn.in_step, dn.in_inv_smooth)
        want_dq = O.requant(O.gemm_i32(q2, dn.wq), dn.quant_m, dn.trunc, qmax)
        assert np.array_equal(v["down_q"][pi:pi + 1].astype(np.int32), want_dq), f"down pair {pi}"
    # combine: exact accumulation order over the slots
    osc = np.stack([q.out_step_chan for q in p.dn])
    want = O.moe_combine(v["down_q"].astype(np.int32), v["idx"], v["w"], osc, E, slots)
    assert np.array_equal(out, want)


@pytest.mark.parametrize("dtype", [DTYPE_INT8, DTYPE_INT16])
@pytest.mark.parametrize("T,k,S", [(1, 2, 1), (5, 3, 2), (9, 4, 0)])
def test_small_layer_stages_bit_exact(ctx, dtype, T, k, S):
    p = make_moe_params(H=256, I=160, E=8, S=S, k=k, seed=T * 10 + k, device="cuda",
                        dn_out_dtype=dtype)
    if dtype == DTYPE_INT16:  # int16 stage: a finer QuantM grid
        for q in p.dn:
            q.quant_m = np.clip(q.quant_m.astype(np.int32) * 64, 1, 32767).astype(np.int16)
    layer = MoELayer(ctx, p, max_tokens=16)
    _check_layer(layer, synth.activations(T, 256, seed=T).numpy())


_V2_LITE = {}


@pytest.mark.parametrize("T", [1, 8, 64])
def test_deepseek_v2_lite_shaped_layer(ctx, T):
    """Config-3 shape: hidden 2048, 64 routed + 2 shared experts of 1408, top-6, no renorm."""
    if "layer" not in _V2_LITE:
        p = make_moe_params(H=2048, I=1408, E=64, S=2, k=6, seed=3, device="cuda")
        _V2_LITE["layer"] = MoELayer(ctx, p, max_tokens=64)
    layer = _V2_LITE["layer"]
    x = synth.activations(T, 2048, seed=100 + T).numpy()
    rng = np.random.default_rng(T)
    n_pairs = T * layer.slots
    sample = None if n_pairs <= 64 else sorted(rng.choice(n_pairs, 48, replace=False).tolist())
    _check_layer(layer, x, sample)
    ctx.check()
