"""The int16 w2 stage of the reference's SwiGLU MLP subgraph (int16 input silu(gate) * up, int16
weight codes, QuantM with trunc 28): the oracle's restatement is pinned to the reference's own
engine model (tests/golden/mlp_w2_int16.npz, recorded from attribute_int8_error.sim_mlp_npu as it
ran), and the GPU linear16 must give the same int16 outputs, plus the unpack, on that fixture,
on a package-scale shape and at the int16 extremes."""
from __future__ import annotations

from pathlib import Path

import numpy as np
import pytest
import torch

from oracle import oracle as O
import romanaccio_b200 as rb

G = np.load(Path(__file__).resolve().parent / "golden" / "mlp_w2_int16.npz")


@pytest.mark.parametrize("tag", ["a", "b"])
def test_oracle_matches_reference_engine_model(tag):
    y = O.gemm_i16_requant(G[f"{tag}_x"], G[f"{tag}_w"], G[f"{tag}_qm"], int(G["trunc"]))
    assert np.array_equal(y, G[f"{tag}_yq"])
    # and the reference's float output: out_q * out_step in float64, then fp32
    assert np.array_equal((y.astype(np.float64) * float(G[f"{tag}_out_s"])).astype(np.float32),
                          G[f"{tag}_y"])


def _cases():
    rng = np.random.default_rng(5)
    yield "fixture_a", G["a_x"], G["a_w"], G["a_qm"], 28
    yield "fixture_b", G["b_x"], G["b_w"], G["b_qm"], 28
    # an LFM3-scale w2 (2048 out x 8192 in), 3 tokens; trunc 25..28 as the builder uses
    for trunc in (25, 28):
        x = rng.integers(-32767, 32768, size=(3, 8192)).astype(np.int16)
        w = rng.integers(-32767, 32768, size=(2048, 8192)).astype(np.int16)
        qm = rng.integers(1, 32768, size=2048).astype(np.int16)
        yield f"lfm3_t{trunc}", x, w, qm, trunc
    # extremes: every product at +-32767^2 (saturation both ways), K not a multiple of 8
    x = np.full((2, 1001), 32767, np.int16)
    x[1] = -32767
    w = np.full((16, 1001), 32767, np.int16)
    yield "extremes", x, w, np.full(16, 32767, np.int16), 28


@pytest.mark.gpu
@pytest.mark.parametrize("case", list(range(5)))
def test_linear16_matches_oracle(ctx, case):
    name, x, w, qm, trunc = list(_cases())[case]
    osc = (np.random.default_rng(case).random(w.shape[0]) * 1e-3 + 1e-6).astype(np.float32)
    lin = rb.Linear16(ctx, w, qm, trunc=trunc, out_step_chan=osc, max_tokens=8)
    xd = torch.from_numpy(np.ascontiguousarray(x)).cuda()
    yq = lin.forward(xd, rb.OUT_QUANT).cpu().numpy()
    want = O.gemm_i16_requant(x, w, qm, trunc)
    assert np.array_equal(yq, want), name
    y = lin.forward(xd, rb.OUT_F32).cpu().numpy()
    assert np.array_equal(y, want.astype(np.float32) * osc[None, :]), name
    ctx.check()
