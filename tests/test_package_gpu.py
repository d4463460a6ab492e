"""A package built by the reference's own builder (tests/golden/pkg_mini: weight regions from
build_single_conv_region, quant_scales.json / quant_chan_scales.bin in the reference's package
format) ingested through romanaccio_b200.package into W8A8 linears, run on the GPU, must match
the oracle fed with the builder's own values: int8 outputs and fp32 unpacked outputs bit for bit,
dyntok and static input modes."""
from __future__ import annotations

import json
from pathlib import Path

import numpy as np
import pytest
import torch

from oracle import oracle as O
import romanaccio_b200 as rb
from romanaccio_b200.package import load_quant_scales, read_weight_region

PKG = Path(__file__).resolve().parent / "golden" / "pkg_mini"
NAMES = ["mini_l00_conv_in", "mini_l00_attn_qkv"]


def _ingest(name):
    scales = load_quant_scales(PKG)
    wmap = json.loads((PKG / "weights_map.json").read_text())[name]
    tmpl = json.loads((PKG / "region_offsets.json").read_text())[name]
    blob = (PKG / f"die{wmap['die']}.bin").read_bytes()
    region = blob[wmap["weight_offset"]:wmap["weight_offset"] + wmap["weight_size"]]
    wq, qm = read_weight_region(region, tmpl["offsets"], tmpl["N"], tmpl["K"])
    return scales[name], wq, qm, tmpl["trunc"]


@pytest.mark.parametrize("name", NAMES)
def test_ingest_equals_builder_values(name):
    """(CPU) the reader recovers exactly what the reference builder produced."""
    e = np.load(PKG / "expected.npz")
    sc, wq, qm, _ = _ingest(name)
    assert np.array_equal(wq, e[f"{name}_wq"]) and np.array_equal(qm, e[f"{name}_qm"])
    assert np.array_equal(sc.in_inv_smooth, e[f"{name}_inv"])
    assert np.array_equal(sc.out_step_chan, e[f"{name}_osc"])
    assert sc.in_thresh == np.float32(e[f"{name}_in_t"])


@pytest.mark.gpu
@pytest.mark.parametrize("name", NAMES)
def test_ingested_package_linear_matches_oracle(ctx, name):
    e = np.load(PKG / "expected.npz")
    sc, wq, qm, trunc = _ingest(name)
    lin = rb.W8A8Linear(ctx, wq, sc, quant_m=qm, trunc=trunc)
    x = e[f"{name}_x"].astype(np.float32)
    xd = torch.from_numpy(x).cuda()
    inv, osc = e[f"{name}_inv"], e[f"{name}_osc"]
    # dyntok input (the engine's mode for these subgraphs), fp32 unpacked and int8 outputs
    y = lin.forward(xd, rb.OUT_F32, dyntok=True).cpu().numpy()
    yq = lin.forward(xd, rb.OUT_QUANT, dyntok=True).cpu().numpy()
    _, _, _, want_q, want_y = O.linear(x, e[f"{name}_wq"], e[f"{name}_qm"], trunc, osc, inv,
                                       in_thresh=float(np.float32(e[f"{name}_in_t"])))
    assert np.array_equal(yq.astype(np.int32), want_q)
    assert np.array_equal(y, want_y)
    # static input with the package's input_step
    ys = lin.forward(xd, rb.OUT_F32, dyntok=False).cpu().numpy()
    _, _, _, _, want_s = O.linear(x, e[f"{name}_wq"], e[f"{name}_qm"], trunc, osc, inv,
                                  in_step=float(sc.in_step))
    assert np.array_equal(ys, want_s)
    ctx.check()
