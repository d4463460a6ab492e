"""Package ingest (romanaccio_b200/package.py): the reference's NVDLA weight tiling undone
(fixture tiled by the reference builder's own tile_int8_slice / tile_int16_slice), a weight
region read slice by slice, and quant_scales.json + quant_chan_scales.bin parsed with the
engine's defaults and validity rule."""
from __future__ import annotations

import json
from pathlib import Path

import numpy as np
import pytest

from romanaccio_b200 import DTYPE_FP16, DTYPE_INT8, DTYPE_INT16
from romanaccio_b200.package import (load_quant_scales, read_weight_region, untile_int8,
                                     untile_int16)

G = np.load(Path(__file__).resolve().parent / "golden" / "nvdla_tiles.npz")


@pytest.mark.parametrize("tag", ["a", "b", "c"])
def test_untile_int8_matches_reference_tiling(tag):
    q = G[f"i8_{tag}_q"]
    got = untile_int8(G[f"i8_{tag}_tiled"].tobytes(), *q.shape)
    assert np.array_equal(got, q)


@pytest.mark.parametrize("tag", ["a", "b"])
def test_untile_int16_matches_reference_tiling(tag):
    q = G[f"i16_{tag}_q"]
    got = untile_int16(G[f"i16_{tag}_tiled"].tobytes(), *q.shape)
    assert np.array_equal(got, q)


def test_region_slices():
    """A 528-channel region: a 512-row slice and a 16-row slice, each with its QuantM vector, at
    scattered offsets (the template decides them)."""
    # slice 0: the reference-tiled 512 x 96 slice a; slice 1: 16 rows of the 24 x 96 slice c,
    # tiled with the reference's axis order
    t_a = G["i8_a_tiled"].tobytes()
    q_c = G["i8_c_q"][:16]
    rng = np.random.default_rng(0)
    qm = rng.integers(1, 32767, size=528).astype(np.int16)
    c16 = q_c.reshape(2, 8, 1, 3, 8, 4).transpose(0, 2, 3, 4, 1, 5).tobytes()
    offs = [64, 64 + len(t_a) + 96, 64 + len(t_a) + 96 + 1024 + 32, 200000]
    region = bytearray(offs[3] + 16 * 2 + 64)
    region[offs[0]:offs[0] + len(t_a)] = t_a
    region[offs[1]:offs[1] + 1024] = qm[:512].tobytes()
    region[offs[2]:offs[2] + len(c16)] = c16
    region[offs[3]:offs[3] + 32] = qm[512:].tobytes()
    w, q = read_weight_region(bytes(region), offs, 528, 96)
    assert np.array_equal(w[:512], G["i8_a_q"]) and np.array_equal(w[512:], q_c)
    assert np.array_equal(q, qm)


def test_quant_scales(tmp_path):
    side = np.arange(40, dtype=np.float32) * 0.5
    side.tofile(tmp_path / "quant_chan_scales.bin")
    subs = {
        "lfm3_l00_conv_in": {"input_dtype": "int8", "output_dtype": "int8",
                             "input_threshold": 3.25, "input_step": 3.25 / 127,
                             "output_threshold": 9.0, "output_step": 9.0 / 127,
                             "in_smooth_offset": 0, "in_smooth_count": 8,
                             "out_step_offset": 8, "out_step_count": 12},
        "lfm3_l00_mlp": {"input_dtype": "int8", "output_dtype": "int16",
                         "input_threshold": 2.0, "input_step": 2.0 / 127,
                         "in_smooth_offset": 20, "in_smooth_count": 8,
                         "out_step_offset": 28, "out_step_count": 12},
        "plain": {"input_dtype": "fp16", "input_threshold": 5.0},
        "rejected": {"input_dtype": "int8", "input_threshold": 1.0},
        "out_of_range": {"input_threshold": 1.0, "in_smooth_offset": 39, "in_smooth_count": 8,
                         "out_step_offset": 0, "out_step_count": 1},
    }
    (tmp_path / "quant_scales.json").write_text(json.dumps({"subgraphs": subs}))
    got = load_quant_scales(tmp_path)
    assert set(got) == {"lfm3_l00_conv_in", "lfm3_l00_mlp", "plain"}
    a = got["lfm3_l00_conv_in"]
    assert (a.in_dtype, a.out_dtype) == (DTYPE_INT8, DTYPE_INT8)
    assert a.in_thresh == np.float32(3.25) and a.out_step == np.float32(9.0 / 127)
    assert np.array_equal(a.in_inv_smooth, side[:8]) and np.array_equal(a.out_step_chan, side[8:20])
    m = got["lfm3_l00_mlp"]
    assert m.out_dtype == DTYPE_INT16 and m.out_thresh == 1.0 and np.array_equal(m.out_step_chan,
                                                                                 side[28:40])
    p = got["plain"]
    assert p.in_dtype == DTYPE_FP16 and p.in_inv_smooth is None and p.in_step == np.float32(1 / 127)
