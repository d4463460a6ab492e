"""Column-split tensor parallelism of a linear (lfm3_v2.cpp:1920-1975, build_lfm3_tp2_pkg.py:
80-160) checked on the oracle: the output-channel shards, run on the same input and
concatenated, reproduce the unsplit linear bit for bit (int32 accumulators, requantised int8,
dequantised fp32, dyntok ratios)."""
from __future__ import annotations

import numpy as np
import pytest

from oracle import oracle as O
from romanaccio_b200 import synth
from romanaccio_b200.quantize import split_columns


@pytest.mark.parametrize("n", [1, 2, 3, 8])
def test_split_columns_matches_unsplit_linear(n):
    K, N, T = 192, 136, 3
    p = synth.make_linear(K, N, seed=n)
    x = synth.activations(T, K, seed=10 + n).numpy()
    full = O.linear(x, p.wq, p.quant_m, p.trunc, p.out_step_chan, p.in_inv_smooth, p.in_thresh)
    parts = [O.linear(x, s.wq, s.quant_m, s.trunc, s.out_step_chan, s.in_inv_smooth, s.in_thresh)
             for s in split_columns(p, n)]
    for j in (2, 3, 4):  # acc, yq, y
        assert np.array_equal(np.concatenate([pt[j] for pt in parts], axis=1), full[j])
    for pt in parts:
        assert np.array_equal(pt[0], full[0]) and np.array_equal(pt[1], full[1])


def test_split_columns_rejects_more_shards_than_channels():
    p = synth.make_linear(32, 4, seed=0)
    with pytest.raises(ValueError):
        split_columns(p, 5)
