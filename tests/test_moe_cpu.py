"""MoE routing and combine on the CPU oracle, pinned to the reference: the restated router
equals MoERouter::route compiled from the reference sources (when the tree is present) and the
committed fixture generated from it (always); the combine follows lfm2_moe.cpp:2300-2318."""
from __future__ import annotations

from pathlib import Path

import numpy as np
import pytest

from oracle import oracle as O

GOLDEN = Path(__file__).resolve().parent / "golden" / "moe_route.npz"


def test_router_matches_reference_fixture():
    g = np.load(GOLDEN)
    k = int(g["k"])
    for kw, key in (({}, "raw"), ({"norm_topk": True, "scaling": 2.5}, "norm"),
                    ({"bias": g["bias"]}, "bias")):
        idx, w = O.moe_route(g["hidden"], g["gate_w"], k, **kw)
        assert np.array_equal(idx, g[f"idx_{key}"])
        assert np.array_equal(w, g[f"w_{key}"])


@pytest.mark.skipif(not O.ref_available(), reason="reference C++ not built here")
@pytest.mark.parametrize("seed,E,k,norm", [(1, 64, 6, False), (2, 16, 2, True), (3, 160, 8, False)])
def test_router_matches_reference_cpp(seed, E, k, norm):
    rng = np.random.default_rng(seed)
    h = rng.standard_normal((7, 256)).astype(np.float32)
    gw = (rng.standard_normal((E, 256)) * 0.05).astype(np.float32)
    gw[E - 1] = gw[0]  # an exact tie between two experts: the lower index comes first
    a = O.moe_route(h, gw, k, norm_topk=norm)
    b = O.ref_moe_route(h, gw, k, norm_topk=norm)
    assert np.array_equal(a[0], b[0]) and np.array_equal(a[1], b[1])


def test_combine_order_and_shared_slots():
    T, k, S, H, E = 2, 2, 1, 3, 4
    yq = np.arange(T * (k + S) * H, dtype=np.int32).reshape(T * (k + S), H) - 5
    idx = np.array([[3, 1], [0, 2]], np.int32)
    w = np.array([[0.5, 0.25], [0.125, 1.0]], np.float32)
    osc = (np.arange((E + S) * H, dtype=np.float32).reshape(E + S, H) + 1) * 0.01
    out = O.moe_combine(yq, idx, w, osc, n_routed=E, slots=k + S)
    want = np.zeros((T, H), np.float32)
    for t in range(T):
        for j in range(k + S):
            e = idx[t, j] if j < k else E + (j - k)
            wj = w[t, j] if j < k else np.float32(1.0)
            want[t] = want[t] + yq[t * (k + S) + j].astype(np.float32) * (wj * osc[e])
    assert np.array_equal(out, want)
