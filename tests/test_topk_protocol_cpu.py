"""The grid top-k protocol of csrc/topk.cuh restated on the host and checked against a full sort:
every CTA keeps its sorted top-k list and its head; the last CTA takes T0 = the k-th largest
head, gathers the entries >= T0 of the k lists headed by the k largest heads, and their top-k is
the grid's.  Checked on random keys, on winners concentrated in one list, on many empty lists,
on fewer rows than k, and for the gather bound k * k that sizes the kernel's shared buffer."""
from __future__ import annotations

import numpy as np
import pytest


def protocol(keys_per_cta: list[np.ndarray], k: int):
    lists = [np.sort(c)[::-1][:k] for c in keys_per_cta]
    heads = np.array([l[0] if len(l) else 0 for l in lists], dtype=np.uint64)
    order = np.argsort(-heads.astype(np.float64), kind="stable")[:k]
    t0 = heads[order[-1]] if len(order) == k else np.uint64(0)
    gathered = []
    for g in order:
        if heads[g] == 0:
            continue
        gathered.extend(int(x) for x in lists[g] if x >= t0)
    return sorted(gathered, reverse=True)[:k], len(gathered)


def unique_keys(rng, n: int) -> np.ndarray:
    """n distinct keys in [1, 2^40) in random order (the kernel's keys are distinct: the vocab id
    is part of each)."""
    k = np.unique(rng.integers(1, 1 << 40, size=2 * n + 16, dtype=np.int64))[:n]
    assert k.size == n
    return rng.permutation(k).astype(np.uint64)


@pytest.mark.parametrize("G,rows,k", [(296, 513, 40), (238, 80, 40), (288, 528, 64), (7, 16, 64),
                                      (50, 3, 40), (1, 100, 64), (300, 1, 1)])
def test_random_keys(G, rows, k):
    rng = np.random.default_rng(G * rows + k)
    keys = unique_keys(rng, G * rows)
    per = [keys[g * rows:(g + 1) * rows] for g in range(G)]
    got, n = protocol(per, k)
    want = sorted((int(x) for x in keys), reverse=True)[:k]
    assert got == want
    assert n <= k * k


def test_winners_in_one_list_and_empty_lists():
    rng = np.random.default_rng(3)
    k, G, rows = 64, 200, 500
    keys = unique_keys(rng, G * rows)
    # CTA 17 holds every one of the largest keys; every third CTA owns no rows
    top = np.sort(keys)[::-1][:rows]
    rest = np.setdiff1d(keys, top)
    per = [rest[g * (rows - 2):(g + 1) * (rows - 2)] for g in range(G)]
    per[17] = top
    for g in range(0, G, 3):
        if g != 17:
            per[g] = np.array([], dtype=np.uint64)
    got, n = protocol(per, k)
    all_keys = np.concatenate(per)
    assert got == sorted((int(x) for x in all_keys), reverse=True)[:k]
    assert n <= k * k
