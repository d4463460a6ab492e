"""The candidate sampler (w8a8_sampler_*, host only) against the reference's own Sampler compiled
from its sources (oracle/_ref): the reference samples from the full logit vector, ours from the
64 largest (logit, id) pairs that the GPU LM head leaves.  With the same seed both must draw the
same token sequence, step after step (each sampled token is accepted into the history, so the
repetition penalty and the loop breaker act on later steps)."""
from __future__ import annotations

import numpy as np
import pytest

from oracle import oracle as O
from romanaccio_b200 import W8A8Error
from romanaccio_b200._lib import ERR_NOT_SUPPORTED
from romanaccio_b200.sampler import CandidateSampler, SamplingConfig

needs_ref = pytest.mark.skipif(not O.ref_available(), reason="reference sampler not built here")


def candidates(row: np.ndarray, n: int):
    """The n largest logits in (value desc, id asc) order, as the GPU merge returns them."""
    order = np.lexsort((np.arange(row.shape[0]), -row))[:n]
    return row[order], order.astype(np.int32)


def run_ours(cfg: SamplingConfig, history, logits: np.ndarray, n_cand: int):
    s = CandidateSampler(cfg)
    for t in history:
        s.accept(int(t))
    out = []
    for row in logits:
        v, i = candidates(row, n_cand)
        tok = s.sample(v, i, row.shape[0])
        s.accept(tok)
        out.append(tok)
    return np.array(out, np.int32)


def steps(S: int, V: int, seed: int, scale: float = 3.0) -> np.ndarray:
    return (np.random.default_rng(seed).standard_normal((S, V)) * scale).astype(np.float32)


CONFIGS = [
    SamplingConfig(seed=7),                                          # reference defaults
    SamplingConfig(seed=11, temperature=1.3, top_p=0.97, min_p=0.01),
    SamplingConfig(seed=5, top_p=1.0, min_p=0.0, top_k=32),
    SamplingConfig(seed=3, repeat_penalty=1.6, repeat_window=16),
    SamplingConfig(seed=9, temperature=0.0),                         # greedy with penalties
]


@needs_ref
@pytest.mark.parametrize("cfg", CONFIGS, ids=lambda c: f"t{c.temperature}_k{c.top_k}_s{c.seed}")
def test_candidates_match_reference(cfg):
    V, S = 5000, 40
    logits = steps(S, V, seed=cfg.seed + 100)
    # history with tokens that sit among the top logits of later steps
    history = list(np.argsort(-logits[0])[:12]) + [17, 17]
    want = O.ref_sampler_run(cfg.as_dict(), history, logits)
    got = run_ours(cfg, history, logits, n_cand=64)
    assert np.array_equal(got, want)


@needs_ref
def test_loop_breaking_matches_reference():
    """The same logits every step: greedy decoding repeats a token until the loop breaker blocks
    it, and an ABABAB history blocks B."""
    V, S = 3000, 12
    row = steps(1, V, seed=1)[0]
    logits = np.repeat(row[None, :], S, axis=0)
    top = np.argsort(-row)[:2]
    history = [top[0], top[1]] * 3
    for cfg in (SamplingConfig(seed=4, temperature=0.0, repeat_penalty=1.0),
                SamplingConfig(seed=4, temperature=0.8, repeat_penalty=1.0, top_p=1.0)):
        want = O.ref_sampler_run(cfg.as_dict(), history, logits)
        got = run_ours(cfg, history, logits, n_cand=64)
        assert np.array_equal(got, want)


@needs_ref
def test_complete_candidates_any_top_k():
    """With every token a candidate (small vocabulary) top_k = 0 is decided too."""
    V, S = 100, 25
    logits = steps(S, V, seed=3)
    cfg = SamplingConfig(seed=21, top_k=0, top_p=0.95)
    want = O.ref_sampler_run(cfg.as_dict(), [5, 6, 5], logits)
    got = run_ours(cfg, [5, 6, 5], logits, n_cand=V)
    assert np.array_equal(got, want)


@needs_ref
def test_undecided_draws_nothing():
    """top_k = 0 over a partial list cannot be decided: the call refuses and draws no random
    number, so the next decided call still follows the reference's random stream."""
    V, S = 4000, 6
    logits = steps(S, V, seed=8)
    cfg = SamplingConfig(seed=13)
    want = O.ref_sampler_run(cfg.as_dict(), [], logits)
    s = CandidateSampler(cfg)
    refuse = CandidateSampler(SamplingConfig(seed=13, top_k=0))
    v, i = candidates(logits[0], 64)
    with pytest.raises(W8A8Error) as e:
        refuse.sample(v, i, V)
    assert e.value.status == ERR_NOT_SUPPORTED
    got = []
    for row in logits:
        v, i = candidates(row, 64)
        assert s.try_sample(v[:10], i[:10], V) is None  # 10 candidates cannot hold top_k = 40
        tok = s.sample(v, i, V)
        s.accept(tok)
        got.append(tok)
    assert np.array_equal(np.array(got, np.int32), want)


@pytest.mark.parametrize("name", ["default", "greedy"])
def test_candidates_match_reference_fixture(name):
    """Token sequences the reference drew (tests/golden/sampler_seq.npz), reproduced from the
    64 largest logits of each step."""
    from pathlib import Path
    g = np.load(Path(__file__).resolve().parent / "golden" / "sampler_seq.npz")
    keys = ("temperature", "top_k", "top_p", "min_p", "repeat_penalty", "repeat_window",
            "max_consecutive_duplicates", "seed")
    cfg = SamplingConfig(**{k: g[f"{name}_{k}"].item() for k in keys})
    got = run_ours(cfg, g["history"].tolist(), g["logits"], n_cand=64)
    assert np.array_equal(got, g[f"{name}_tokens"])


def test_greedy_without_reference():
    """Greedy decoding is the lowest id among the largest candidates, and the loop breaker
    blocks a token repeated max_consecutive_duplicates times."""
    s = CandidateSampler(SamplingConfig(temperature=0.0, repeat_penalty=1.0, seed=1))
    v = np.array([5.0, 5.0, 4.0, 1.0], np.float32)
    ids = np.array([10, 12, 3, 7], np.int32)
    assert s.sample(v, ids, 100) == 10
    s.accept(10)
    s.accept(10)
    assert s.sample(v, ids, 100) == 12
