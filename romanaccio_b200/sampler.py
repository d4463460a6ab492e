"""Token sampler over the merged LM-head candidates (w8a8_sampler_*, host only).

The reference samples with Sampler::sample over the full logit vector (sampler.cpp:83-179).
Here the GPU LM head leaves the k largest (logit, vocab id) pairs and the sampler applies the
reference's steps to them; for the same seed it returns the reference's token whenever the
candidates decide it, and raises W8A8Error(ERR_NOT_SUPPORTED) otherwise (no random number is
drawn then), so the caller can pass more candidates.
"""
from __future__ import annotations

import ctypes as C
from dataclasses import dataclass

import numpy as np

from ._lib import ERR_NOT_SUPPORTED, SamplerParams, W8A8Error, check, load


@dataclass
class SamplingConfig:
    """SamplerParams with the reference's defaults (sampler.hpp:10-19)."""
    temperature: float = 0.7
    top_k: int = 40
    top_p: float = 0.9
    min_p: float = 0.05
    repeat_penalty: float = 1.15
    repeat_window: int = 64
    max_consecutive_duplicates: int = 2
    seed: int = 0

    def as_dict(self) -> dict:
        return dict(self.__dict__)


class CandidateSampler:
    """Sampler::sample / accept / reset over candidate lists (w8a8_sampler_*)."""

    def __init__(self, cfg: SamplingConfig | None = None):
        self._lib = load()
        c = cfg or SamplingConfig()
        p = SamplerParams(c.temperature, c.top_k, c.top_p, c.min_p, c.repeat_penalty,
                          c.repeat_window, c.max_consecutive_duplicates, c.seed)
        h = C.c_void_p()
        check(self._lib.w8a8_sampler_create(C.byref(p), C.byref(h)), "w8a8_sampler_create")
        self.handle = h

    def accept(self, token: int) -> None:
        check(self._lib.w8a8_sampler_accept(self.handle, int(token)), "w8a8_sampler_accept")

    def reset(self) -> None:
        check(self._lib.w8a8_sampler_reset(self.handle), "w8a8_sampler_reset")

    def sample(self, values, ids, vocab: int) -> int:
        """values / ids: the n largest raw logits and their vocab ids, (value desc, id asc)."""
        v = np.ascontiguousarray(np.asarray(values, dtype=np.float32).reshape(-1))
        i = np.ascontiguousarray(np.asarray(ids, dtype=np.int32).reshape(-1))
        if v.shape != i.shape:
            raise ValueError("values and ids differ in length")
        out = C.c_int32()
        check(self._lib.w8a8_sampler_sample(self.handle, v.ctypes.data, i.ctypes.data, v.shape[0],
                                            int(vocab), C.byref(out)), "w8a8_sampler_sample")
        return int(out.value)

    def try_sample(self, values, ids, vocab: int) -> int | None:
        """As sample(), but None when the candidates do not decide the token."""
        try:
            return self.sample(values, ids, vocab)
        except W8A8Error as e:
            if e.status == ERR_NOT_SUPPORTED:
                return None
            raise

    def close(self) -> None:
        if getattr(self, "handle", None):
            self._lib.w8a8_sampler_destroy(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


__all__ = ["CandidateSampler", "SamplingConfig"]
