"""Seeded synthetic workloads with the shapes of the decode / prefill configurations.

The reference measures on no public dataset; these generators stand in for its models:
weights ~ N(0, 0.02) quantised per output row, activations ~ N(0, 1) with a fixed 1 % of
channels scaled x20 (outliers), SmoothQuant + QuantM from a 64-token calibration batch drawn
from the same distribution.
"""
from __future__ import annotations

from dataclasses import dataclass

import numpy as np
import torch

from .quantize import TRUNC_CONV, TRUNC_QKV, LinearParams, build_linear


@dataclass(frozen=True)
class DecodeShape:
    name: str
    hidden: int
    layers: int
    q: int
    kv: int
    o_in: int
    ffn: int
    vocab: int

    def subgraphs(self) -> list[tuple[str, int, int, int]]:
        """Per layer: (name, K, N, trunc).  q|k|v and gate|up are fused subgraphs sharing one
        input smoothing, like the reference's attn_qkv subgraph."""
        return [
            ("qkv", self.hidden, self.q + 2 * self.kv, TRUNC_QKV),
            ("o", self.o_in, self.hidden, TRUNC_CONV),
            ("gate_up", self.hidden, 2 * self.ffn, TRUNC_CONV),
            ("down", self.ffn, self.hidden, TRUNC_CONV),
        ]

    def weight_bytes_per_layer(self) -> int:
        return sum(k * n for _, k, n, _ in self.subgraphs())


SMOLLM_135M = DecodeShape("smollm-135m", 576, 30, 576, 192, 576, 1536, 49152)
QWEN25_15B = DecodeShape("qwen2.5-1.5b", 1536, 28, 1536, 256, 1536, 8960, 151936)
GEMMA_12B = DecodeShape("gemma-12b-class", 3840, 48, 4096, 2048, 4096, 15360, 262144)
DEEPSEEK_V2_LITE_LMHEAD = (2048, 102400)
DEEPSEEK_V2_LITE_EXPERT = ((2048, 1408), (2048, 1408), (1408, 2048))  # gate, up, down (K, N)
PREFILL_SWEEP = [(m, k, n) for m in (128, 512, 2048)
                 for (k, n) in ((2048, 2048), (8192, 8192), (2048, 8192), (8192, 2048))]


def outlier_channels(K: int, seed: int = 1234) -> np.ndarray:
    rng = np.random.default_rng(seed)
    return np.sort(rng.choice(K, size=max(1, K // 100), replace=False))


def activations(T: int, K: int, seed: int, device="cpu") -> torch.Tensor:
    """x ~ N(0, 1) with 1 % of channels (a fixed seeded set) scaled x20."""
    g = torch.Generator(device=device).manual_seed(seed)
    x = torch.randn((T, K), generator=g, device=device, dtype=torch.float32)
    x[:, torch.as_tensor(outlier_channels(K), device=device)] *= 20.0
    return x


def weights(N: int, K: int, seed: int, device="cpu") -> torch.Tensor:
    g = torch.Generator(device=device).manual_seed(seed)
    return torch.randn((N, K), generator=g, device=device, dtype=torch.float32) * 0.02


def make_linear(K: int, N: int, seed: int, trunc: int = TRUNC_CONV, stat: str = "rms",
                clamp=(0.05, 20.0), device="cpu") -> LinearParams:
    """Seeded weights + calibration -> W8A8 parameters (see quantize.build_linear)."""
    w = weights(N, K, seed, device)
    calib = activations(64, K, seed + 1, device)
    return build_linear(w, calib, trunc=trunc, stat=stat, clamp=clamp)
