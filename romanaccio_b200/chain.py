"""Persistent decode chain (w8a8_chain_*): a fixed sequence of W8A8 linears, optionally ending
with the LM-head top-k, executed by one cooperative kernel launch per forward.

It stands in for the reference's per-token loop of pack -> submit_task -> unpack calls
(src/LFM3/lfm3_v2.cpp:1743-1990, src/eswin_runtime/src/llm/transformer_session.cpp:650-844).
Buffers are bound at construction, like a recorded graph; the tensors and linears passed in
must stay alive (this object keeps references to them).
"""
from __future__ import annotations

import ctypes as C
from dataclasses import dataclass

import torch

from . import _lib
from ._lib import ACT_DYNTOK, OUT_F32, check
from .linear import Context, W8A8Linear, _stream


@dataclass
class ChainStepSpec:
    linear: W8A8Linear
    x: torch.Tensor                     # fp32 [T, K] view (unit column stride)
    y: torch.Tensor | None = None       # [T, N] output per out_mode (None for the top-k step)
    act_mode: int = ACT_DYNTOK
    out_mode: int = OUT_F32
    ratio: torch.Tensor | None = None   # optional [T] fp32 dyntok ratios
    topk_k: int = 0
    row_offset: int = 0
    topk_val: torch.Tensor | None = None
    topk_idx: torch.Tensor | None = None
    # RMSNorm folded into the STATIC pack (the LM head's input step): norm weight / in_step [K]
    emb_norm: torch.Tensor | None = None
    norm_eps: float = 1e-5


class DecodeChain:
    def __init__(self, ctx: Context, steps: list[ChainStepSpec], T: int):
        self._lib = ctx._lib
        self.ctx = ctx
        self.T = int(T)
        self._keep = list(steps)
        arr = (_lib.ChainStep * len(steps))()
        for i, s in enumerate(steps):
            if s.x.dim() != 2 or s.x.stride(1) != 1 or s.x.shape[1] != s.linear.K:
                raise ValueError(f"step {i}: x must be a [T, K] row-major view")
            if s.x.shape[0] != self.T:
                raise ValueError(f"step {i}: x has {s.x.shape[0]} rows, chain T={self.T}")
            arr[i].linear = s.linear.handle
            arr[i].x_dev = s.x.data_ptr()
            arr[i].ldx = s.x.stride(0)
            arr[i].act_mode = int(s.act_mode)
            arr[i].out_mode = int(s.out_mode)
            if s.y is not None:
                if s.y.stride(1) != 1 or s.y.shape[1] != s.linear.N:
                    raise ValueError(f"step {i}: y must be a [T, N] row-major view")
                arr[i].y_dev = s.y.data_ptr()
                arr[i].ldy = s.y.stride(0)
            arr[i].ratio_dev = s.ratio.data_ptr() if s.ratio is not None else None
            arr[i].topk_k = int(s.topk_k)
            arr[i].row_offset = int(s.row_offset)
            arr[i].topk_val_dev = s.topk_val.data_ptr() if s.topk_val is not None else None
            arr[i].topk_idx_dev = s.topk_idx.data_ptr() if s.topk_idx is not None else None
            if s.emb_norm is not None:
                if (s.emb_norm.dtype != torch.float32 or not s.emb_norm.is_contiguous()
                        or s.emb_norm.numel() != s.linear.K):
                    raise ValueError(f"step {i}: emb_norm must be a contiguous fp32 [K] tensor")
                arr[i].emb_norm_dev = s.emb_norm.data_ptr()
            arr[i].norm_eps = float(s.norm_eps)
        h = C.c_void_p()
        check(self._lib.w8a8_chain_create(ctx.handle, arr, len(steps), self.T, C.byref(h)),
              "w8a8_chain_create")
        self.handle = h

    @property
    def barriers(self) -> int:
        return int(self._lib.w8a8_chain_barriers(self.handle))

    @property
    def grid(self) -> int:
        return int(self._lib.w8a8_chain_grid(self.handle))

    def enable_trace(self) -> torch.Tensor:
        """Allocates and attaches the per-step timer buffer [grid, n_steps, 8] (int64 ns)."""
        buf = torch.zeros((self.grid, len(self._keep), 8), dtype=torch.int64,
                          device=self._keep[0].x.device)
        check(self._lib.w8a8_chain_set_trace(self.handle, buf.data_ptr()), "w8a8_chain_set_trace")
        self._trace = buf
        return buf

    def forward(self, stream=None) -> None:
        check(self._lib.w8a8_chain_forward(self.handle, _stream(stream)), "w8a8_chain_forward")

    def close(self) -> None:
        if getattr(self, "handle", None):
            self._lib.w8a8_chain_destroy(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
