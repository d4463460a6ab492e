"""The reference's fused norm + quantisation steps around each linear and in front of the LM
head, on the GPU (w8a8_rmsnorm_pack_dyntok, w8a8_post_op_ffn_pack, w8a8_emb_norm_pack;
lfm3_v2.cpp:652-831), bit-identical to it."""
from __future__ import annotations

import numpy as np
import torch

from ._lib import check
from .linear import Context, _stream


def _f32(t: torch.Tensor, C: int) -> None:
    if t.dtype != torch.float32 or not t.is_cuda or t.stride(-1) != 1 or t.shape[-1] < C:
        raise ValueError("expected a CUDA float32 tensor with unit stride along C")


def rmsnorm_pack_dyntok(ctx: Context, h: torch.Tensor, smooth: torch.Tensor, in_thresh: float,
                        eps: float = 1e-5, norm: torch.Tensor | None = None, stream=None):
    """fused_rms_norm_pack_dyntok_t1 per row of h [T, C]: (q int8 [T, C], ratio [T], u_out or None)."""
    T, C = h.shape
    _f32(h, C)
    _f32(smooth, C)
    q = torch.empty((T, C), dtype=torch.int8, device=h.device)
    ratio = torch.empty((T,), dtype=torch.float32, device=h.device)
    u = torch.empty((T, C), dtype=torch.float32, device=h.device) if norm is not None else None
    check(ctx._lib.w8a8_rmsnorm_pack_dyntok(
        ctx.handle, h.data_ptr(), h.stride(0), T, C, norm.data_ptr() if norm is not None else None,
        smooth.data_ptr(), float(in_thresh), float(eps), q.data_ptr(), C, ratio.data_ptr(),
        u.data_ptr() if u is not None else None, C, _stream(stream)), "w8a8_rmsnorm_pack_dyntok")
    return q, ratio, u


def post_op_ffn_pack(ctx: Context, op_out: torch.Tensor, post_norm: torch.Tensor, h: torch.Tensor,
                     ffn_scaled: torch.Tensor, eps: float = 1e-5, stream=None):
    """fused_post_op_residual_ffn_pack_mlp_t1 per row: (h_mid [T, C], q int8 [T, C])."""
    T, C = op_out.shape
    for t in (op_out, post_norm, h, ffn_scaled):
        _f32(t, C)
    h_mid = torch.empty((T, C), dtype=torch.float32, device=op_out.device)
    q = torch.empty((T, C), dtype=torch.int8, device=op_out.device)
    check(ctx._lib.w8a8_post_op_ffn_pack(
        ctx.handle, op_out.data_ptr(), op_out.stride(0), post_norm.data_ptr(), h.data_ptr(),
        h.stride(0), T, C, ffn_scaled.data_ptr(), float(eps), h_mid.data_ptr(), C, q.data_ptr(), C,
        _stream(stream)), "w8a8_post_op_ffn_pack")
    return h_mid, q


def emb_norm_scaled(weight: np.ndarray, in_step: float) -> np.ndarray:
    """The LM head's input-norm table as the reference loader builds it (lfm3_v2.cpp:3906-3912):
    weight[c] * (1 / in_step), in fp32."""
    inv_step = np.float32(1.0) / np.float32(in_step)
    return (np.asarray(weight, np.float32) * inv_step).astype(np.float32)


def emb_norm_pack(ctx: Context, h: torch.Tensor, emb_norm_scaled_t: torch.Tensor,
                  eps: float = 1e-5, stream=None) -> torch.Tensor:
    """fused_emb_norm_broadcast_t1 per row of h [T, C]: the LM head's static int8 input q [T, C]
    = round_clamp(h * inv_rms * emb_norm_scaled, 127)."""
    T, C = h.shape
    _f32(h, C)
    _f32(emb_norm_scaled_t, C)
    q = torch.empty((T, C), dtype=torch.int8, device=h.device)
    ldh = h.stride(0) if T > 1 else C  # (a single row may carry any leading stride)
    check(ctx._lib.w8a8_emb_norm_pack(ctx.handle, h.data_ptr(), ldh, T, C,
                                      emb_norm_scaled_t.data_ptr(), float(eps), q.data_ptr(), C,
                                      _stream(stream)), "w8a8_emb_norm_pack")
    return q

