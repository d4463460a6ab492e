"""Offline W8A8 parameter synthesis: SmoothQuant scales, per-row int8 weights, QuantM.

Host-side tooling (not on the GPU path) that produces what a W8A8 linear consumes, following
romanaccio's package builder step by step:

  quantize_rows_int8     tile_int8_slice           src/LFM3/build_lfm3_int8_pkg.py:95-108
                         (float64, round-half-even, per-row step; the NVDLA tiling is replaced
                         by a row-major [N, K] layout)
  smooth_scales          build_single_conv_region  src/LFM3/build_lfm3_int8_pkg.py:190-195
  build_linear           build_single_conv_region  src/LFM3/build_lfm3_int8_pkg.py:171-224
                         (QuantM = clip(round(in_s*w_step/out_s_c*2^trunc), 1, 32767),
                         out_step_chan = in_s*w_step*2^trunc/QuantM)
  TRUNCS                 src/LFM3/build_lfm3_int8_pkg.py:49-54

The same torch operations are used in the same order as the reference builder, so on CPU the
parameters come out bit-identical (pinned by tests/test_quantize_golden.py).
"""
from __future__ import annotations

from dataclasses import dataclass

import numpy as np
import torch
import torch.nn.functional as F

# Right shifts of the SDP CvtPrecision op per subgraph family (build_lfm3_int8_pkg.py:49-54).
TRUNC_CONV = 22
TRUNC_PROJ = 22
TRUNC_QKV = 23


def quantize_rows_int8(w: np.ndarray, max_ws: float | None = None) -> tuple[np.ndarray, np.ndarray]:
    """Per-output-row symmetric int8 quantisation in float64 with round-half-even.

    Returns (wq int8 [N, K], w_step float64 [N]).
    """
    w64 = np.asarray(w).astype(np.float64)
    amax = np.maximum(np.max(np.abs(w64), axis=1, keepdims=True), 1e-12)
    step = amax / 127.0
    if max_ws is not None:
        step = np.minimum(step, max_ws)
    wq = np.clip(np.round(w64 / step), -127, 127).astype(np.int8)
    return wq, step[:, 0]


def smooth_scales(x: torch.Tensor, w: torch.Tensor, stat: str = "rms",
                  clamp: tuple[float, float] | None = (0.05, 20.0)) -> torch.Tensor:
    """SmoothQuant input scales s_in[c] = sqrt(s_x[c] / s_w[c]).

    stat "rms": s_x = rms over calibration tokens of x[:, c] (the reference builder);
    stat "max": s_x = max |x[:, c]| (the SmolLM-shaped workload's definition).
    s_w = max_r |W[r, c]|.  clamp=None leaves s_in unclamped.
    """
    xf = x.float()
    wf = w.float()
    if stat == "rms":
        s_x = xf.pow(2).mean(dim=0).sqrt().clamp(min=1e-5)
    elif stat == "max":
        s_x = xf.abs().amax(dim=0).clamp(min=1e-5)
    else:
        raise ValueError(f"unknown smoothing statistic {stat!r}")
    s_w = wf.abs().amax(dim=0).clamp(min=1e-5)
    s_in = (s_x / s_w).sqrt()
    if clamp is not None:
        s_in = s_in.clamp(min=clamp[0], max=clamp[1])
    return s_in


@dataclass
class LinearParams:
    """Everything one W8A8 linear needs (one quant_scales.json entry + its weight region)."""

    wq: np.ndarray             # int8 [N, K]
    w_step: np.ndarray         # float64 [N]
    in_inv_smooth: np.ndarray  # float32 [K]
    quant_m: np.ndarray        # int16 [N]
    out_step_chan: np.ndarray  # float32 [N]
    in_thresh: float           # input_threshold
    in_step: float             # input_step = in_thresh / 127
    trunc: int

    @property
    def acc_step(self) -> np.ndarray:
        """fp32 step of the raw accumulator: in_step * w_step[n] (logit mode)."""
        return (self.in_step * self.w_step).astype(np.float32)


def build_linear(w: np.ndarray | torch.Tensor, calib_x: torch.Tensor, trunc: int = TRUNC_CONV,
                 stat: str = "rms", clamp: tuple[float, float] | None = (0.05, 20.0),
                 slice_rows: int = 512) -> LinearParams:
    """SmoothQuant + per-row int8 + per-output-channel QuantM for one linear.

    w: float [N, K] (output channel rows); calib_x: [M, K] calibration activations.
    """
    w0 = torch.as_tensor(np.asarray(w) if not isinstance(w, torch.Tensor) else w).float()
    x = calib_x.float()
    s_in = smooth_scales(x, w0, stat=stat, clamp=clamp)
    in_inv_smooth = (1.0 / s_in).float()

    # Static input range measured on the smoothed calibration tokens (dyntok-quantised per token).
    x_sc = x / s_in
    amax_tok = x_sc.abs().amax(dim=-1, keepdim=True).clamp(min=1e-8)
    in_t = float(amax_tok.max().item())
    in_s = in_t / 127.0
    x_q = torch.clamp(torch.round(x_sc * (127.0 / amax_tok)), -127.0, 127.0).double()

    # Smoothed weights, per-row step, and the per-channel output bound with an L2-norm floor.
    w_sc = (w0 * s_in.unsqueeze(0)).double()
    ws = w_sc.abs().amax(dim=1).clamp(min=1e-12) / 127.0
    wq_t = torch.clamp(torch.round(w_sc / ws.unsqueeze(1)), -127.0, 127.0)
    u_c = w_sc.norm(dim=1).clamp(min=1e-8)
    y_norm_max = (F.linear(x_q, wq_t).abs().amax(dim=0)) * (in_s * ws)
    qf = torch.quantile(y_norm_max / u_c, 0.80)
    y_bound_c = torch.maximum(y_norm_max * 1.15, qf * u_c * 1.15)
    out_s_c = (y_bound_c / 127.0).cpu().numpy()

    # Per-row int8 quantisation + QuantM.  Every operation below is an exactly rounded float64
    # elementwise op (abs, max, /, *, round-half-even), so torch on any device reproduces the
    # reference's numpy slice loop bit for bit; rows are independent, so slicing by 512 rows
    # does not change any value.
    del slice_rows
    amax = torch.clamp(w_sc.abs().amax(dim=1, keepdim=True), min=1e-12)
    step = amax / 127.0
    wq_t = torch.clamp(torch.round(w_sc / step), -127, 127).to(torch.int8)
    w_step = step[:, 0]
    out_s = torch.as_tensor(out_s_c, dtype=torch.float64, device=w_step.device)
    qm_f = torch.clamp(torch.round((in_s * w_step / out_s) * float(1 << trunc)), 1.0, 32767.0)
    out_step_chan = ((in_s * w_step * float(1 << trunc)) / qm_f).to(torch.float32)
    return LinearParams(wq=wq_t.cpu().numpy(), w_step=w_step.cpu().numpy(),
                        in_inv_smooth=in_inv_smooth.cpu().numpy(),
                        quant_m=qm_f.to(torch.int16).cpu().numpy(),
                        out_step_chan=out_step_chan.cpu().numpy(), in_thresh=in_t,
                        in_step=in_s, trunc=trunc)


def split_columns(p: LinearParams, n: int) -> list[LinearParams]:
    """Column-split tensor parallelism of one linear over n shards (lfm3_v2.cpp:1920-1975,
    build_lfm3_tp2_pkg.py:80-160): shard s keeps the contiguous output channels
    [s*N/n, (s+1)*N/n) with their weight rows, QuantM and out_step_chan (the per-die
    out_step_chan offset of lfm3_v2.cpp:3852-3860) and shares the input side (in_inv_smooth,
    in_thresh, in_step, trunc).  Every output channel's arithmetic is unchanged, so the shards'
    outputs concatenated along N equal the unsplit linear's outputs bit for bit."""
    N = p.wq.shape[0]
    if not 1 <= n <= N:
        raise ValueError(f"cannot split {N} output channels into {n} shards")
    out = []
    for s in range(n):
        lo, hi = (s * N) // n, ((s + 1) * N) // n
        out.append(LinearParams(wq=np.ascontiguousarray(p.wq[lo:hi]), w_step=p.w_step[lo:hi].copy(),
                                in_inv_smooth=p.in_inv_smooth, quant_m=p.quant_m[lo:hi].copy(),
                                out_step_chan=p.out_step_chan[lo:hi].copy(),
                                in_thresh=p.in_thresh, in_step=p.in_step, trunc=p.trunc))
    return out
