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

Every float operation is the builder's, applied in the builder's order (the grouping into
helpers below is this module's own), so on CPU the parameters come out bit-identical to the
reference builder's (pinned by tests/test_oracle_golden.py against fixtures it produced).
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


def _calibration_range(x_smooth: torch.Tensor) -> tuple[float, float, torch.Tensor]:
    """Static input range of the smoothed calibration tokens, each token quantised dyntok-style.

    Returns (in_thresh = the largest per-token max |x|, in_step = in_thresh / 127, the tokens'
    int8 codes as float64)."""
    tok_absmax = x_smooth.abs().amax(dim=-1, keepdim=True).clamp(min=1e-8)
    in_thresh = float(tok_absmax.max().item())
    codes = torch.clamp(torch.round(x_smooth * (127.0 / tok_absmax)), -127.0, 127.0)
    return in_thresh, in_thresh / 127.0, codes.double()


def _row_codes(w_smooth: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """Per-row symmetric int8 codes of the float64 smoothed weights (round-half-even) and the
    row steps max|w| / 127.  Exactly rounded elementwise float64 ops only, so any device gives
    the builder's numpy bytes; rows are independent, so the builder's 512-row slices change
    nothing."""
    row_step = w_smooth.abs().amax(dim=1).clamp(min=1e-12) / 127.0
    codes = torch.clamp(torch.round(w_smooth / row_step.unsqueeze(1)), -127.0, 127.0)
    return codes, row_step


def _output_steps(x_codes: torch.Tensor, w_codes: torch.Tensor, row_step: torch.Tensor,
                  in_step: float, row_norm: torch.Tensor) -> np.ndarray:
    """Per-output-channel output step: 1.15x the channel's largest calibration output, floored
    at 1.15x the 80th percentile of (largest output / weight-row L2 norm) times that norm,
    over 127."""
    peak_out = F.linear(x_codes, w_codes).abs().amax(dim=0) * (in_step * row_step)
    ratio_q80 = torch.quantile(peak_out / row_norm, 0.80)
    bound = torch.maximum(peak_out * 1.15, ratio_q80 * row_norm * 1.15)
    return (bound / 127.0).cpu().numpy()


def _quantm(in_step: float, row_step: torch.Tensor, out_step: np.ndarray,
            trunc: int) -> tuple[torch.Tensor, torch.Tensor]:
    """QuantM[n] = clip(RNE(in_step * w_step[n] / out_step[n] * 2^trunc), 1, 32767) and the
    fp32 out_step_chan[n] = in_step * w_step[n] * 2^trunc / QuantM[n] the requantised int8
    outputs are unpacked with."""
    target = torch.as_tensor(out_step, dtype=torch.float64, device=row_step.device)
    two_t = float(1 << trunc)
    qm = torch.clamp(torch.round((in_step * row_step / target) * two_t), 1.0, 32767.0)
    return qm, ((in_step * row_step * two_t) / qm).to(torch.float32)


def build_linear(w: np.ndarray | torch.Tensor, calib_x: torch.Tensor, trunc: int = TRUNC_CONV,
                 stat: str = "rms", clamp: tuple[float, float] | None = (0.05, 20.0)
                 ) -> LinearParams:
    """SmoothQuant + per-row int8 + per-output-channel QuantM for one linear.

    w: float [N, K] (output channel rows); calib_x: [M, K] calibration activations.
    """
    w32 = torch.as_tensor(np.asarray(w) if not isinstance(w, torch.Tensor) else w).float()
    x = calib_x.float()
    col_scale = smooth_scales(x, w32, stat=stat, clamp=clamp)
    in_thresh, in_step, x_codes = _calibration_range(x / col_scale)
    w_smooth = (w32 * col_scale.unsqueeze(0)).double()
    w_codes, row_step = _row_codes(w_smooth)
    out_step = _output_steps(x_codes, w_codes, row_step, in_step,
                             w_smooth.norm(dim=1).clamp(min=1e-8))
    qm, out_step_chan = _quantm(in_step, row_step, out_step, trunc)
    return LinearParams(wq=w_codes.to(torch.int8).cpu().numpy(), w_step=row_step.cpu().numpy(),
                        in_inv_smooth=(1.0 / col_scale).float().cpu().numpy(),
                        quant_m=qm.to(torch.int16).cpu().numpy(),
                        out_step_chan=out_step_chan.cpu().numpy(), in_thresh=in_thresh,
                        in_step=in_step, trunc=trunc)


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
