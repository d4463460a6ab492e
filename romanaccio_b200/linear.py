"""Host-side mirror of romanaccio's quantised-linear boundary over the C ABI (libw8a8.so).

The reference drives each INT8 linear through three calls (src/LFM3/lfm3_v2.cpp):

    pack_npu_input(src_tc, act_buf, T, C, scale_info, dyntok_ratios)      :1186-1204
    m_pool.submit_task(die, model_id, {act, weights}, {out}, &driver_ns)    :1941-1960
    unpack_npu_output(out_buf, dst_tc, T, C_out, scale_info, dyntok_ratios) :1207-1225

`W8A8Linear` keeps those names and argument meanings (`dyntok_ratios` given => per-token
dynamic scaling, else the static `in_step`) on device tensors, and adds the fused `forward`
that runs all three as one pipelined launch sequence.  Device buffers are torch CUDA tensors
(plumbing only); every computation runs in the CUDA kernels of libw8a8.so.
"""
from __future__ import annotations

import ctypes as C
from dataclasses import dataclass, field

import numpy as np
import torch

from . import _lib
from ._lib import (ACT_DYNTOK, ACT_STATIC, DTYPE_FP16, DTYPE_INT8, DTYPE_INT16, OUT_ACC_I32,
                   OUT_F32, OUT_F32_ACC, OUT_QUANT, check)


def _ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


def _stream(stream: torch.cuda.Stream | None) -> int:
    s = stream if stream is not None else torch.cuda.current_stream()
    return s.cuda_stream


class Context:
    """One per CUDA device (w8a8_ctx)."""

    def __init__(self, device: int = 0):
        self._lib = _lib.load()
        h = C.c_void_p()
        check(self._lib.w8a8_ctx_create(int(device), C.byref(h)), "w8a8_ctx_create")
        self.handle = h
        self.device = int(device)

    @property
    def sm_count(self) -> int:
        return int(self._lib.w8a8_ctx_sm_count(self.handle))

    def check(self) -> None:
        """Synchronises and raises if a kernel recorded a bounded-wait timeout."""
        check(self._lib.w8a8_ctx_check(self.handle), "w8a8_ctx_check")

    def close(self) -> None:
        if self.handle:
            self._lib.w8a8_ctx_destroy(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


@dataclass
class SubgraphScaleInfo:
    """Mirrors SubgraphScaleInfo (src/LFM3/lfm3_v2.cpp:556-565)."""

    in_dtype: int = DTYPE_FP16
    out_dtype: int = DTYPE_FP16
    in_thresh: float = 1.0
    in_step: float = 1.0 / 127.0
    out_thresh: float = 1.0
    out_step: float = 1.0 / 127.0
    in_inv_smooth: np.ndarray | None = field(default=None, repr=False)
    out_step_chan: np.ndarray | None = field(default=None, repr=False)


class W8A8Linear:
    """One INT8 subgraph: int8 weights [N, K] + QuantM [N] + trunc + scale info."""

    def __init__(self, ctx: Context, weights: np.ndarray, scale: SubgraphScaleInfo,
                 quant_m: np.ndarray | None = None, trunc: int = 22,
                 acc_step: np.ndarray | None = None):
        self._lib = ctx._lib
        self.ctx = ctx
        w = np.ascontiguousarray(weights, dtype=np.int8)
        if w.ndim != 2:
            raise ValueError("weights must be [N, K]")
        self.N, self.K = map(int, w.shape)
        self.scale = scale
        self.out_i16 = scale.out_dtype == DTYPE_INT16
        keep = [w]
        inv = None
        if scale.in_inv_smooth is not None:
            inv = np.ascontiguousarray(scale.in_inv_smooth, dtype=np.float32)
            assert inv.shape == (self.K,)
            keep.append(inv)
        osc = None
        if scale.out_step_chan is not None:
            osc = np.ascontiguousarray(scale.out_step_chan, dtype=np.float32)
            assert osc.shape == (self.N,)
            keep.append(osc)
        qm = None
        if quant_m is not None:
            qm = np.ascontiguousarray(quant_m, dtype=np.int16)
            assert qm.shape == (self.N,)
            keep.append(qm)
        ast = None
        if acc_step is not None:
            ast = np.ascontiguousarray(acc_step, dtype=np.float32)
            assert ast.shape == (self.N,)
            keep.append(ast)
        si = _lib.ScaleInfo(
            out_dtype=int(scale.out_dtype if scale.out_dtype != DTYPE_FP16 else DTYPE_INT8),
            in_thresh=float(scale.in_thresh), in_step=float(scale.in_step),
            out_thresh=float(scale.out_thresh), out_step=float(scale.out_step),
            in_inv_smooth=inv.ctypes.data if inv is not None else None,
            out_step_chan=osc.ctypes.data if osc is not None else None)
        desc = _lib.LinearDesc(
            K=self.K, N=self.N, weights=w.ctypes.data, weights_ld=self.K,
            quant_m=qm.ctypes.data if qm is not None else None, trunc=int(trunc),
            acc_step=ast.ctypes.data if ast is not None else None, scale=si)
        h = C.c_void_p()
        check(self._lib.w8a8_linear_create(ctx.handle, C.byref(desc), C.byref(h)),
              "w8a8_linear_create")
        del keep
        self.handle = h
        self.trunc = int(trunc)

    @property
    def device_bytes(self) -> int:
        return int(self._lib.w8a8_linear_device_bytes(self.handle))

    @classmethod
    def from_params(cls, ctx: Context, p) -> "W8A8Linear":
        """From quantize.LinearParams (one quant_scales.json entry + its int8 weights)."""
        scale = SubgraphScaleInfo(in_dtype=DTYPE_INT8, out_dtype=DTYPE_INT8,
                                  in_thresh=p.in_thresh, in_step=p.in_step,
                                  in_inv_smooth=p.in_inv_smooth, out_step_chan=p.out_step_chan)
        return cls(ctx, p.wq, scale, quant_m=p.quant_m, trunc=p.trunc, acc_step=p.acc_step)

    def enable_trace(self, sm_count: int, device) -> torch.Tensor:
        """Per-CTA timeline [2 * sm_count, 8] (int64 %globaltimer ns) of every launch (tensor-core
        launches fill the first sm_count rows)."""
        buf = torch.zeros((2 * sm_count, 8), dtype=torch.int64, device=device)
        check(self._lib.w8a8_linear_set_trace(self.handle, buf.data_ptr()), "w8a8_linear_set_trace")
        self._trace = buf
        return buf

    def set_path(self, path: int) -> None:
        """Contraction engine: PATH_AUTO, PATH_GEMV (weight streaming) or PATH_TENSOR (tcgen05)."""
        check(self._lib.w8a8_linear_set_path(self.handle, int(path)), "w8a8_linear_set_path")

    def reserve(self, max_tokens: int, max_k: int = 0, stream=None) -> None:
        """Allocates up front the scratch that forwards of up to max_tokens tokens (top-k
        forwards with k <= max_k) on the current path would grow on first use, so that those
        forwards allocate nothing and can be captured in a CUDA graph."""
        check(self._lib.w8a8_linear_reserve(self.handle, int(max_tokens), int(max_k),
                                            _stream(stream)), "w8a8_linear_reserve")

    def close(self) -> None:
        if getattr(self, "handle", None):
            self._lib.w8a8_linear_destroy(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    # ---------------------------------------------------------------- boundary stages
    def pack_npu_input(self, x: torch.Tensor, dyntok_ratios: torch.Tensor | None = None,
                       out: torch.Tensor | None = None, stream=None) -> torch.Tensor:
        """fp32 [T, K] -> int8 [T, K]; dyntok when `dyntok_ratios` ([T] fp32) is given."""
        _check_dev(x, torch.float32, self.K)
        T = x.shape[0]
        q = out if out is not None else torch.empty((T, self.K), dtype=torch.int8, device=x.device)
        mode = ACT_DYNTOK if dyntok_ratios is not None else ACT_STATIC
        check(self._lib.w8a8_pack_input(self.handle, x.data_ptr(), x.stride(0), T, mode,
                                        q.data_ptr(), q.stride(0), _ptr(dyntok_ratios),
                                        _stream(stream)), "w8a8_pack_input")
        return q

    def submit(self, q: torch.Tensor, out_mode: int = OUT_QUANT,
               dyntok_ratios: torch.Tensor | None = None, out: torch.Tensor | None = None,
               stream=None) -> torch.Tensor:
        """The NPU step: int8 [T, K] -> int32 acc / int8|int16 requant / fp32 per out_mode."""
        _check_dev(q, torch.int8, self.K)
        T = q.shape[0]
        y = out if out is not None else torch.empty((T, self.N), dtype=self._out_dtype(out_mode),
                                                   device=q.device)
        mode = ACT_DYNTOK if dyntok_ratios is not None else ACT_STATIC
        check(self._lib.w8a8_linear_forward_q(self.handle, q.data_ptr(), q.stride(0), T, mode,
                                              _ptr(dyntok_ratios), int(out_mode), y.data_ptr(),
                                              y.stride(0), _stream(stream)),
              "w8a8_linear_forward_q")
        return y

    def unpack_npu_output(self, yq: torch.Tensor, dyntok_ratios: torch.Tensor | None = None,
                          out: torch.Tensor | None = None, stream=None) -> torch.Tensor:
        """int8/int16 [T, N] -> fp32 [T, N] with out_step_chan (x ratio in dyntok mode)."""
        T = yq.shape[0]
        y = out if out is not None else torch.empty((T, self.N), dtype=torch.float32, device=yq.device)
        mode = ACT_DYNTOK if dyntok_ratios is not None else ACT_STATIC
        check(self._lib.w8a8_unpack_output(self.handle, yq.data_ptr(), yq.stride(0), T, mode,
                                           _ptr(dyntok_ratios), y.data_ptr(), y.stride(0),
                                           _stream(stream)), "w8a8_unpack_output")
        return y

    # ---------------------------------------------------------------- fused forward
    def forward(self, x: torch.Tensor, out_mode: int = OUT_F32, dyntok: bool = True,
                out: torch.Tensor | None = None, ratios_out: torch.Tensor | None = None,
                stream=None) -> torch.Tensor:
        _check_dev(x, torch.float32, self.K)
        T = x.shape[0]
        y = out if out is not None else torch.empty((T, self.N), dtype=self._out_dtype(out_mode),
                                                   device=x.device)
        check(self._lib.w8a8_linear_forward(self.handle, x.data_ptr(), x.stride(0), T,
                                            ACT_DYNTOK if dyntok else ACT_STATIC, int(out_mode),
                                            y.data_ptr(), y.stride(0), _ptr(ratios_out),
                                            _stream(stream)), "w8a8_linear_forward")
        return y

    def forward_topk(self, x: torch.Tensor, k: int, row_offset: int = 0, out_mode: int = OUT_F32_ACC,
                     dyntok: bool = False, val: torch.Tensor | None = None,
                     idx: torch.Tensor | None = None, logits: torch.Tensor | None = None,
                     stream=None) -> tuple[torch.Tensor, torch.Tensor]:
        """Shard logits never leave the SM: returns the sorted top-k (value, vocab id) per token."""
        _check_dev(x, torch.float32, self.K)
        T = x.shape[0]
        v = val if val is not None else torch.empty((T, k), dtype=torch.float32, device=x.device)
        i = idx if idx is not None else torch.empty((T, k), dtype=torch.int32, device=x.device)
        check(self._lib.w8a8_linear_forward_topk(
            self.handle, x.data_ptr(), x.stride(0), T, ACT_DYNTOK if dyntok else ACT_STATIC,
            int(out_mode), int(k), int(row_offset), v.data_ptr(), i.data_ptr(), _ptr(logits),
            logits.stride(0) if logits is not None else 0, _stream(stream)),
            "w8a8_linear_forward_topk")
        return v, i

    def _out_dtype(self, out_mode: int) -> torch.dtype:
        if out_mode == OUT_ACC_I32:
            return torch.int32
        if out_mode == OUT_QUANT:
            return torch.int16 if self.out_i16 else torch.int8
        return torch.float32


def topk_merge(ctx: Context, vals: torch.Tensor, idxs: torch.Tensor, k_out: int,
               stream=None) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    """Merges candidate lists into the global top-k_out + argmax.

    vals/idxs: [T, n_lists, k_in] views (any token / list strides, unit stride along k_in),
    e.g. the [n_lists, T, k_in] result of an all-gather permuted to token-major.
    """
    T, n_lists, k_in = vals.shape
    if vals.stride() != idxs.stride() or vals.stride(2) != 1:
        raise ValueError("vals and idxs need identical strides with unit stride along k")
    v = torch.empty((T, k_out), dtype=torch.float32, device=vals.device)
    i = torch.empty((T, k_out), dtype=torch.int32, device=vals.device)
    a = torch.empty((T,), dtype=torch.int32, device=vals.device)
    check(ctx._lib.w8a8_topk_merge(ctx.handle, vals.data_ptr(), idxs.data_ptr(), T, n_lists, k_in,
                                   vals.stride(1), vals.stride(0), k_out, v.data_ptr(),
                                   i.data_ptr(), a.data_ptr(), _stream(stream)),
          "w8a8_topk_merge")
    return v, i, a


def _check_dev(t: torch.Tensor, dtype: torch.dtype, cols: int | None = None) -> None:
    if not t.is_cuda:
        raise ValueError("expected a CUDA tensor (the W8A8 path has no CPU fallback)")
    if t.dtype != dtype:
        raise ValueError(f"expected {dtype}, got {t.dtype}")
    if t.dim() != 2 or t.stride(1) != 1:
        raise ValueError("expected a 2-D row-major tensor")
    if cols is not None and t.shape[1] != cols:
        raise ValueError(f"expected {cols} columns, got {t.shape[1]}")


class Linear16:
    """int16 x int16 linear with the QuantM requant to int16 (w8a8_linear16_*): the w2 stage of
    the reference's SwiGLU MLP subgraph (int16 product silu(gate) * up in, int16 weight codes,
    trunc 28), optionally unpacked to fp32 with out_step_chan."""

    def __init__(self, ctx: Context, weights: np.ndarray, quant_m: np.ndarray, trunc: int = 28,
                 out_step_chan: np.ndarray | None = None, max_tokens: int = 64):
        import ctypes as C
        self._lib = ctx._lib
        self.ctx = ctx
        w = np.ascontiguousarray(weights, dtype=np.int16)
        qm = np.ascontiguousarray(quant_m, dtype=np.int16)
        osc = None if out_step_chan is None else np.ascontiguousarray(out_step_chan, np.float32)
        self.N, self.K = map(int, w.shape)
        h = C.c_void_p()
        check(self._lib.w8a8_linear16_create(ctx.handle, self.K, self.N, w.ctypes.data, self.K,
                                             qm.ctypes.data, int(trunc),
                                             osc.ctypes.data if osc is not None else None,
                                             int(max_tokens), C.byref(h)), "w8a8_linear16_create")
        self.handle = h

    def forward(self, x: torch.Tensor, out_mode: int = OUT_QUANT, out=None, stream=None):
        T = x.shape[0]
        if x.dtype != torch.int16 or x.stride(-1) != 1 or x.shape[1] != self.K:
            raise ValueError("x must be an int16 [T, K] tensor with unit column stride")
        dt = torch.float32 if out_mode == OUT_F32 else torch.int16
        y = out if out is not None else torch.empty((T, self.N), dtype=dt, device=x.device)
        ldx = x.stride(0) if T > 1 else self.K
        check(self._lib.w8a8_linear16_forward(self.handle, x.data_ptr(), ldx, T, int(out_mode),
                                              y.data_ptr(), y.stride(0) if T > 1 else self.N,
                                              _stream(stream)), "w8a8_linear16_forward")
        return y

    def close(self) -> None:
        if getattr(self, "handle", None):
            self._lib.w8a8_linear16_destroy(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

