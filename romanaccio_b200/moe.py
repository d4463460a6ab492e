"""Mixture-of-experts decode layer over the C ABI (w8a8_moe_*): device router, W8A8 experts
(gate|up, silu * up, down) and the weighted combine, with no host round trip in between.

Reference: MoERouter::route (src/eswin_runtime/src/llm/moe_router.cpp:211-260) and the expert
combine of src/LFM2.5-8B-A1B/lfm2_moe.cpp:2300-2318 (mlp_out += y_q * (w_k * out_step_chan)).
Pair p = t * slots + j: slots 0..k-1 are the token's routed experts in routing order, the rest
the shared experts (weight 1), stored after the routed ones.
"""
from __future__ import annotations

import ctypes as C
from dataclasses import dataclass

import numpy as np
import torch

from . import _lib
from ._lib import DTYPE_INT8, DTYPE_INT16, check
from .linear import Context, _stream
from .quantize import LinearParams, build_linear
from .synth import activations


class _DeviceArray:
    """Zero-copy __cuda_array_interface__ view of a device buffer owned by the library."""

    def __init__(self, ptr: int, shape: tuple[int, ...], typestr: str):
        self.__cuda_array_interface__ = {"shape": tuple(shape), "typestr": typestr,
                                         "data": (int(ptr), False), "version": 2}


@dataclass
class MoEParams:
    """Expert-major host arrays of one MoE layer (E routed + S shared experts)."""

    gate_w: np.ndarray            # fp32 [E, H]
    gate_bias: np.ndarray | None  # fp32 [E]
    gu: list[LinearParams]        # E + S gate|up linears, [2I, H] each (gate rows first)
    dn: list[LinearParams]        # E + S down linears, [H, I] each
    top_k: int
    norm_topk_prob: bool = False
    routed_scaling: float = 1.0
    dn_out_dtype: int = DTYPE_INT8

    @property
    def n_routed(self) -> int:
        return int(self.gate_w.shape[0])

    @property
    def n_shared(self) -> int:
        return len(self.gu) - self.n_routed

    @property
    def hidden(self) -> int:
        return int(self.gate_w.shape[1])

    @property
    def inter(self) -> int:
        return int(self.gu[0].wq.shape[0] // 2)


def make_moe_params(H: int, I: int, E: int, S: int, k: int, seed: int, device="cpu",
                    dn_out_dtype: int = DTYPE_INT8) -> MoEParams:
    """Seeded DeepSeek-V2-Lite-style layer: N(0, 0.02) weights quantised by the SmoothQuant
    builder per expert (gate|up calibrated on the layer-input distribution, down on a separate
    seeded batch), router weights N(0, 0.02)."""
    g = torch.Generator().manual_seed(seed)
    gate_w = (torch.randn((E, H), generator=g) * 0.02).numpy().astype(np.float32)
    gu, dn = [], []
    for e in range(E + S):
        s = seed * 1009 + e * 7
        g1 = torch.Generator(device=device).manual_seed(s)
        w1 = torch.randn((2 * I, H), generator=g1, device=device) * 0.02
        gu.append(build_linear(w1, activations(64, H, s + 1, device=device)))
        g2 = torch.Generator(device=device).manual_seed(s + 2)
        w2 = torch.randn((H, I), generator=g2, device=device) * 0.02
        dn.append(build_linear(w2, activations(64, I, s + 3, device=device)))
    return MoEParams(gate_w=gate_w, gate_bias=None, gu=gu, dn=dn, top_k=k,
                     dn_out_dtype=dn_out_dtype)


class MoELayer:
    def __init__(self, ctx: Context, p: MoEParams, max_tokens: int = 64):
        self._lib = ctx._lib
        self.ctx = ctx
        self.p = p
        X = len(p.gu)
        H, I = p.hidden, p.inter
        self.slots = p.top_k + p.n_shared
        self.max_tokens = int(max_tokens)
        if len({q.trunc for q in p.gu}) != 1 or len({q.trunc for q in p.dn}) != 1:
            raise ValueError("all experts of a projection must share trunc")
        arr = {
            "gate_w": np.ascontiguousarray(p.gate_w, np.float32),
            "gu_w": np.ascontiguousarray(np.stack([q.wq for q in p.gu]), np.int8),
            "gu_qm": np.ascontiguousarray(np.stack([q.quant_m for q in p.gu]), np.int16),
            "gu_os": np.ascontiguousarray(np.stack([q.out_step_chan for q in p.gu]), np.float32),
            "gu_s": np.ascontiguousarray(np.stack([q.in_inv_smooth for q in p.gu]), np.float32),
            "gu_thr": np.array([q.in_thresh for q in p.gu], np.float32),
            "dn_w": np.ascontiguousarray(np.stack([q.wq for q in p.dn]), np.int8),
            "dn_qm": np.ascontiguousarray(np.stack([q.quant_m for q in p.dn]), np.int16),
            "dn_os": np.ascontiguousarray(np.stack([q.out_step_chan for q in p.dn]), np.float32),
            "dn_s": np.ascontiguousarray(np.stack([q.in_inv_smooth for q in p.dn]), np.float32),
            "dn_step": np.array([q.in_step for q in p.dn], np.float32),
        }
        bias = None if p.gate_bias is None else np.ascontiguousarray(p.gate_bias, np.float32)
        assert arr["gu_w"].shape == (X, 2 * I, H) and arr["dn_w"].shape == (X, H, I)
        d = _lib.MoeDesc(
            hidden=H, inter=I, n_routed=p.n_routed, n_shared=p.n_shared, top_k=p.top_k,
            norm_topk_prob=int(p.norm_topk_prob), routed_scaling=float(p.routed_scaling),
            max_tokens=self.max_tokens, gate_w=arr["gate_w"].ctypes.data,
            gate_bias=bias.ctypes.data if bias is not None else None,
            gu_weights=arr["gu_w"].ctypes.data, gu_quant_m=arr["gu_qm"].ctypes.data,
            gu_out_step_chan=arr["gu_os"].ctypes.data, gu_inv_smooth=arr["gu_s"].ctypes.data,
            gu_in_thresh=arr["gu_thr"].ctypes.data, gu_trunc=int(p.gu[0].trunc),
            dn_weights=arr["dn_w"].ctypes.data, dn_quant_m=arr["dn_qm"].ctypes.data,
            dn_out_step_chan=arr["dn_os"].ctypes.data, dn_inv_smooth=arr["dn_s"].ctypes.data,
            dn_in_step=arr["dn_step"].ctypes.data, dn_trunc=int(p.dn[0].trunc),
            dn_out_dtype=int(p.dn_out_dtype))
        h = C.c_void_p()
        check(self._lib.w8a8_moe_create(ctx.handle, C.byref(d), C.byref(h)), "w8a8_moe_create")
        self.handle = h

    def route(self, hidden: torch.Tensor, stream=None) -> tuple[torch.Tensor, torch.Tensor]:
        T = hidden.shape[0]
        idx = torch.empty((T, self.p.top_k), dtype=torch.int32, device=hidden.device)
        w = torch.empty((T, self.p.top_k), dtype=torch.float32, device=hidden.device)
        check(self._lib.w8a8_moe_route(self.handle, hidden.data_ptr(), hidden.stride(0), T,
                                       idx.data_ptr(), w.data_ptr(), _stream(stream)),
              "w8a8_moe_route")
        return idx, w

    def forward(self, hidden: torch.Tensor, out: torch.Tensor | None = None,
                stream=None) -> torch.Tensor:
        T = hidden.shape[0]
        y = out if out is not None else torch.empty((T, self.p.hidden), dtype=torch.float32,
                                                    device=hidden.device)
        check(self._lib.w8a8_moe_forward(self.handle, hidden.data_ptr(), hidden.stride(0), T,
                                         y.data_ptr(), y.stride(0), _stream(stream)),
              "w8a8_moe_forward")
        return y

    def views(self, T: int) -> dict[str, torch.Tensor]:
        """Copies of the last forward's intermediates (routing, expert stages) for T tokens."""
        ptrs = [C.c_void_p() for _ in range(5)]
        check(self._lib.w8a8_moe_views(self.handle, *[C.byref(p) for p in ptrs]),
              "w8a8_moe_views")
        P, H, I, k = T * self.slots, self.p.hidden, self.p.inter, self.p.top_k
        dq = "<i2" if self.p.dn_out_dtype == DTYPE_INT16 else "|i1"
        torch.cuda.synchronize()

        def grab(ptr, shape, typestr):
            return torch.as_tensor(_DeviceArray(ptr.value, shape, typestr), device="cuda").clone()

        return {"idx": grab(ptrs[0], (T, k), "<i4"), "w": grab(ptrs[1], (T, k), "<f4"),
                "gate_up": grab(ptrs[2], (P, 2 * I), "<f4"),
                "act": grab(ptrs[3], (P, I), "<f4"), "down_q": grab(ptrs[4], (P, H), dq)}

    def close(self) -> None:
        if getattr(self, "handle", None):
            self._lib.w8a8_moe_destroy(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


EP_HANDLE_BYTES = 64


class ExpertParallelMoE:
    """Expert parallelism of one MoE layer over processes (w8a8_moe_ep_*): this rank computes
    the experts e with e % world == rank for every token and the library exchanges and sums the
    ranks' partial combines in rank order (peer stores into CUDA-IPC-mapped memory), so forward()
    returns the whole layer's output on every rank.  The layer's own forward() computes only
    this rank's partial while this object lives.

    Set-up: create on every rank, exchange export() bytes and connect(handles in rank order), or
    connect_local(eps) for ranks of one process (one per GPU).
    """

    def __init__(self, layer: MoELayer, rank: int, world: int, max_tokens: int | None = None):
        self.layer = layer
        self._lib = layer._lib
        self.rank, self.world = int(rank), int(world)
        self.max_tokens = int(max_tokens or layer.max_tokens)
        h = C.c_void_p()
        check(self._lib.w8a8_moe_ep_create(layer.handle, self.rank, self.world,
                                           self.max_tokens, C.byref(h)), "w8a8_moe_ep_create")
        self.handle = h

    def export(self) -> bytes:
        buf = (C.c_ubyte * EP_HANDLE_BYTES)()
        check(self._lib.w8a8_moe_ep_export(self.handle, buf), "w8a8_moe_ep_export")
        return bytes(buf)

    def connect(self, handles: list[bytes]) -> None:
        if len(handles) != self.world or any(len(b) != EP_HANDLE_BYTES for b in handles):
            raise ValueError("one 64-byte handle per rank, in rank order")
        check(self._lib.w8a8_moe_ep_connect(self.handle, b"".join(handles)), "w8a8_moe_ep_connect")

    @staticmethod
    def connect_local(eps: list["ExpertParallelMoE"]) -> None:
        arr = (C.c_void_p * len(eps))(*[x.handle.value for x in eps])
        check(eps[0]._lib.w8a8_moe_ep_connect_local(arr, len(eps)), "w8a8_moe_ep_connect_local")

    def forward(self, hidden: torch.Tensor, out: torch.Tensor | None = None,
                stream=None) -> torch.Tensor:
        T = hidden.shape[0]
        y = out if out is not None else torch.empty((T, self.layer.p.hidden), dtype=torch.float32,
                                                    device=hidden.device)
        check(self._lib.w8a8_moe_ep_forward(self.handle, hidden.data_ptr(), hidden.stride(0), T,
                                            y.data_ptr(), y.stride(0), _stream(stream)),
              "w8a8_moe_ep_forward")
        return y

    def close(self) -> None:
        if getattr(self, "handle", None):
            self._lib.w8a8_moe_ep_destroy(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

