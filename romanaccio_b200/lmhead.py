"""Vocab-sharded W8A8 LM head with a fused top-k / argmax epilogue.

The reference splits the LM head into contiguous vocab halves across its two NPU dies
(src/eswin_compiler/passes/dual_die_splitter.py:63-147: die 0 gets rows [0, V//2), die 1 the
rest), runs both halves concurrently (run_dual_die, src/LFM3/lfm3_v2.cpp:1311-1332;
forward_lm_head_dual_die, src/eswin_runtime/src/llm/transformer_session.cpp:538-614),
concatenates the logits on the host and samples over the full vocabulary
(src/eswin_runtime/src/nlp/sampler.cpp:83-121).

Here each of n ranks (one process per GPU) owns rows [floor(r*V/n), floor((r+1)*V/n)), its
kernel keeps the shard's logits on chip and emits only the sorted top-k (value, vocab id)
pairs, the ranks exchange those k*8 bytes, and a merge kernel produces the global top-k and the
greedy argmax (lowest id on ties, as Sampler::sample's strict '>').
"""
from __future__ import annotations

import numpy as np
import torch

from ._lib import DTYPE_INT8, OUT_F32_ACC, check
from .linear import Context, SubgraphScaleInfo, W8A8Linear, topk_merge


def shard_range(V: int, n: int, r: int) -> tuple[int, int]:
    """Contiguous vocab block of shard r of n (n = 2 gives the reference's halves)."""
    return (r * V) // n, ((r + 1) * V) // n


def candidate_buffers(T_all: int, k: int, world: int, device) -> tuple[torch.Tensor, torch.Tensor]:
    """(local [2, T_all, k], gathered [world * 2, T_all, k]) int32 exchange buffers; row 0 of a
    pair holds the float32 values bit-cast, row 1 the vocab ids."""
    local = torch.empty((2, T_all, k), dtype=torch.int32, device=device)
    gathered = torch.empty((world * 2, T_all, k), dtype=torch.int32, device=device)
    return local, gathered


def exchange_candidates(local: torch.Tensor, gathered: torch.Tensor, group=None) -> None:
    """All-gather every shard's [2, T_all, k] candidate block (k * 8 bytes per token per shard)."""
    import torch.distributed as dist

    dist.all_gather_into_tensor(gathered, local, group=group)


def token_candidates(gathered: torch.Tensor, world: int, t0: int, T: int):
    """[T, world, k] views (values, ids) of tokens [t0, t0 + T) in the gathered block."""
    g = gathered.view(world, 2, gathered.shape[1], gathered.shape[2])
    vals = g[:, 0, t0:t0 + T].view(torch.float32).permute(1, 0, 2)
    ids = g[:, 1, t0:t0 + T].permute(1, 0, 2)
    return vals, ids


class LmHeadShard:
    """This rank's block of vocab rows as a W8A8 linear whose output is a top-k list."""

    def __init__(self, ctx: Context, wq_rows: np.ndarray, acc_step_rows: np.ndarray,
                 in_step: float, row_offset: int, in_inv_smooth: np.ndarray | None = None,
                 quant_m_rows: np.ndarray | None = None, trunc: int = 22,
                 out_step_chan_rows: np.ndarray | None = None, out_step: float = 1.0 / 127.0):
        scale = SubgraphScaleInfo(in_dtype=DTYPE_INT8, out_dtype=DTYPE_INT8, in_step=in_step,
                                  in_thresh=in_step * 127.0, out_step=out_step,
                                  in_inv_smooth=in_inv_smooth, out_step_chan=out_step_chan_rows)
        self.linear = W8A8Linear(ctx, wq_rows, scale, quant_m=quant_m_rows, trunc=trunc,
                                 acc_step=acc_step_rows)
        self.row_offset = int(row_offset)
        self.rows = int(wq_rows.shape[0])

    def set_input_norm(self, emb_norm_scaled: torch.Tensor | None, eps: float = 1e-5) -> None:
        """Fuses the reference's LM-head input RMSNorm (fused_emb_norm_broadcast_t1) into the
        static pack of forward(): h is then the un-normalised final hidden state."""
        if emb_norm_scaled is not None and (emb_norm_scaled.dtype != torch.float32
                                            or not emb_norm_scaled.is_contiguous()
                                            or emb_norm_scaled.numel() != self.linear.K):
            raise ValueError("emb_norm_scaled must be a contiguous fp32 [K] tensor")
        self._norm = emb_norm_scaled  # kept alive: the library holds the device pointer
        check(self.linear._lib.w8a8_linear_set_input_norm(
            self.linear.handle, emb_norm_scaled.data_ptr() if emb_norm_scaled is not None else None,
            float(eps)), "w8a8_linear_set_input_norm")

    def forward(self, h: torch.Tensor, k: int, out_mode: int = OUT_F32_ACC, val=None, idx=None,
                logits=None, stream=None):
        return self.linear.forward_topk(h, k, row_offset=self.row_offset, out_mode=out_mode,
                                        dyntok=False, val=val, idx=idx, logits=logits,
                                        stream=stream)


class VocabShardedLmHead:
    """LM head over `world` ranks; rank `rank` builds only its shard.

    forward(h) -> (top-k values [T, k], top-k vocab ids [T, k], argmax [T]) on every rank.
    The exchange is one all-gather of the [T, k] (value, id) pairs through torch.distributed
    (NCCL over NVLink between GPUs); with world == 1 there is no exchange.
    """

    def __init__(self, ctx: Context, V: int, rank: int = 0, world: int = 1, group=None):
        self.ctx = ctx
        self.V = int(V)
        self.rank = int(rank)
        self.world = int(world)
        self.group = group
        self.lo, self.hi = shard_range(self.V, self.world, self.rank)
        self.shard: LmHeadShard | None = None
        self._bufs: dict[tuple[int, int], tuple[torch.Tensor, torch.Tensor]] = {}

    def load_shard(self, wq_full_or_rows: np.ndarray, acc_step: np.ndarray, in_step: float,
                   rows_are_shard: bool = False, **kw) -> None:
        """Uploads this rank's rows (pass the full [V, K] matrix or only the shard's rows)."""
        if rows_are_shard:
            rows, steps = wq_full_or_rows, acc_step
        else:
            rows = wq_full_or_rows[self.lo:self.hi]
            steps = acc_step[self.lo:self.hi]
        self.shard = LmHeadShard(self.ctx, rows, steps, in_step, self.lo, **kw)

    def _buffers(self, T: int, k: int, device) -> tuple[torch.Tensor, torch.Tensor]:
        key = (T, k)
        if key not in self._bufs:
            self._bufs[key] = candidate_buffers(T, k, self.world, device)
        return self._bufs[key]

    def forward(self, h: torch.Tensor, k: int = 40, out_mode: int = OUT_F32_ACC, stream=None):
        """h: the same [T, K] hidden states on every rank (the reference broadcasts the final
        hidden state into both dies' input buffers)."""
        assert self.shard is not None, "load_shard() first"
        T = h.shape[0]
        if self.world == 1:
            v, i = self.shard.forward(h, k, out_mode=out_mode, stream=stream)
            return v, i, i[:, 0]
        local, gathered = self._buffers(T, k, h.device)
        self.shard.forward(h, k, out_mode=out_mode, val=local[0].view(torch.float32),
                           idx=local[1], stream=stream)
        exchange_candidates(local, gathered, self.group)
        vals, ids = token_candidates(gathered, self.world, 0, T)
        return topk_merge(self.ctx, vals, ids, k, stream=stream)


class MultiDeviceLmHead:
    """Vocab-sharded LM head over several devices driven by this process (w8a8_lmhead_*).

    Shard s holds vocab rows shard_range(V, n, s) on the device of ctxs[s]; forward(h) with h
    on ctxs[0]'s device returns (top-k values [T, k], top-k vocab ids [T, k], argmax [T]) there.
    Device 0 stores the quantised h into every shard's staging buffer over NVLink, the shards
    store their candidates into device 0, and one merge kernel finishes; shards on other devices
    synchronise through device-memory counters (no stream events), so a head with such shards is
    not graph-capturable and takes at most 8 tokens a forward.
    """

    def __init__(self, ctxs: list[Context], wq: np.ndarray, acc_step: np.ndarray,
                 in_step: float, max_tokens: int = 8, k_max: int = 64):
        import ctypes as C
        from ._lib import check
        self._lib = ctxs[0]._lib
        self.ctxs = list(ctxs)
        self.device = ctxs[0].device
        w = np.ascontiguousarray(wq, dtype=np.int8)
        st = np.ascontiguousarray(acc_step, dtype=np.float32)
        self.V, self.K = map(int, w.shape)
        arr = (C.c_void_p * len(ctxs))(*[c.handle.value for c in ctxs])
        h = C.c_void_p()
        check(self._lib.w8a8_lmhead_create(arr, len(ctxs), self.K, self.V, w.ctypes.data,
                                           self.K, st.ctypes.data, float(in_step),
                                           int(max_tokens), int(k_max), C.byref(h)),
              "w8a8_lmhead_create")
        self.handle = h
        self._check = check

    @property
    def shards(self) -> int:
        return int(self._lib.w8a8_lmhead_shards(self.handle))

    def set_input_norm(self, emb_norm_scaled: torch.Tensor | None, eps: float = 1e-5) -> None:
        """Fuses the reference's LM-head input RMSNorm (fused_emb_norm_broadcast_t1) into the
        forward: h is then the un-normalised final hidden state.  None turns it off."""
        self._norm = emb_norm_scaled  # kept alive: the library holds the device pointer
        self._check(self._lib.w8a8_lmhead_set_input_norm(
            self.handle, emb_norm_scaled.data_ptr() if emb_norm_scaled is not None else None,
            float(eps)), "w8a8_lmhead_set_input_norm")

    def forward(self, h: torch.Tensor, k: int, val=None, idx=None, argmax=None, stream=None):
        from .linear import _stream
        T = h.shape[0]
        dev = h.device
        v = val if val is not None else torch.empty((T, k), dtype=torch.float32, device=dev)
        i = idx if idx is not None else torch.empty((T, k), dtype=torch.int32, device=dev)
        a = argmax if argmax is not None else torch.empty((T,), dtype=torch.int32, device=dev)
        self._check(self._lib.w8a8_lmhead_forward(self.handle, h.data_ptr(), T, int(k),
                                                  v.data_ptr(), i.data_ptr(), a.data_ptr(),
                                                  _stream(stream)), "w8a8_lmhead_forward")
        return v, i, a

    def enable_trace(self) -> tuple[torch.Tensor, list[torch.Tensor]]:
        """Diagnostics: device-0 forward timeline [8] and each shard's per-CTA timeline
        [2 * sm_count, 8] (int64 %globaltimer ns, w8a8_lmhead_set_trace)."""
        import ctypes as C
        head = torch.zeros((8,), dtype=torch.int64, device=f"cuda:{self.device}")
        shards = [torch.zeros((2 * c.sm_count, 8), dtype=torch.int64, device=f"cuda:{c.device}")
                  for c in self.ctxs]
        arr = (C.c_void_p * len(shards))(*[t.data_ptr() for t in shards])
        self._check(self._lib.w8a8_lmhead_set_trace(self.handle, head.data_ptr(), arr),
                    "w8a8_lmhead_set_trace")
        self._trace = (head, shards)
        return head, shards

    def close(self) -> None:
        if getattr(self, "handle", None):
            self._lib.w8a8_lmhead_destroy(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


RANK_HANDLE_BYTES = 64


class RankLmHead:
    """One rank's part of an LM head vocab-sharded over processes (w8a8_lmhead_rank_*): this
    rank's contiguous vocab rows; the exchange of activations and candidates between the ranks is
    done by the library (peer stores into CUDA-IPC-mapped device memory, device counters), so
    forward() is three launches on one stream (four with two or more tokens over all ranks) and
    can be captured in a CUDA graph.

    Set-up: create on every rank, exchange export() bytes (connect(handles) with the list of all
    ranks' handles in rank order), or connect_local(heads) for ranks driven by one process.
    """

    def __init__(self, ctx: Context, rank: int, world: int, wq_rows: np.ndarray,
                 acc_step_rows: np.ndarray, in_step: float, V: int, max_tokens: int = 8,
                 k_max: int = 64):
        import ctypes as C
        from ._lib import check
        self._lib = ctx._lib
        self._check = check
        self.ctx, self.rank, self.world, self.V = ctx, int(rank), int(world), int(V)
        w = np.ascontiguousarray(wq_rows, dtype=np.int8)
        st = np.ascontiguousarray(acc_step_rows, dtype=np.float32)
        self.K = int(w.shape[1])
        lo, hi = shard_range(V, world, rank)
        if w.shape[0] != hi - lo or st.shape[0] != hi - lo:
            raise ValueError(f"rank {rank} of {world} holds vocab rows [{lo}, {hi})")
        h = C.c_void_p()
        check(self._lib.w8a8_lmhead_rank_create(ctx.handle, self.rank, self.world, self.K,
                                                self.V, w.ctypes.data, self.K, st.ctypes.data,
                                                float(in_step), int(max_tokens), int(k_max),
                                                C.byref(h)), "w8a8_lmhead_rank_create")
        self.handle = h
        self.lo, self.hi = lo, hi

    def export(self) -> bytes:
        import ctypes as C
        buf = (C.c_ubyte * RANK_HANDLE_BYTES)()
        self._check(self._lib.w8a8_lmhead_rank_export(self.handle, buf), "w8a8_lmhead_rank_export")
        return bytes(buf)

    def connect(self, handles: list[bytes]) -> None:
        if len(handles) != self.world or any(len(b) != RANK_HANDLE_BYTES for b in handles):
            raise ValueError("one 64-byte handle per rank, in rank order")
        blob = b"".join(handles)
        self._check(self._lib.w8a8_lmhead_rank_connect(self.handle, blob),
                    "w8a8_lmhead_rank_connect")

    def set_input_norm(self, emb_norm_scaled: torch.Tensor | None, eps: float = 1e-5) -> None:
        """Fuses the reference's LM-head input RMSNorm (fused_emb_norm_broadcast_t1) into the
        forward's quantisation: h is then the un-normalised final hidden state."""
        self._norm = emb_norm_scaled
        self._check(self._lib.w8a8_lmhead_rank_set_input_norm(
            self.handle, emb_norm_scaled.data_ptr() if emb_norm_scaled is not None else None,
            float(eps)), "w8a8_lmhead_rank_set_input_norm")

    @staticmethod
    def connect_local(heads: list["RankLmHead"]) -> None:
        import ctypes as C
        arr = (C.c_void_p * len(heads))(*[x.handle.value for x in heads])
        heads[0]._check(heads[0]._lib.w8a8_lmhead_rank_connect_local(arr, len(heads)),
                        "w8a8_lmhead_rank_connect_local")

    def forward(self, h: torch.Tensor, k: int, val=None, idx=None, argmax=None, stream=None):
        from .linear import _stream
        T = h.shape[0]
        dev = h.device
        v = val if val is not None else torch.empty((T, k), dtype=torch.float32, device=dev)
        i = idx if idx is not None else torch.empty((T, k), dtype=torch.int32, device=dev)
        a = argmax if argmax is not None else torch.empty((T,), dtype=torch.int32, device=dev)
        if h.dtype != torch.float32 or not h.is_contiguous() or h.shape[1] != self.K:
            raise ValueError("h must be a contiguous fp32 [T, K] tensor")
        self._check(self._lib.w8a8_lmhead_rank_forward(self.handle, h.data_ptr(), T, int(k),
                                                       v.data_ptr(), i.data_ptr(), a.data_ptr(),
                                                       _stream(stream)), "w8a8_lmhead_rank_forward")
        return v, i, a

    def close(self) -> None:
        if getattr(self, "handle", None):
            self._lib.w8a8_lmhead_rank_destroy(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

