"""One decode step of a W8A8 model: every linear of every layer, then the vocab-sharded LM
head with top-k / argmax -- the hot path of the reference's decode loop
(Lfm3Engine::forward_chunk, src/LFM3/lfm3_v2.cpp:1743, and TransformerSession::step,
src/eswin_runtime/src/llm/transformer_session.cpp:616-846), restricted to the quantised
linears and the LM head.  Attention, norms, residual adds and the SwiGLU product are not part
of that path: each linear consumes the previous linear's output (o takes the q slice of qkv,
down takes the gate slice of gate_up), so the chain has real data dependences.

Multi-GPU (one process per GPU): every rank runs its own T tokens through a full replica of the
linear stack; each rank's int8-quantised final hidden states go to every rank (the reference
broadcasts the final hidden state into both dies' buffers, lfm3_v2.cpp:810-831), every rank runs
its contiguous vocab shard of the LM head over all ranks' tokens, and only each token's top-k
(value, id) pairs go back to the token's owner, which merges them.  That exchange is done by the
library (RankLmHead: peer stores into CUDA-IPC-mapped memory, device counters), so the whole step
is one CUDA graph on every rank with no collective call.
"""
from __future__ import annotations

import math
from dataclasses import dataclass

import numpy as np
import torch

from ._lib import (ACT_STATIC, DTYPE_INT8, ERR_NOT_SUPPORTED, OUT_F32, OUT_F32_ACC,
                   TC_MIN_TOKENS, W8A8Error)
from .chain import ChainStepSpec, DecodeChain
from .linear import Context, SubgraphScaleInfo, W8A8Linear
from .lmhead import LmHeadShard, RankLmHead, shard_range
from .quantize import build_linear
from .synth import DecodeShape, activations, outlier_channels

LM_CHUNK = 4096  # LM-head rows are generated in seeded chunks so every sharding agrees
LM_NORM_EPS = 1e-5  # the final RMSNorm's epsilon (fused_emb_norm_broadcast_t1's default)


@dataclass
class StepBytes:
    linear: int      # algorithmic bytes of all linears (per rank per step)
    lm_head: int     # algorithmic bytes of this rank's LM-head shard
    gemv_launch: int  # algorithmic bytes of one launch of the dominant GEMV (gate_up)


def _lm_rows(K: int, lo: int, hi: int, seed: int, device) -> tuple[np.ndarray, np.ndarray]:
    """Rows [lo, hi) of the synthetic LM head: fp32 N(0, 0.02) quantised per row."""
    wq_parts, step_parts = [], []
    c0 = lo // LM_CHUNK
    c1 = (hi + LM_CHUNK - 1) // LM_CHUNK
    for c in range(c0, c1):
        g = torch.Generator(device=device).manual_seed(seed * 1_000_003 + c)
        w = torch.randn((LM_CHUNK, K), generator=g, device=device, dtype=torch.float32) * 0.02
        r0, r1 = max(lo, c * LM_CHUNK), min(hi, (c + 1) * LM_CHUNK)
        w = w[r0 - c * LM_CHUNK:r1 - c * LM_CHUNK].double()
        step = w.abs().amax(dim=1, keepdim=True).clamp(min=1e-12) / 127.0
        wq = torch.clamp(torch.round(w / step), -127, 127).to(torch.int8)
        wq_parts.append(wq.cpu().numpy())
        step_parts.append(step[:, 0].cpu().numpy())
    return np.concatenate(wq_parts), np.concatenate(step_parts)


def lm_input_norm(K: int, seed: int, device,
                  calib: torch.Tensor | None = None) -> tuple[float, np.ndarray]:
    """The synthetic final RMSNorm of the LM head's input: (in_step, emb_norm_scaled [K] fp32).
    Norm weight 1 + N(0, 0.05^2); in_step = max |normalised calibration row| / 127 over the
    calibration rows (the stack's final calibration hidden states, else 64 synthetic rows);
    emb_norm_scaled = weight * (1 / in_step) in fp32 (lfm3_v2.cpp:3906-3912)."""
    g = torch.Generator(device=device).manual_seed(seed * 1_000_003 + 29)
    norm_w = 1.0 + 0.05 * torch.randn((K,), generator=g, device=device, dtype=torch.float32)
    if calib is None:
        calib = activations(64, K, seed + 23, device=device)
    normed = calib * torch.rsqrt(calib.pow(2).mean(dim=1, keepdim=True) + LM_NORM_EPS) * norm_w
    in_step = float(normed.abs().amax().item()) / 127.0
    inv_step = np.float32(1.0) / np.float32(in_step)
    return in_step, (norm_w.cpu().numpy() * inv_step).astype(np.float32)


class DecodeStack:
    """stat / clamp select the SmoothQuant statistic of every linear (quantize.smooth_scales):
    the reference builder's rms with the [0.05, 20] clamp by default, or max |x| with no clamp
    (the SmolLM-shaped workload).  share_from: another stack of the same shape, seed, layers,
    smoothing and sharding whose linears and LM-head shard this one uses instead of building its
    own (a second token count over the same weights)."""

    def __init__(self, ctx: Context, shape: DecodeShape, T: int, rank: int = 0, world: int = 1,
                 group=None, seed: int = 0, layers: int | None = None, k: int = 40,
                 lm_vocab: int | None = None, use_chain: bool = True, stat: str = "rms",
                 clamp: tuple[float, float] | None = (0.05, 20.0),
                 share_from: "DecodeStack | None" = None):
        self.ctx = ctx
        self.shape = shape
        self.T = int(T)
        self.rank, self.world, self.group = int(rank), int(world), group
        self.k = int(k)
        self.layers = shape.layers if layers is None else int(layers)
        dev = torch.device("cuda", ctx.device)
        self.dev = dev
        self.subgraphs = shape.subgraphs()
        self.linears: list[list[W8A8Linear]] = []
        self.params_host = []  # kept for the CPU baseline and the oracle check
        if share_from is not None:
            src = share_from
            if (src.shape != shape or src.layers != self.layers or src.world != self.world
                    or src.rank != self.rank or src.ctx is not ctx):
                raise ValueError("share_from must be a stack of the same shape, layers, "
                                 "sharding and context")
            self.linears, self.params_host = src.linears, src.params_host
            self.V, self.lo, self.hi = src.V, src.lo, src.hi
            self.lm_in_step, self.lm_host, self.lm = src.lm_in_step, src.lm_host, src.lm
            self.lm_norm, self.lm_emb = src.lm_norm, src.lm_emb
            self.rank_head = src.rank_head
            if self.rank_head is not None and self.T * self.world > 64:
                raise ValueError("a vocab-sharded head takes world * T <= 64 tokens a forward")
            self._shared = src  # keeps the owner alive
            self._buffers()
            self._plan_chain(use_chain)
            return
        # Weights N(0, 1/K) (variance preserving: the linears-only stack has no norms between
        # layers).  Calibration as in post-training quantisation: 64 calibration rows (N(0, 1)
        # with 1 % outlier channels x20) enter layer 0, and every linear is calibrated on the
        # fp32 outputs its calibration rows give upstream (o on the q slice of qkv, down on the
        # gate slice of gate_up), so each linear's output steps match the activations it sees
        # and the quantised stack tracks the fp32 one over any depth.
        calib_h = activations(64, shape.hidden, seed * 7919 + 1, device=dev)
        for layer in range(self.layers):
            row = []
            cal_out = {}
            for j, (name, K, N, trunc) in enumerate(self.subgraphs):
                s = seed * 7919 + layer * 16 + j
                g = torch.Generator(device=dev).manual_seed(s)
                w = torch.randn((N, K), generator=g, device=dev, dtype=torch.float32) / math.sqrt(K)
                calib = {"qkv": lambda: calib_h,
                         "o": lambda: cal_out["qkv"][:, :shape.q],
                         "gate_up": lambda: cal_out["o"],
                         "down": lambda: cal_out["gate_up"][:, :shape.ffn]}[name]().contiguous()
                p = build_linear(w, calib, trunc=trunc, stat=stat, clamp=clamp)
                cal_out[name] = calib @ w.t()
                del w, calib
                scale = SubgraphScaleInfo(in_dtype=DTYPE_INT8, out_dtype=DTYPE_INT8,
                                          in_thresh=p.in_thresh, in_step=p.in_step,
                                          in_inv_smooth=p.in_inv_smooth,
                                          out_step_chan=p.out_step_chan)
                row.append(W8A8Linear(ctx, p.wq, scale, quant_m=p.quant_m, trunc=p.trunc,
                                      acc_step=p.acc_step))
                self.params_host.append((name, p))
            self.linears.append(row)
            calib_h = cal_out["down"]
            del cal_out
        # LM head: the final RMSNorm folded into a static int8 pack, as the reference's
        # fused_emb_norm_broadcast_t1 (lfm3_v2.cpp:810-831): q = round_clamp(h * inv_rms *
        # emb_norm_scaled[c], 127) with emb_norm_scaled = norm weight * (1 / in_step)
        # (:3906-3912), in_step calibrated on normalised rows; logit = float(acc) * in_step *
        # w_step[v].  The norm weight is seeded 1 + N(0, 0.05^2).
        K = shape.hidden
        V = shape.vocab if lm_vocab is None else int(lm_vocab)
        self.V = V
        self.lo, self.hi = shard_range(V, self.world, self.rank)
        wq, w_step = _lm_rows(K, self.lo, self.hi, seed + 17, dev)
        self.lm_in_step, emb = lm_input_norm(K, seed, dev, calib=calib_h)
        del calib_h
        self.lm_norm = (emb, LM_NORM_EPS)
        self.lm_emb = torch.from_numpy(emb).to(dev)
        acc_step = (self.lm_in_step * w_step).astype(np.float32)
        self.lm_host = (wq, acc_step)
        self.lm, self.rank_head = None, None
        if self.world == 1:
            self.lm = LmHeadShard(ctx, wq, acc_step, self.lm_in_step, row_offset=self.lo)
            self.lm.set_input_norm(self.lm_emb, LM_NORM_EPS)
        else:
            # this rank's vocab shard; the library exchanges activations and candidates with the
            # other ranks (peer stores into CUDA-IPC-mapped memory).  The 64-byte handles are
            # exchanged once here, over the process group (set-up plumbing only).
            import torch.distributed as dist
            self.rank_head = RankLmHead(ctx, self.rank, self.world, wq, acc_step,
                                        self.lm_in_step, V, max_tokens=max(self.T, 8) if
                                        self.world * 8 <= 64 else self.T, k_max=self.k)
            self.rank_head.set_input_norm(self.lm_emb, LM_NORM_EPS)
            handles = [None] * self.world
            dist.all_gather_object(handles, self.rank_head.export(), group=self.group)
            self.rank_head.connect(handles)
        self._buffers()
        self._plan_chain(use_chain)

    def _buffers(self) -> None:
        """Persistent device buffers of one step."""
        dev, K = self.dev, self.shape.hidden
        self.x = torch.zeros((self.T, K), dtype=torch.float32, device=dev)
        self.outs = [torch.empty((self.T, N), dtype=torch.float32, device=dev)
                     for (_, _, N, _) in self.subgraphs]
        self.ids = torch.empty((self.T,), dtype=torch.int32, device=dev)
        self.top_val = torch.empty((self.T, self.k), dtype=torch.float32, device=dev)
        self.top_idx = torch.empty((self.T, self.k), dtype=torch.int32, device=dev)
        self.graph = None

    def _plan_chain(self, use_chain: bool) -> None:
        # the persistent chain kernel covers decode batches of up to 8 tokens; larger batches run
        # each linear as act_quant + tensor-core GEMM
        self.chain_lm = False  # the chain's last step is the (unsharded) LM head
        self.chain = None
        if use_chain and self.T <= 8:
            # one token: the LM head is the chain's last step; several tokens: it runs after the
            # chain, where each token's top-k selection has a CTA of its own (T = 8: 2.35 against
            # 2.42 ms per step with the head inside)
            if self.world == 1 and self.T == 1:
                try:
                    self.chain = self._build_chain(with_lm=True)
                    self.chain_lm = True
                except W8A8Error as e:
                    # the LM head's per-CTA logit keys for T tokens do not fit the kernel's
                    # shared memory next to the linears' staging: the head runs as its own
                    # top-k GEMV after the chain
                    if e.status != ERR_NOT_SUPPORTED:
                        raise
            if self.chain is None:
                self.chain = self._build_chain(with_lm=False)

    def _build_chain(self, with_lm: bool) -> DecodeChain:
        """The whole linear stack (+ the LM head when with_lm) as one persistent kernel: same
        buffers and the same data dependences as run_linears / run_lm_head."""
        qkv, o, gu, down = self.outs
        x = self.x
        steps = []
        for row in self.linears:
            steps.append(ChainStepSpec(row[0], x, qkv))
            steps.append(ChainStepSpec(row[1], qkv[:, :self.shape.q], o))
            steps.append(ChainStepSpec(row[2], o, gu))
            steps.append(ChainStepSpec(row[3], gu[:, :self.shape.ffn], down))
            x = down
        if with_lm:
            steps.append(ChainStepSpec(self.lm.linear, down, None, act_mode=ACT_STATIC,
                                       out_mode=OUT_F32_ACC, topk_k=self.k,
                                       row_offset=self.lo, topk_val=self.top_val,
                                       topk_idx=self.top_idx, emb_norm=self.lm_emb,
                                       norm_eps=LM_NORM_EPS))
        return DecodeChain(self.ctx, steps, self.T)

    def launches_per_step(self) -> int:
        """Kernels of this library launched per step."""
        T_all = self.T * self.world
        # LM head: act_quant + top-k GEMV per group of 8 tokens, + the per-token selection kernel
        # after a GEMV of two or more tokens (+ merge when sharded, + the argmax copy when not)
        groups = [min(8, T_all - g) for g in range(0, T_all, 8)]
        lm = 1 + len(groups) + sum(1 for g in groups if g >= 2) + 1
        if self.world == 1 and self.T >= TC_MIN_TOKENS:
            # act_quant, one tensor-core GEMM into the logits, row lists, selection, argmax copy
            lm = 5
        if self.chain is not None:
            return 1 + (1 if self.chain_lm else lm)
        # each linear: act_quant + one tensor-core GEMM, or a GEMV per group of 8 tokens
        contraction = 1 if self.T >= TC_MIN_TOKENS else (self.T + 7) // 8
        return self.layers * 4 * (1 + contraction) + lm

    def lm_oracle(self) -> tuple:
        """This rank's LM head for the oracle: (wq, acc_step, in_step, emb_norm_scaled, eps)."""
        return (self.lm_host[0], self.lm_host[1], self.lm_in_step, self.lm_norm[0], self.lm_norm[1])

    # ------------------------------------------------------------------ byte accounting
    def step_bytes(self) -> StepBytes:
        T = self.T
        lin = 0
        for (_, K, N, _) in self.subgraphs:
            lin += N * K + T * K * 4 + T * N * 4 + K * 4 + N * (4 + 2 + 4)
        lin *= self.layers
        K = self.shape.hidden
        Vs = self.hi - self.lo
        T_all = T * self.world
        lm = Vs * K + T_all * K * 4 + Vs * 4 + T_all * self.k * 8
        _, K, N, _ = self.subgraphs[2]  # gate_up, the largest subgraph
        gemv = N * K + T * K + T * N * 4 + N * (2 + 4)
        return StepBytes(lin, lm, gemv)

    # ------------------------------------------------------------------ the step
    def run_linears(self) -> None:
        x = self.x
        qkv, o, gu, down = self.outs
        q_width = self.shape.q
        for row in self.linears:
            row[0].forward(x, OUT_F32, dyntok=True, out=qkv)
            row[1].forward(qkv[:, :q_width], OUT_F32, dyntok=True, out=o)
            row[2].forward(o, OUT_F32, dyntok=True, out=gu)
            row[3].forward(gu[:, :self.shape.ffn], OUT_F32, dyntok=True, out=down)
            x = down

    def run_lm_head(self) -> None:
        h = self.outs[3]
        if self.world == 1:
            self.lm.forward(h, self.k, OUT_F32_ACC, val=self.top_val, idx=self.top_idx)
            self.ids.copy_(self.top_idx[:, 0])
            return
        # this rank's shard over every rank's tokens; each token's candidates go to its owner,
        # which merges them (all inside the library, on this stream)
        self.rank_head.forward(h, self.k, val=self.top_val, idx=self.top_idx, argmax=self.ids)

    def run_device(self) -> None:
        """One whole step on the device (the sharded head's exchange included)."""
        if self.chain is not None:
            self.chain.forward()
            if self.chain_lm:
                self.ids.copy_(self.top_idx[:, 0])
            else:
                self.run_lm_head()
            return
        self.run_linears()
        self.run_lm_head()

    def capture(self) -> None:
        """Captures the whole step in a CUDA graph."""
        s = torch.cuda.Stream(device=self.dev)
        s.wait_stream(torch.cuda.current_stream(self.dev))
        with torch.cuda.stream(s):
            self.run_device()
        torch.cuda.current_stream(self.dev).wait_stream(s)
        torch.cuda.synchronize(self.dev)
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            self.run_device()
        self.graph = g

    def step(self) -> None:
        if self.graph is not None:
            self.graph.replay()
        else:
            self.run_device()

    def capture_host(self, x_host: torch.Tensor, ids_host: torch.Tensor) -> None:
        """Captures the end-to-end step for these pinned host buffers as one CUDA graph: the
        host -> device copy of the activations, the whole step and the device -> host copy of the
        sampled ids (both copies run on every replay)."""
        s = torch.cuda.Stream(device=self.dev)
        s.wait_stream(torch.cuda.current_stream(self.dev))
        with torch.cuda.stream(s):
            self.x.copy_(x_host, non_blocking=True)
            self.run_device()
            ids_host.copy_(self.ids, non_blocking=True)
        torch.cuda.current_stream(self.dev).wait_stream(s)
        torch.cuda.synchronize(self.dev)
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            self.x.copy_(x_host, non_blocking=True)
            self.run_device()
            ids_host.copy_(self.ids, non_blocking=True)
        self.host_graph = (g, x_host, ids_host)

    def step_host(self, x_host: torch.Tensor, ids_host: torch.Tensor) -> None:
        """End-to-end step through the public API: pinned host activations in, sampled ids out
        (one graph replay when capture_host was called for these buffers)."""
        hg = getattr(self, "host_graph", None)
        if hg is not None and hg[1] is x_host and hg[2] is ids_host:
            hg[0].replay()
            return
        self.x.copy_(x_host, non_blocking=True)
        self.step()
        ids_host.copy_(self.ids, non_blocking=True)

    def release(self) -> None:
        self.graph = None
        self.host_graph = None
