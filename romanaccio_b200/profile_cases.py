"""Small, self-contained launches of one kernel each, sized for an ncu capture.

    python -m romanaccio_b200.profile_cases chain --layers 4 --vocab 1024 --reps 5
    python -m romanaccio_b200.profile_cases gemm 2048 8192 8192 --reps 3 [--pair]
    python -m romanaccio_b200.profile_cases lmhead 151936 --shards 1 --reps 3
    python -m romanaccio_b200.profile_cases moe 64 --reps 3

chain   the persistent decode-chain kernel over a Qwen2.5-1.5B-shaped stack of `layers` layers
        and a `vocab`-row LM head (T = 1), launched `reps` times;
gemm    the tcgen05 tensor-core GEMM of an M x K x N W8A8 linear (int8 input in HBM, int8
        requantised output), launched `reps` times after one tile-building launch (--pair: the
        CTA-pair kernel, PATH_TENSOR_PAIR);
lmhead  the LM-head top-40 GEMV over one shard of a 1536 x `vocab` head (T = 1);
moe     one DeepSeek-V2-Lite-shaped W8A8 MoE layer (hidden 2048, 64 routed + 2 shared experts of
        1408, top-6) over T tokens (router, grouping, expert GEMVs, combine), `reps` times.

Every case checks the context's device error word at the end (a bounded wait that ran out
raises).  The inputs are seeded synthetic tensors of the workloads' shapes.
"""
from __future__ import annotations

import argparse

import numpy as np
import torch

from . import OUT_F32_ACC, OUT_QUANT, PATH_TENSOR, Context, SubgraphScaleInfo, W8A8Linear
from ._lib import PATH_TENSOR_PAIR
from . import DTYPE_INT8, synth


def _random_linear(ctx: Context, K: int, N: int, seed: int = 0) -> W8A8Linear:
    rng = np.random.default_rng(seed)
    wq = rng.integers(-127, 128, size=(N, K)).astype(np.int8)
    qm = rng.integers(1, 32768, size=N).astype(np.int16)
    scale = SubgraphScaleInfo(in_dtype=DTYPE_INT8, out_dtype=DTYPE_INT8, in_thresh=3.0,
                              in_step=0.05,
                              out_step_chan=(rng.random(N) * 0.01 + 1e-5).astype(np.float32))
    return W8A8Linear(ctx, wq, scale, quant_m=qm, trunc=22,
                      acc_step=(rng.random(N) * 1e-4 + 1e-7).astype(np.float32))


def run_chain(ctx: Context, layers: int, vocab: int, reps: int) -> None:
    from .decode import DecodeStack
    stack = DecodeStack(ctx, synth.QWEN25_15B, 1, layers=layers, lm_vocab=vocab)
    for _ in range(reps):
        stack.chain.forward()


def run_gemm(ctx: Context, M: int, K: int, N: int, reps: int, pair: bool = False) -> None:
    lin = _random_linear(ctx, K, N)
    lin.set_path(PATH_TENSOR_PAIR if pair else PATH_TENSOR)
    q = torch.randint(-127, 128, (M, K), dtype=torch.int8, device="cuda")
    y = torch.empty((M, N), dtype=torch.int8, device="cuda")
    for _ in range(reps):
        lin.submit(q, OUT_QUANT, out=y)


def run_lmhead(ctx: Context, vocab: int, shards: int, reps: int) -> None:
    K = synth.QWEN25_15B.hidden
    rows = (vocab + shards - 1) // shards
    lin = _random_linear(ctx, K, rows)
    x = synth.activations(1, K, seed=3).cuda()
    for _ in range(reps):
        lin.forward_topk(x, 40, out_mode=OUT_F32_ACC)


def run_moe(ctx: Context, T: int, reps: int) -> None:
    from .moe import MoELayer, make_moe_params
    dev = torch.device("cuda", ctx.device)
    p = make_moe_params(H=2048, I=1408, E=64, S=2, k=6, seed=3, device=dev)
    layer = MoELayer(ctx, p, max_tokens=max(T, 1))
    x = synth.activations(T, 2048, seed=100 + T).to(dev)
    y = torch.empty((T, 2048), dtype=torch.float32, device=dev)
    for _ in range(reps):
        layer.forward(x, out=y)
    torch.cuda.synchronize()
    layer.close()


def main() -> None:
    ap = argparse.ArgumentParser()
    sub = ap.add_subparsers(dest="case", required=True)
    c = sub.add_parser("chain")
    c.add_argument("--layers", type=int, default=4)
    c.add_argument("--vocab", type=int, default=1024)
    c.add_argument("--reps", type=int, default=5)
    g = sub.add_parser("gemm")
    g.add_argument("M", type=int)
    g.add_argument("K", type=int)
    g.add_argument("N", type=int)
    g.add_argument("--reps", type=int, default=3)
    g.add_argument("--pair", action="store_true")
    h = sub.add_parser("lmhead")
    h.add_argument("vocab", type=int)
    h.add_argument("--shards", type=int, default=1)
    h.add_argument("--reps", type=int, default=3)
    m = sub.add_parser("moe")
    m.add_argument("T", type=int)
    m.add_argument("--reps", type=int, default=3)
    args = ap.parse_args()
    ctx = Context(0)
    if args.case == "chain":
        run_chain(ctx, args.layers, args.vocab, args.reps)
    elif args.case == "gemm":
        run_gemm(ctx, args.M, args.K, args.N, args.reps, args.pair)
    elif args.case == "moe":
        run_moe(ctx, args.T, args.reps)
    else:
        run_lmhead(ctx, args.vocab, args.shards, args.reps)
    torch.cuda.synchronize()
    ctx.check()
    print(f"{args.case}: done")


if __name__ == "__main__":
    main()
