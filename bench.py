"""Decode benchmark of the W8A8 hot path on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--batch T] [--impl ours|reference]
    (N > 1: torchrun --nproc-per-node N ... bench.py --gpus N ...)

One step = one decode step of the Qwen2.5-1.5B-shaped W8A8 workload: 28 layers x
{qkv 1536x2048, o 1536x1536, gate_up 1536x17920, down 8960x1536} (the seven linears, q|k|v and
gate|up fused as shared-input subgraphs) + the 1536x151936 LM head with a fused top-40 /
argmax, vocab-sharded over the N GPUs.  Each GPU decodes its own T tokens (replica of the
linear stack); the LM head shards its vocab across all N GPUs for all N*T tokens.

Prints one JSON line (rank 0).  Besides the headline it carries:
  parity      the measured step (same input) against the oracle's 28-layer step: final hidden
              state bit for bit, top-40 ids and values and the argmax identical (at N > 1 rank 0
              checks its tokens' merged candidates against the whole-vocabulary head);
  per_config  (N = 1) one record per BASELINE configuration with its own CUDA-event time,
              roofline fraction and oracle parity flag: SmolLM-135M T=1, Qwen2.5-1.5B T=8 and
              T=32, the prefill GEMM sweep, the DeepSeek-V2-Lite MoE layer at T=1/64 with its
              102400-row head, Gemma-12B-class T=1 with its 262144-row head;
  lmhead_us   the LM-head tail's cost per step (step minus the same linear stack alone).
`--impl reference` times the reference's CPU path (the C restatement of the NPU integer steps
around the reference's pack/unpack arithmetic, OpenMP over all host cores) on the same workload.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time
from pathlib import Path

import numpy as np
import torch

ROOT = Path(__file__).resolve().parent
METRIC = "decode tok/s & HBM GB/s of W8A8 linear + sharded LM-head argmax, 1/2/4/8 B200"
WORKLOAD = "qwen2.5-1.5b-shaped W8A8 decode: 28 x {qkv,o,gate_up,down} + LM head 1536x151936 top-40"
# DRAM bytes (read + write) per launch of the gate_up GEMV at T=1, from one ncu capture of
# that launch: 27.666688 MB read + 0 B written.
GEMV_TRAFFIC_BYTES = 27666688
# DRAM bytes per algorithmic byte of the chain kernel, from one ncu capture of a 4-layer,
# 1024-vocab chain: 189.84 MB read / 188.7 MB algorithmic.
CHAIN_TRAFFIC_RATIO = 1.006
# DRAM bytes (read + write) of one launch of the M=2048, K=N=8192 tensor-core GEMM, from one ncu
# capture of that launch: 84.005632 MB read + 6.348032 MB written.
PREFILL_GEMM_TRAFFIC_BYTES = 90353664


def env_int(name: str, default: int) -> int:
    try:
        return int(os.environ.get(name, default))
    except ValueError:
        return default


def measured_peaks() -> tuple[float, str]:
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        try:
            return float(json.loads(p.read_text())["hbm_gbs"]), "measured"
        except Exception:
            pass
    return 6650.0, "fallback"


class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled every 200 ms during the timed region."""

    QUERY = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.file = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)
        self.proc = None

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.QUERY}", "--format=csv,noheader,nounits",
                 "-lms", "200", "-i", str(self.gpu)], stdout=self.file, stderr=subprocess.DEVNULL)
        except FileNotFoundError:
            self.proc = None
        time.sleep(0.3)
        return self

    def __exit__(self, *exc):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self) -> dict:
        self.file.flush()
        rows = [ln.split(",") for ln in Path(self.file.name).read_text().splitlines() if ln.strip()]
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for r in rows:
            r = [c.strip() for c in r]
            if len(r) < 9:
                continue
            try:
                sm.append(float(r[1]))
                mx = float(r[2])
            except ValueError:
                continue
            for nm, v in zip(names, r[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(nm)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx,
                "reasons": sorted(reasons), "samples": len(sm)}


# ---------------------------------------------------------------------------- CPU paths
def cpu_model(T: int, layers: int, seed: int = 0):
    """Host-side synthetic model for the CPU arms (generated on the CPU, same shapes)."""
    from romanaccio_b200 import synth
    from romanaccio_b200.quantize import build_linear
    shape = synth.QWEN25_15B
    params = []
    # the DecodeStack recipe: N(0, 1/K) weights, calibration rows propagated through the stack
    calib_h = synth.activations(64, shape.hidden, seed * 7919 + 1)
    for layer in range(layers):
        cal_out = {}
        for j, (name, K, N, trunc) in enumerate(shape.subgraphs()):
            s = seed * 7919 + layer * 16 + j
            g = torch.Generator().manual_seed(s)
            w = torch.randn((N, K), generator=g) / float(K) ** 0.5
            calib = {"qkv": lambda: calib_h, "o": lambda: cal_out["qkv"][:, :shape.q],
                     "gate_up": lambda: cal_out["o"],
                     "down": lambda: cal_out["gate_up"][:, :shape.ffn]}[name]().contiguous()
            params.append((name, build_linear(w, calib, trunc=trunc)))
            cal_out[name] = calib @ w.t()
        calib_h = cal_out["down"]
    K, V = shape.hidden, shape.vocab
    g = torch.Generator().manual_seed(seed + 17)
    w = torch.randn((V, K), generator=g) * 0.02
    step = w.double().abs().amax(dim=1, keepdim=True).clamp(min=1e-12) / 127.0
    wq = torch.clamp(torch.round(w.double() / step), -127, 127).to(torch.int8).numpy()
    from romanaccio_b200.decode import LM_NORM_EPS, lm_input_norm
    in_step, emb = lm_input_norm(K, seed, "cpu", calib=calib_h)
    return params, (wq, (in_step * step[:, 0].numpy()).astype(np.float32), in_step, emb,
                    LM_NORM_EPS)


def decode_step_on(stack, x_host: np.ndarray) -> None:
    """One GPU step on x_host (every rank of a sharded head takes part)."""
    stack.x.copy_(torch.from_numpy(x_host[:stack.T]))
    stack.step()
    torch.cuda.synchronize()


def decode_parity(stack, x_host: np.ndarray, lm=None) -> dict:
    """Checks the stack's last step (run on x_host by decode_step_on) against the oracle's step
    on the same input: the final hidden state (bit for bit), the top-k ids and values
    (identical) and the argmax.  lm: the full-vocabulary LM head (wq, acc_step, in_step,
    emb_norm_scaled, eps) when the stack holds one shard of it."""
    import time as _t
    T = stack.T
    h = stack.outs[3].cpu().numpy()
    val, idx = stack.top_val.cpu().numpy(), stack.top_idx.cpu().numpy()
    ids = stack.ids.cpu().numpy()
    if lm is None:
        lm = stack.lm_oracle()
    t0 = _t.perf_counter()
    from oracle.oracle import DecodeOracle
    orc = DecodeOracle(stack.params_host, lm, T, stack.shape, k=stack.k)
    h_ref, val_ref, idx_ref = orc.run(x_host[:T])
    out = {
        "oracle": "C restatement of the reference path (OpenMP), same weights and input",
        "layers": stack.layers, "tokens": T, "vocab": int(lm[0].shape[0]), "k": stack.k,
        "hidden_equal": bool(np.array_equal(h, h_ref)),
        "hidden_finite": bool(np.isfinite(h_ref).all()),
        "topk_ids_equal": bool(np.array_equal(idx, idx_ref)),
        "topk_values_equal": bool(np.array_equal(val, val_ref)),
        "argmax_equal": bool(np.array_equal(ids, idx_ref[:, 0])),
        # a non-degenerate head: distinct logit values among token 0's top-k
        "topk_distinct_values": int(len(np.unique(val_ref[0]))),
        "oracle_s": round(_t.perf_counter() - t0, 2),
    }
    out["parity"] = (out["hidden_equal"] and out["hidden_finite"] and out["topk_ids_equal"]
                     and out["topk_values_equal"] and out["argmax_equal"])
    return out


def cpu_step_fn(params, lm, T: int, shape):
    """Returns a closure running one decode step through the OpenMP oracle baseline."""
    from oracle.oracle import DecodeOracle
    orc = DecodeOracle(params, lm, T, shape)
    x0 = np.random.default_rng(0).standard_normal((T, shape.hidden)).astype(np.float32)

    def run():
        return orc.run(x0)[2][:, 0]

    return run, orc.cores


def cpu_model_name() -> str:
    try:
        for ln in Path("/proc/cpuinfo").read_text().splitlines():
            if ln.startswith("model name"):
                return ln.split(":", 1)[1].strip()
    except OSError:
        pass
    return "unknown"


def reference_cpp_available() -> bool:
    sys.path.insert(0, str(ROOT))
    from oracle import oracle as O
    return O.ref_available()


def reference_cpp_baseline(params, lm, T: int, shape, seconds: float) -> dict | None:
    """The decode step through the reference's own C++ where it has CPU code (oracle.ReferenceDecode:
    its pack / unpack per linear, TransformerSession's host fp32 LM head, Sampler::sample
    greedy; the NPU GEMM + requant in between is the C restatement), timed for about `seconds`
    on every host core this process may use.  None when the reference C++ is not built."""
    if T != 1 or not reference_cpp_available():
        return None
    from oracle.oracle import ReferenceDecode
    wq, acc_step, in_step = lm[:3]
    w_f32 = (wq.astype(np.float32) * (acc_step / np.float32(in_step))[:, None]).astype(np.float32)
    rd = ReferenceDecode(params, w_f32, T, shape)
    del w_f32
    x0 = np.random.default_rng(0).standard_normal((T, shape.hidden)).astype(np.float32)
    rd.run(x0)
    for key in rd.seconds:
        rd.seconds[key] = 0.0
    n, t0 = 0, time.perf_counter()
    while time.perf_counter() - t0 < seconds or n < 2:
        rd.run(x0)
        n += 1
    dt = (time.perf_counter() - t0) / n
    out = {"value": T / dt, "unit": "tok/s", "cores": rd.cores, "kind": "reference",
           "cpu_model": cpu_model_name(),
           "sample": f"{n} full decode steps: the reference's pack_npu_input_int8_dyntok / "
                     "unpack_npu_output_int8_dyntok around each linear's int8 GEMM + QuantM "
                     "requant (the NPU step: C restatement, OpenMP), TransformerSession's host "
                     "fp32 LM head over 151936 rows and Sampler::sample (greedy), compiled from "
                     "the reference sources",
           "ms_per_step_by_piece": {k: round(v / n * 1e3, 3) for k, v in rd.seconds.items()}}
    rd.close()
    return out


def run_reference(args) -> None:
    rank = env_int("RANK", 0)
    if rank != 0:
        return
    from romanaccio_b200 import synth
    T = args.batch
    shape = synth.QWEN25_15B
    params, lm = cpu_model(T, shape.layers)
    if T == 1 and reference_cpp_available():
        # the reference's own C++ where it has CPU code for the path (see ReferenceDecode)
        from oracle.oracle import ReferenceDecode
        wq, acc_step, in_step = lm
        w_f32 = (wq.astype(np.float32) * (acc_step / np.float32(in_step))[:, None]).astype(np.float32)
        rd = ReferenceDecode(params, w_f32, T, shape)
        del w_f32
        x0 = np.random.default_rng(0).standard_normal((T, shape.hidden)).astype(np.float32)

        def run():
            return rd.run(x0)

        cores, kind = rd.cores, "reference"
        sample = (f"{args.steps} full decode steps: the reference's pack / unpack around each "
                  "linear's int8 GEMM + requant (NPU step: C restatement, OpenMP), "
                  "TransformerSession's host fp32 LM head and Sampler::sample, compiled from the "
                  "reference sources")
    else:
        run, cores = cpu_step_fn(params, lm, T, shape)
        kind = "port"
        sample = (f"{args.steps} full decode steps (all 28 layers + LM head), C restatement of "
                  "the reference path, OpenMP")
    for _ in range(args.warmup):
        run()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        run()
    dt = (time.perf_counter() - t0) / args.steps
    value = T / dt
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": "tok/s",
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": dt * 1e3, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "int8", "data": "synthetic",
        "config": {"workload": WORKLOAD, "batch_per_gpu": T, "layers": synth.QWEN25_15B.layers,
                   "vocab": synth.QWEN25_15B.vocab, "parallelism": "host cores (OpenMP)"},
        "cpu_baseline": {"value": value, "unit": "tok/s", "cores": cores, "kind": kind,
                         "cpu_model": cpu_model_name(), "sample": sample},
        "e2e": {"value": value, "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# ---------------------------------------------------------------------------- per-config records
def time_steps(step, steps: int, warmup: int, flush: torch.Tensor | None = None) -> float:
    """Mean device time (CUDA events on the current stream) of `steps` calls of step(), after
    `warmup` untimed ones; with flush, a buffer larger than L2 is rewritten before every step,
    outside the events."""
    stream = torch.cuda.current_stream()
    for _ in range(warmup):
        step()
    torch.cuda.synchronize()
    evs = []
    for _ in range(steps):
        if flush is not None:
            flush.add_(1)
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record(stream)
        step()
        b.record(stream)
        evs.append((a, b))
    torch.cuda.synchronize()
    return sum(a.elapsed_time(b) for a, b in evs) / steps


def decode_record(name: str, stack, x_host: np.ndarray, steps: int, warmup: int, peak: float,
                  flush: torch.Tensor | None, note: str) -> dict:
    """Timed decode steps (graph replays) of one stack + the oracle check of the same step."""
    stack.x.copy_(torch.from_numpy(x_host[:stack.T]))
    stack.step()
    torch.cuda.synchronize()
    try:
        stack.capture()
    except RuntimeError:
        stack.graph = None
    ms = time_steps(stack.step, steps, warmup, flush)
    sb = stack.step_bytes()
    nbytes = sb.linear + sb.lm_head
    rec = {"workload": name, "tokens_per_step": stack.T, "layers": stack.layers,
           "vocab": stack.V, "steps": steps, "ms_per_step": round(ms, 4),
           "tok_s": round(stack.T / (ms / 1e3), 1),
           "kernel": ("persistent chain (linears" + (" + LM head" if stack.chain_lm else "")
                      + "), 1 launch" if stack.chain is not None
                      else "act_quant + tcgen05 GEMM per linear"),
           "roofline": {"bound": "hbm", "algorithmic_bytes": nbytes,
                        "achieved_gbs": round(nbytes / (ms / 1e3) / 1e9, 1), "peak_gbs": peak,
                        "frac": round(nbytes / (ms / 1e3) / 1e9 / peak, 4)},
           "l2": note}
    decode_step_on(stack, x_host)
    par = decode_parity(stack, x_host)
    rec["parity"] = par.pop("parity")
    rec["parity_detail"] = par
    stack.release()
    return rec


def moe_record(ctx, dev, steps: int, warmup: int, peak: float, flush: torch.Tensor) -> dict:
    """Config 3: one DeepSeek-V2-Lite-shaped W8A8 MoE decode layer (hidden 2048, 64 routed + 2
    shared experts of 1408, top-6) at T = 1 and 64, and its 2048 x 102400 LM head (top-40),
    on one GPU; oracle-checked routing, expert stages and combine."""
    sys.path.insert(0, str(ROOT))
    from oracle import oracle as O
    from romanaccio_b200 import LmHeadShard, synth
    from romanaccio_b200.moe import MoELayer, make_moe_params
    H, I, E, S, k = 2048, 1408, 64, 2, 6
    p = make_moe_params(H=H, I=I, E=E, S=S, k=k, seed=3, device=dev)
    layer = MoELayer(ctx, p, max_tokens=64)
    expert_bytes = 2 * I * H + H * I
    out = {"workload": "deepseek-v2-lite-shaped W8A8 MoE layer: hidden 2048, 64 routed + 2 "
                       "shared experts (gate|up 2048x2816, down 1408x2048), top-6",
           "l2": "256 MB rewritten before every timed step (a layer's active experts fit in L2)"}
    ok_all = True
    for T in (1, 64):
        x = synth.activations(T, H, seed=100 + T)
        xd = x.to(dev)
        y = torch.empty((T, H), dtype=torch.float32, device=dev)
        ms = time_steps(lambda: layer.forward(xd, out=y), steps, warmup, flush)
        v = {kk: t.cpu().numpy() for kk, t in layer.views(T).items()}
        active = len(set(v["idx"].reshape(-1).tolist())) + S
        nbytes = active * expert_bytes + T * H * 4 * 2
        # oracle: routing ids identical, weights within float rounding of the logit sum order,
        # every expert stage bit-exact on a sample of (token, slot) pairs, combine bit-exact
        xh = x.numpy()
        idx, w = O.moe_route(xh, p.gate_w, k)
        ids_ok = bool(np.array_equal(v["idx"], idx))
        w_ok = bool(np.allclose(v["w"], w, rtol=1e-4, atol=0))
        slots = k + S
        rng = np.random.default_rng(T)
        pairs = range(T * slots) if T * slots <= 16 else sorted(rng.choice(T * slots, 16, replace=False).tolist())
        stage_ok = True
        for pi in pairs:
            t, j = divmod(pi, slots)
            e = int(v["idx"][t, j]) if j < k else E + (j - k)
            gu, dn = p.gu[e], p.dn[e]
            q, r = O.pack_dyntok(xh[t:t + 1], gu.in_thresh, gu.in_inv_smooth)
            yq = O.requant(O.gemm_i32(q, gu.wq), gu.quant_m, gu.trunc, 127)
            stage_ok &= bool(np.array_equal(v["gate_up"][pi:pi + 1], O.unpack(yq, 0.0, gu.out_step_chan, r)))
            q2 = O.pack_static(v["act"][pi:pi + 1], dn.in_step, dn.in_inv_smooth)
            want = O.requant(O.gemm_i32(q2, dn.wq), dn.quant_m, dn.trunc, 127)
            stage_ok &= bool(np.array_equal(v["down_q"][pi:pi + 1].astype(np.int32), want))
        osc = np.stack([q.out_step_chan for q in p.dn])
        comb = O.moe_combine(v["down_q"].astype(np.int32), v["idx"], v["w"], osc, E, slots)
        comb_ok = bool(np.array_equal(layer.forward(xd).cpu().numpy(), comb))
        par = ids_ok and w_ok and stage_ok and comb_ok
        ok_all &= par
        out[f"T{T}"] = {"ms_per_layer": round(ms, 4), "tok_s_per_layer": round(T / (ms / 1e3), 1),
                        "active_experts": active,
                        "roofline": {"bound": "hbm", "algorithmic_bytes": nbytes,
                                     "achieved_gbs": round(nbytes / (ms / 1e3) / 1e9, 1),
                                     "peak_gbs": peak,
                                     "frac": round(nbytes / (ms / 1e3) / 1e9 / peak, 4)},
                        "parity": par,
                        "parity_detail": {"expert_ids_equal": ids_ok, "weights_rel_1e-4": w_ok,
                                          "sampled_pairs": len(pairs), "stages_bit_exact": stage_ok,
                                          "combine_bit_exact": comb_ok}}
    layer.close()
    # the 2048 x 102400 LM head with the fused top-40 (one shard at N = 1)
    K, V = synth.DEEPSEEK_V2_LITE_LMHEAD
    from romanaccio_b200.decode import _lm_rows
    wq, w_step = _lm_rows(K, 0, V, 31, dev)
    in_step = float(synth.activations(64, K, 37).abs().max()) / 127.0
    acc_step = (in_step * w_step).astype(np.float32)
    shard = LmHeadShard(ctx, wq, acc_step, in_step, row_offset=0)
    h = synth.activations(1, K, seed=41)
    hd = h.to(dev)
    val = torch.empty((1, 40), dtype=torch.float32, device=dev)
    idx = torch.empty((1, 40), dtype=torch.int32, device=dev)
    ms = time_steps(lambda: shard.forward(hd, 40, val=val, idx=idx), steps, warmup, flush)
    lg = O.dequant_acc(O.gemm_i32(O.pack_static(h.numpy(), in_step), wq), acc_step)
    wv, wi = O.topk(lg, 40)
    lm_ok = bool(np.array_equal(idx.cpu().numpy(), wi) and np.array_equal(val.cpu().numpy(), wv))
    ok_all &= lm_ok
    nbytes = V * K + K * 4 + V * 4 + 40 * 8
    out["lm_head_2048x102400"] = {"ms": round(ms, 4),
                                  "roofline": {"bound": "hbm", "algorithmic_bytes": nbytes,
                                               "achieved_gbs": round(nbytes / (ms / 1e3) / 1e9, 1),
                                               "peak_gbs": peak,
                                               "frac": round(nbytes / (ms / 1e3) / 1e9 / peak, 4)},
                                  "parity": lm_ok}
    out["parity"] = ok_all
    return out


def moe_ep_record(ctx, dev, rank: int, world: int, steps: int, warmup: int, peak: float) -> dict:
    """Config 3 at N > 1: the DeepSeek-V2-Lite-shaped MoE layer expert-parallel over the `world`
    ranks (experts e % world == rank, the library's peer-store exchange of the partial combines,
    ordered sum), T = 1 and 64 tokens (the same tokens on every rank), device time max over
    ranks; rank 0 checks the output against the oracle's expert-parallel combine of every rank's
    requantised expert outputs (gathered after the timing, for the check only)."""
    import torch.distributed as dist
    sys.path.insert(0, str(ROOT))
    from romanaccio_b200 import synth
    from romanaccio_b200.moe import ExpertParallelMoE, MoELayer, make_moe_params
    H, I, E, S, k = 2048, 1408, 64, 2, 6
    p = make_moe_params(H=H, I=I, E=E, S=S, k=k, seed=3, device=dev)
    layer = MoELayer(ctx, p, max_tokens=64)
    ep = ExpertParallelMoE(layer, rank, world)
    handles = [None] * world
    dist.all_gather_object(handles, ep.export())
    ep.connect(handles)
    expert_bytes = 2 * I * H + H * I
    out = {"workload": "deepseek-v2-lite-shaped W8A8 MoE layer, expert-parallel over "
                       f"{world} GPUs (experts e % {world} == rank, partials exchanged by peer "
                       "stores and summed in rank order)"}
    ok_all = True
    for T in (1, 64):
        x = synth.activations(T, H, seed=100 + T)
        xd = x.to(dev)
        y = torch.empty((T, H), dtype=torch.float32, device=dev)
        dist.barrier()
        ms = time_steps(lambda: ep.forward(xd, out=y), steps, warmup)
        t = torch.tensor([ms], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
        ep.forward(xd, out=y)
        torch.cuda.synchronize()
        v = {kk: tt.cpu().numpy() for kk, tt in layer.views(T).items()}
        parts = [None] * world
        dist.all_gather_object(parts, {"down_q": v["down_q"], "idx": v["idx"]})
        rec = {"ms_per_layer": round(ms, 4)}
        if rank == 0:
            from oracle import oracle as O
            slots = k + S
            yq = np.zeros_like(v["down_q"]).astype(np.int32)
            for pi in range(T * slots):
                tt_, j = divmod(pi, slots)
                e = int(v["idx"][tt_, j]) if j < k else E + (j - k)
                yq[pi] = parts[e % world]["down_q"][pi]
            osc = np.stack([q.out_step_chan for q in p.dn])
            want = O.moe_combine_ep(yq, v["idx"], v["w"], osc, E, slots, world)
            idx_ref, _ = O.moe_route(x.numpy(), p.gate_w, k)
            par = bool(np.array_equal(y.cpu().numpy(), want) and np.array_equal(v["idx"], idx_ref)
                       and all(np.array_equal(q["idx"], v["idx"]) for q in parts))
            ok_all &= par
            active = len(set(v["idx"].reshape(-1).tolist())) + S
            nbytes = active * expert_bytes
            rec.update({"tok_s_per_layer": round(T / (ms / 1e3), 1), "active_experts": active,
                        "roofline": {"bound": "hbm", "algorithmic_bytes": nbytes,
                                     "note": "weights of the active experts over all ranks",
                                     "achieved_gbs": round(nbytes / (ms / 1e3) / 1e9, 1),
                                     "peak_gbs": peak * world,
                                     "frac": round(nbytes / (ms / 1e3) / 1e9 / (peak * world), 4)},
                        "parity": par})
        out[f"T{T}"] = rec
        dist.barrier()
    ep.close()
    layer.close()
    out["parity"] = ok_all
    return out


def per_config_records(ctx, dev, headline, args, peak: float) -> dict:
    """Untimed against the headline: one record per BASELINE configuration (decode configs 0, 1
    at T = 8 and 32, 3 and 4, the prefill sweep of config 2), each with its own CUDA-event time,
    roofline fraction and oracle parity flag."""
    from romanaccio_b200 import synth
    from romanaccio_b200.decode import DecodeStack
    steps, warmup = args.config_steps, 3
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
    rng = np.random.default_rng(7)
    recs = {}

    def guarded(key, fn):
        t0 = time.perf_counter()
        try:
            recs[key] = fn()
        except Exception as e:  # a failing configuration is reported, not hidden
            recs[key] = {"error": f"{type(e).__name__}: {str(e).splitlines()[0][:200]}",
                         "parity": False}
        recs[key]["wall_s"] = round(time.perf_counter() - t0, 1)
        torch.cuda.empty_cache()

    def c0():
        sh = synth.SMOLLM_135M
        st = DecodeStack(ctx, sh, 1, seed=0, stat="max", clamp=None)
        x = synth.activations(1, sh.hidden, seed=11).numpy()
        r = decode_record("smollm-135m-shaped W8A8 decode T=1 (30 layers, LM head 576x49152, "
                          "smoothing sqrt(max|X|/max|W|), no clamp)", st, x, steps, warmup, peak,
                          flush, "model 134 MB: 256 MB rewritten before every timed step")
        del st
        return r

    def c1(T):
        def f():
            st = DecodeStack(ctx, synth.QWEN25_15B, T, seed=0, share_from=headline)
            x = rng.standard_normal((T, synth.QWEN25_15B.hidden)).astype(np.float32)
            r = decode_record(f"qwen2.5-1.5b-shaped W8A8 decode T={T}", st, x, steps, warmup,
                              peak, None, "weights streamed every step: 1.54 GB > L2")
            del st
            return r
        return f

    def c4():
        # T = 1 (the persistent chain), then T = 16 and 64 (tensor-core linears) over the same
        # weights; one record per batch
        sh = synth.GEMMA_12B
        st = DecodeStack(ctx, sh, 1, seed=0)
        x = synth.activations(64, sh.hidden, seed=13).numpy()
        out = {}
        out["T1"] = decode_record("gemma-12b-class W8A8 decode T=1 (48 layers, LM head 3840x262144)",
                                  st, x[:1], steps, warmup, peak, None,
                                  "weights streamed every step: 11.8 GB > L2")
        for T in (16, 64):
            sub = DecodeStack(ctx, sh, T, seed=0, share_from=st)
            out[f"T{T}"] = decode_record(
                f"gemma-12b-class W8A8 decode T={T} (48 layers, LM head 3840x262144)", sub,
                x[:T], max(3, steps // 2), warmup, peak, None,
                "weights streamed every step: 11.8 GB > L2")
            sub.release()
            del sub
        del st
        # the T = 1 figures at the top level, as before
        r = dict(out["T1"])
        r["T16"], r["T64"] = out["T16"], out["T64"]
        r["parity"] = all(v.get("parity", False) for v in out.values())
        return r

    guarded("c0_smollm_t1", c0)
    guarded("c1_qwen_t8", c1(8))
    guarded("c1_qwen_t32", c1(32))
    guarded("c2_prefill_sweep", lambda: prefill_record(ctx, dev, steps, warmup, flush))
    guarded("c3_moe_v2lite", lambda: moe_record(ctx, dev, steps, warmup, peak, flush))
    guarded("c4_gemma_t1", c4)
    guarded("lmhead_sharded", lambda: sharded_head_record(1, steps, warmup))
    recs["all_parity"] = all(r.get("parity", False) for k, r in recs.items() if isinstance(r, dict))
    return recs


# ------------------------------------------------------------- sharded LM head (strong scaling)
def sharded_head_record(n: int, steps: int, warmup: int) -> dict:
    """One token's Qwen2.5-1.5B LM head (1536 x 151936, top-40 + argmax) vocab-sharded over GPUs
    0 .. n-1 by this one process (w8a8_lmhead_*): the reference's dual-die LM-head split, every
    shard streaming V / n rows of the same token.  Latency: CUDA events on GPU 0 from "h ready"
    (after a ~100 us GPU delay standing in for the layers, during which the host issues the
    forward) to the argmax ids in pinned host memory; e2e: the same with GPU 0 idle before it (the
    host's launches on the clock).  L2 flushed on every GPU before every step.  Parity: top-40 ids
    and values and the argmax against the oracle's head on the same weights and input."""
    sys.path.insert(0, str(ROOT))
    from oracle import oracle as O
    from romanaccio_b200 import Context, MultiDeviceLmHead, synth
    K, V, k, T = synth.QWEN25_15B.hidden, synth.QWEN25_15B.vocab, 40, 1
    rng = np.random.default_rng(17)
    wq = rng.integers(-127, 128, size=(V, K), dtype=np.int16).astype(np.int8)
    w_step = (rng.random(V) * 0.02 / 127 + 1e-5)
    in_step = float(synth.activations(64, K, 23).abs().max()) / 127.0
    acc_step = (in_step * w_step).astype(np.float32)
    h_host = synth.activations(T, K, seed=5)
    ctxs = [Context(d) for d in range(n)]
    torch.cuda.set_device(0)
    h = h_host.cuda()
    ids_host = torch.empty((T,), dtype=torch.int32).pin_memory()
    flush = [torch.empty(256 << 20, dtype=torch.uint8, device=f"cuda:{d}") for d in range(n)]
    stream = torch.cuda.current_stream()
    lm = MultiDeviceLmHead(ctxs, wq, acc_step, in_step, max_tokens=8, k_max=k)
    val = torch.empty((T, k), dtype=torch.float32, device="cuda")
    idx = torch.empty((T, k), dtype=torch.int32, device="cuda")

    def step(delay: bool) -> float:
        for f in flush:
            f.fill_(1)
        if delay:
            torch.cuda._sleep(200_000)  # ~100 us at 1.9 GHz
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record(stream)
        lm.forward(h, k, val, idx, ids_host)
        b.record(stream)
        b.synchronize()
        return a.elapsed_time(b) * 1e3

    for _ in range(warmup):
        step(True)
    lat = [step(True) for _ in range(steps)]
    e2e = [step(False) for _ in range(steps)]
    for d in range(n):
        torch.cuda.synchronize(d)
    for c in ctxs:
        c.check()
    q = O.pack_static(h_host.numpy(), in_step)
    want_v, want_i = O.topk(O.dequant_acc(O.gemm_i32(q, wq), acc_step), k)
    ids_ok = bool(np.array_equal(idx.cpu().numpy(), want_i))
    vals_ok = bool(np.array_equal(val.cpu().numpy(), want_v))
    arg_ok = bool(np.array_equal(ids_host.numpy(), want_i[:, 0]))
    del lm, flush
    return {"workload": f"LM head {K}x{V} top-{k} + argmax, one token, vocab-sharded over {n} GPU(s) "
                        "(w8a8_lmhead_*, one process)",
            "n_gpus": n, "steps": steps, "latency_us": round(statistics.median(lat), 2),
            "latency_us_min": round(min(lat), 2), "e2e_us": round(statistics.median(e2e), 2),
            "bytes_per_gpu": (V // n) * K, "l2": "256 MB written on every GPU before every step",
            "parity": ids_ok and vals_ok and arg_ok,
            "parity_detail": {"topk_ids_equal": ids_ok, "topk_values_equal": vals_ok,
                              "argmax_equal": arg_ok}}


# ---------------------------------------------------------------------------- GPU path
def run_ours(args) -> None:
    world = env_int("WORLD_SIZE", 1)
    rank = env_int("RANK", 0)
    local = env_int("LOCAL_RANK", 0)
    if world != args.gpus:
        raise SystemExit(f"--gpus {args.gpus} but WORLD_SIZE={world}")
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    group = None
    if world > 1:
        import datetime
        import torch.distributed as dist
        dist.init_process_group("nccl", device_id=dev, timeout=datetime.timedelta(seconds=300))
    sys.path.insert(0, str(ROOT))
    from romanaccio_b200 import Context, synth
    from romanaccio_b200.decode import DecodeStack, _lm_rows

    T = args.batch
    shape = synth.QWEN25_15B
    ctx = Context(local)
    stack = DecodeStack(ctx, shape, T, rank=rank, world=world, group=group, seed=0,
                        layers=args.layers, use_chain=not args.per_linear)
    x_np = np.random.default_rng(rank).standard_normal((T, shape.hidden)).astype(np.float32)
    x_host = torch.from_numpy(x_np).pin_memory()
    ids_host = torch.empty((T,), dtype=torch.int32).pin_memory()
    stack.x.copy_(x_host)
    stack.step()  # eager warm-up (configures every kernel instantiation)
    torch.cuda.synchronize()
    graph_note = True
    try:
        stack.capture()
        # the end-to-end step (pinned host input copied in, ids copied out) as one graph too
        stack.capture_host(x_host, ids_host)
    except RuntimeError as e:  # a launch the graph cannot hold: run the step eagerly
        graph_note = f"eager ({str(e).splitlines()[0][:80]})"
        stack.graph = None
        stack.host_graph = None
        torch.cuda.synchronize()
    stream = torch.cuda.current_stream()

    def barrier():
        if world > 1:
            import torch.distributed as dist
            dist.barrier()
        torch.cuda.synchronize()

    for _ in range(args.warmup):
        stack.step()
    barrier()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clocks:
        barrier()
        ev0.record(stream)
        for _ in range(args.steps):
            stack.step()
        ev1.record(stream)
        barrier()
    ms = ev0.elapsed_time(ev1) / args.steps
    # end to end: pinned host input -> step -> sampled ids read back on the host, every step
    barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(args.steps):
        stack.step_host(x_host, ids_host)
        stream.synchronize()
    e1.record(stream)
    barrier()
    ms_e2e = e0.elapsed_time(e1) / args.steps

    # the LM-head tail's cost per step: the step against the same linear stack alone (a chain
    # without the head, or the per-linear launches), both as CUDA graphs
    reps = 10
    if stack.chain is not None:
        lin_only = stack.chain if not stack.chain_lm else stack._build_chain(with_lm=False)
        run_lin = lin_only.forward
    else:
        run_lin = stack.run_linears
    run_lin()
    torch.cuda.synchronize()
    g_lin = torch.cuda.CUDAGraph()
    s_cap = torch.cuda.Stream(device=dev)
    s_cap.wait_stream(stream)
    with torch.cuda.stream(s_cap):
        run_lin()
    stream.wait_stream(s_cap)
    torch.cuda.synchronize()
    with torch.cuda.graph(g_lin):
        run_lin()
    for _ in range(3):
        g_lin.replay()
    torch.cuda.synchronize()
    l0, l1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    l0.record(stream)
    for _ in range(reps):
        g_lin.replay()
    l1.record(stream)
    torch.cuda.synchronize()
    ms_lin = l0.elapsed_time(l1) / reps
    del g_lin
    times = torch.tensor([ms, ms_e2e, ms_lin], dtype=torch.float64, device=dev)
    if world > 1:
        import torch.distributed as dist
        dist.all_reduce(times, op=dist.ReduceOp.MAX)
    ms, ms_e2e, ms_lin = times.tolist()

    # dominant kernel: the gate_up GEMV (59 % of the linear weight bytes), int8 input in HBM,
    # one launch per layer over the 28 distinct weight matrices (770 MB > L2), in a graph.
    sb = stack.step_bytes()
    gu = [row[2] for row in stack.linears]
    q_in = torch.zeros((T, shape.hidden), dtype=torch.int8, device=dev)
    y_out = torch.empty((T, 2 * shape.ffn), dtype=torch.float32, device=dev)
    from romanaccio_b200 import OUT_F32
    ratio = torch.ones((T,), dtype=torch.float32, device=dev)
    s = torch.cuda.Stream(device=dev)
    with torch.cuda.stream(s):
        for lin in gu:
            lin.submit(q_in, OUT_F32, dyntok_ratios=ratio, out=y_out)
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        for lin in gu:
            lin.submit(q_in, OUT_F32, dyntok_ratios=ratio, out=y_out)
    for _ in range(3):
        g.replay()
    torch.cuda.synchronize()
    r0, r1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    r0.record(stream)
    for _ in range(reps):
        g.replay()
    r1.record(stream)
    torch.cuda.synchronize()
    gemv_s = r0.elapsed_time(r1) / 1e3 / (reps * len(gu))
    del g
    peak, peak_kind = measured_peaks()
    gemv_achieved = sb.gemv_launch / gemv_s / 1e9
    gemv_roof = {"kernel": "gemv_w8a8 gate_up 1536x17920 T=%d (standalone launches)" % T,
                 "achieved": gemv_achieved, "frac": gemv_achieved / peak,
                 "launch_us": gemv_s * 1e6, "algorithmic_bytes": sb.gemv_launch,
                 "traffic": GEMV_TRAFFIC_BYTES}
    if stack.chain is not None:
        # dominant kernel of the step: the persistent chain kernel; one launch moves the step's
        # algorithmic bytes (linears, plus the LM head when it runs inside the chain)
        chain_bytes = sb.linear + (sb.lm_head if stack.chain_lm else 0)
        for _ in range(3):
            stack.chain.forward()
        torch.cuda.synchronize()
        c0, c1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        c0.record(stream)
        for _ in range(reps):
            stack.chain.forward()
        c1.record(stream)
        torch.cuda.synchronize()
        chain_s = c0.elapsed_time(c1) / 1e3 / reps
        roof_kernel = "chain_kernel (whole decode step, 1 launch)"
        roof_bytes, roof_s = chain_bytes, chain_s
        roof_traffic = int(chain_bytes * CHAIN_TRAFFIC_RATIO) if CHAIN_TRAFFIC_RATIO else None
    else:
        roof_kernel = gemv_roof["kernel"]
        roof_bytes, roof_s, roof_traffic = sb.gemv_launch, gemv_s, GEMV_TRAFFIC_BYTES
    achieved = roof_bytes / roof_s / 1e9

    # oracle parity of the measured step (rank 0: its own tokens against the oracle's step with
    # the whole vocabulary; every rank holds the same linear weights)
    parity = None
    if not args.no_parity:
        decode_step_on(stack, x_np)
    if rank == 0 and not args.no_parity:
        lm_full = None
        if world > 1:
            wq_f, w_step_f = _lm_rows(shape.hidden, 0, stack.V, 17, dev)
            lm_full = (wq_f, (stack.lm_in_step * w_step_f).astype(np.float32), stack.lm_in_step,
                       stack.lm_norm[0], stack.lm_norm[1])
        parity = decode_parity(stack, x_np, lm=lm_full)
    barrier()

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu:
        run_cpu, cores = cpu_step_fn(stack.params_host, stack.lm_oracle(), T, shape)
        run_cpu()
        n, t0 = 0, time.perf_counter()
        while True:
            run_cpu()
            n += 1
            if time.perf_counter() - t0 > args.cpu_seconds:
                break
        dt = (time.perf_counter() - t0) / n
        cpu = {"value": T / dt, "unit": "tok/s", "cores": cores, "kind": "port",
               "cpu_model": cpu_model_name(),
               "sample": f"{n} full decode steps of the same workload (28 layers + LM head), "
                         "C restatement of the reference path, OpenMP"}
        ref_cpp = reference_cpp_baseline(stack.params_host, stack.lm_oracle(), T, shape,
                                         args.cpu_seconds)
        if ref_cpp is not None:
            cpu["reference_cpp"] = ref_cpp

    per_config = None
    if rank == 0 and world == 1 and not args.no_per_config:
        per_config = per_config_records(ctx, dev, stack, args, peak)
    if world > 1 and not args.no_per_config:
        # every rank takes part in the expert-parallel layer; rank 0 reports it
        rec = moe_ep_record(ctx, dev, rank, world, args.config_steps, 3, peak)
        per_config = {"c3_moe_v2lite_ep": rec}
        # one token's LM head over all N GPUs (strong scaling): rank 0 drives every GPU while the
        # other ranks wait at a host (gloo) barrier, launching nothing
        import torch.distributed as dist
        cpu_group = dist.new_group(backend="gloo")
        torch.cuda.synchronize()
        dist.barrier(group=cpu_group)
        if rank == 0:
            t0 = time.perf_counter()
            try:
                rec = sharded_head_record(world, args.config_steps, 3)
            except Exception as e:  # reported, not hidden
                rec = {"error": f"{type(e).__name__}: {str(e).splitlines()[0][:200]}",
                       "parity": False}
            rec["wall_s"] = round(time.perf_counter() - t0, 1)
            per_config["lmhead_sharded"] = rec
            torch.cuda.set_device(local)
        dist.barrier(group=cpu_group)
        if per_config is not None:
            per_config["all_parity"] = all(r.get("parity", False) for r in per_config.values()
                                           if isinstance(r, dict))

    step_bytes = sb.linear + sb.lm_head
    value = world * T / (ms / 1e3)
    launches_per_step = stack.launches_per_step()
    if rank == 0:
        line = {
            "metric": METRIC, "value": value, "unit": "tok/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "int8",
            "data": "synthetic",
            "config": {"workload": WORKLOAD, "batch_per_gpu": T, "layers": stack.layers,
                       "vocab": shape.vocab, "lm_head_shards": world,
                       "parallelism": f"linears replicated per GPU, LM head vocab-sharded x{world}",
                       "l2": f"weights streamed every step: {step_bytes / 1e9:.2f} GB per GPU > 126 MB L2",
                       "cuda_graph": graph_note,
                       "kernel": "per-linear GEMV launches" if args.per_linear else
                                 "persistent decode-chain kernel (1 cooperative launch per step)"},
            "hbm_gbs_step": step_bytes / (ms / 1e3) / 1e9,
            "lmhead_us": round((ms - ms_lin) * 1e3, 2),
            "linears_ms": round(ms_lin, 4),
            "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                         "frac": achieved / peak, "traffic": roof_traffic,
                         "kernel": roof_kernel, "peak_kind": peak_kind,
                         "launch_us": roof_s * 1e6, "algorithmic_bytes": roof_bytes,
                         "secondary": gemv_roof},
            "e2e": {"value": world * T / (ms_e2e / 1e3), "unit": "tok/s",
                    "h2d_bytes_per_step": T * shape.hidden * 4, "d2h_bytes_per_step": T * 4,
                    "path": "every step: the pinned host activations copied in, the step, the "
                            "sampled ids copied out (one CUDA graph), then a host synchronise"},
            "gpu_launches": launches_per_step * args.steps,
            "clocks": clocks.summary(),
        }
        if parity is not None:
            line["parity"] = parity
        if cpu is not None:
            line["cpu_baseline"] = cpu
        if per_config is not None:
            line["per_config"] = per_config
        print(json.dumps(line), flush=True)
    stack.release()
    if world > 1:
        import torch.distributed as dist
        dist.barrier()
        dist.destroy_process_group()


# ---------------------------------------------------------------------------- prefill sweep
PREFILL_METRIC = "prefill int8 GEMM TOPS (W8A8 linear: dyntok act quant + int8 GEMM + int8 requant)"
PREFILL_SHAPES = [(m, k, n) for m in (128, 512, 2048)
                  for (k, n) in ((2048, 2048), (8192, 8192), (2048, 8192), (8192, 2048))]
PREFILL_WORKLOAD = ("prefill sweep: M in {128,512,2048} x (K,N) in {(2048,2048),(8192,8192),"
                    "(2048,8192),(8192,2048)}, SmoothQuant W8A8, per-channel requant to int8")


def prefill_ops(shapes) -> int:
    return sum(2 * m * n * k for (m, k, n) in shapes)


def cpu_prefill_fn(shapes, seed: int = 0):
    """OpenMP oracle linear (dyntok pack + int32 GEMM + QuantM requant + dequant) over shapes."""
    sys.path.insert(0, str(ROOT))
    from oracle import oracle as O
    from romanaccio_b200 import synth
    lib = O.lib()
    lib.orc_set_threads(len(os.sched_getaffinity(0)))
    import ctypes as C
    jobs = []
    for i, (M, K, N) in enumerate(shapes):
        p = synth.make_linear(K, N, seed=seed + i)
        x = synth.activations(M, K, seed=seed + 100 + i).numpy()
        jobs.append((M, K, N, x, np.ascontiguousarray(p.wq), p.in_inv_smooth.astype(np.float32),
                     p.in_thresh, p.quant_m, p.trunc, p.out_step_chan.astype(np.float32),
                     np.empty((M, N), np.float32), np.empty((M, K), np.int8),
                     np.empty(M, np.float32)))

    def run():
        for (M, K, N, x, wq, inv, thr, qm, tr, osc, y, q, r) in jobs:
            lib.orc_linear_dyntok_omp(x.ctypes.data, M, K, N, wq.ctypes.data, inv.ctypes.data,
                                      C.c_float(thr), qm.ctypes.data, tr, osc.ctypes.data,
                                      y.ctypes.data, q.ctypes.data, r.ctypes.data)

    return run, int(lib.orc_num_threads())


def run_prefill_reference(args) -> None:
    if env_int("RANK", 0) != 0:
        return
    sample = [s for s in PREFILL_SHAPES if s[0] == 128]  # bounded sample: the M=128 row
    run, cores = cpu_prefill_fn(sample)
    for _ in range(args.warmup):
        run()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        run()
    dt = (time.perf_counter() - t0) / args.steps
    value = prefill_ops(sample) / dt / 1e12
    line = {
        "impl": "reference", "metric": PREFILL_METRIC, "value": value, "unit": "TOPS",
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": dt * 1e3, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "int8", "data": "synthetic",
        "config": {"workload": PREFILL_WORKLOAD, "parallelism": "host cores (OpenMP)"},
        "cpu_baseline": {"value": value, "unit": "TOPS", "cores": cores, "kind": "port",
                         "sample": "the four M=128 GEMMs of the sweep per step, C restatement "
                                   "of the reference linear, OpenMP"},
        "e2e": {"value": value, "unit": "TOPS", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def prefill_record(ctx, dev, steps: int, warmup: int, flush: torch.Tensor) -> dict:
    """Config 2: the 12 prefill linears, each a fused W8A8 forward (dyntok act quant kernel +
    tcgen05 GEMM with the requant epilogue) on a cold L2, timed per shape; every shape checked
    against the oracle on 16 seeded token rows (rows are independent: per-token ratio, per-row
    requant), int8 outputs bit for bit."""
    sys.path.insert(0, str(ROOT))
    from oracle import oracle as O
    from romanaccio_b200 import OUT_QUANT, PATH_TENSOR, W8A8Linear, synth
    stream = torch.cuda.current_stream()
    per, ok_all, tot_ms = {}, True, 0.0
    for i, (M, K, N) in enumerate(PREFILL_SHAPES):
        prm = synth.make_linear(K, N, seed=i, device=dev)
        lin = W8A8Linear.from_params(ctx, prm)
        lin.set_path(PATH_TENSOR)
        x = synth.activations(M, K, seed=100 + i, device=dev)
        y = torch.empty((M, N), dtype=torch.int8, device=dev)
        ms = time_steps(lambda: lin.forward(x, OUT_QUANT, dyntok=True, out=y), steps, warmup, flush)
        # the tensor-core GEMM alone (its int8 input and ratios already in HBM, same L2 flush):
        # the kernel's own roofline figure
        qx = lin.pack_npu_input(x, dyntok_ratios=torch.zeros(M, dtype=torch.float32, device=dev))
        ms_gemm = time_steps(lambda: lin.submit(qx, OUT_QUANT, out=y), steps, warmup, flush)
        del qx
        lin.forward(x, OUT_QUANT, dyntok=True, out=y)
        rows = np.sort(np.random.default_rng(i).choice(M, 16, replace=False))
        xr = x[torch.as_tensor(rows, device=dev)].cpu().numpy()
        q, r = O.pack_dyntok(xr, prm.in_thresh, prm.in_inv_smooth)
        want = O.requant(O.gemm_i32(q, prm.wq), prm.quant_m, prm.trunc, 127)
        got = y[torch.as_tensor(rows, device=dev)].cpu().numpy().astype(np.int32)
        ok = bool(np.array_equal(got, want))
        ok_all &= ok
        tot_ms += ms
        per[f"{M}x{K}x{N}"] = {"us": round(ms * 1e3, 2),
                               "tops": round(2 * M * N * K / (ms / 1e3) / 1e12, 1),
                               "gemm_us": round(ms_gemm * 1e3, 2),
                               "gemm_tops": round(2 * M * N * K / (ms_gemm / 1e3) / 1e12, 1),
                               "parity_16_rows": ok}
        lin.close()
        del x, y
    ops = prefill_ops(PREFILL_SHAPES)
    big = per["2048x8192x8192"]
    return {"workload": PREFILL_WORKLOAD, "steps": steps, "ms_per_sweep": round(tot_ms, 4),
            "tops": round(ops / (tot_ms / 1e3) / 1e12, 1), "per_shape": per,
            "roofline": {"bound": "tensor (M >= 512), hbm (M = 128)",
                         "largest_gemm_tops": big["tops"], "nominal_int8_tops": 4500.0,
                         "frac_of_nominal": round(big["tops"] / 4500.0, 4),
                         "largest_gemm_kernel_tops": big["gemm_tops"],
                         "kernel_frac_of_nominal": round(big["gemm_tops"] / 4500.0, 4),
                         "note": "tops: fused forward (dyntok act quant kernel + GEMM); "
                                 "gemm_tops: the tcgen05 GEMM kernel alone"},
            "l2": "256 MB rewritten before every timed forward", "parity": ok_all}


def run_prefill(args) -> None:
    """One step = the 12 prefill linears of the sweep, each a fused W8A8 forward (dyntok act
    quant kernel + tcgen05 GEMM with the requant epilogue) from fp32 activations in HBM to int8
    outputs.  Every GEMM runs on a cold L2 (a 256 MB write before it, outside the timed events)."""
    world = env_int("WORLD_SIZE", 1)
    rank = env_int("RANK", 0)
    local = env_int("LOCAL_RANK", 0)
    if world != args.gpus:
        raise SystemExit(f"--gpus {args.gpus} but WORLD_SIZE={world}")
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        import datetime
        import torch.distributed as dist
        dist.init_process_group("nccl", device_id=dev, timeout=datetime.timedelta(seconds=120))
    sys.path.insert(0, str(ROOT))
    from romanaccio_b200 import OUT_QUANT, PATH_TENSOR, Context, W8A8Linear, synth

    ctx = Context(local)
    jobs = []
    for i, (M, K, N) in enumerate(PREFILL_SHAPES):
        p = synth.make_linear(K, N, seed=i, device=dev)
        lin = W8A8Linear.from_params(ctx, p)
        lin.set_path(PATH_TENSOR)
        x = synth.activations(M, K, seed=100 + i, device=dev)
        y = torch.empty((M, N), dtype=torch.int8, device=dev)
        jobs.append((M, K, N, lin, x, y))
    flush = torch.empty(256 << 20, dtype=torch.int8, device=dev)
    stream = torch.cuda.current_stream()

    def barrier():
        if world > 1:
            import torch.distributed as dist
            dist.barrier()
        torch.cuda.synchronize()

    def step(events=None):
        for j, (M, K, N, lin, x, y) in enumerate(jobs):
            flush.zero_()
            if events is not None:
                events[j][0].record(stream)
            lin.forward(x, OUT_QUANT, dyntok=True, out=y)
            if events is not None:
                events[j][1].record(stream)

    for _ in range(args.warmup):
        step()
    barrier()
    evs = [[(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
            for _ in jobs] for _ in range(args.steps)]
    with ClockSampler(local) as clocks:
        barrier()
        for s in range(args.steps):
            step(evs[s])
        barrier()
    per_shape = [0.0] * len(jobs)
    for s in range(args.steps):
        for j, (a, b) in enumerate(evs[s]):
            per_shape[j] += a.elapsed_time(b) / args.steps
    ms = sum(per_shape)

    # end to end through the public API: pinned fp32 activations in, int8 outputs back
    x_host = [torch.empty((M, K), dtype=torch.float32).pin_memory() for (M, K, N, *_ ) in jobs]
    y_host = [torch.empty((M, N), dtype=torch.int8).pin_memory() for (M, K, N, *_ ) in jobs]
    for h, (M, K, N, lin, x, y) in zip(x_host, jobs):
        h.copy_(x)
    h2d = sum(h.numel() * 4 for h in x_host)
    d2h = sum(h.numel() for h in y_host)
    barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(args.steps):
        for h, o, (M, K, N, lin, x, y) in zip(x_host, y_host, jobs):
            x.copy_(h, non_blocking=True)
            lin.forward(x, OUT_QUANT, dyntok=True, out=y)
            o.copy_(y, non_blocking=True)
        stream.synchronize()
    e1.record(stream)
    barrier()
    ms_e2e = e0.elapsed_time(e1) / args.steps

    # dominant kernel: the tensor-core GEMM of M=2048, K=N=8192 alone (int8 input in HBM)
    M, K, N, lin, x, y = jobs[PREFILL_SHAPES.index((2048, 8192, 8192))]
    q = torch.empty((M, K), dtype=torch.int8, device=dev)
    ratio = torch.empty((M,), dtype=torch.float32, device=dev)
    lin.pack_npu_input(x, dyntok_ratios=ratio, out=q)
    reps = 10
    gemm_ms = []
    for r in range(reps + 3):
        flush.zero_()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record(stream)
        lin.submit(q, OUT_QUANT, out=y)
        b.record(stream)
        torch.cuda.synchronize()
        if r >= 3:
            gemm_ms.append(a.elapsed_time(b))
    gemm_s = statistics.median(gemm_ms) / 1e3

    times = torch.tensor([ms, ms_e2e], dtype=torch.float64, device=dev)
    if world > 1:
        import torch.distributed as dist
        dist.all_reduce(times, op=dist.ReduceOp.MAX)
    ms, ms_e2e = times.tolist()

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu:
        sample = [s for s in PREFILL_SHAPES if s[0] == 128]
        run_cpu, cores = cpu_prefill_fn(sample)
        run_cpu()
        n, t0 = 0, time.perf_counter()
        while True:
            run_cpu()
            n += 1
            if time.perf_counter() - t0 > args.cpu_seconds:
                break
        dt = (time.perf_counter() - t0) / n
        cpu = {"value": prefill_ops(sample) / dt / 1e12, "unit": "TOPS", "cores": cores,
               "kind": "port", "sample": f"{n} passes over the four M=128 linears of the sweep, "
                                         "C restatement of the reference linear, OpenMP"}

    ops = prefill_ops(PREFILL_SHAPES)
    peaks = json.loads((ROOT / "MEASURED_PEAKS.json").read_text()) \
        if (ROOT / "MEASURED_PEAKS.json").exists() else {}
    bf16 = float(peaks.get("bf16_tflops", 1590.0))
    peak = 2.0 * bf16
    achieved = 2 * M * N * K / gemm_s / 1e12
    if rank == 0:
        line = {
            "metric": PREFILL_METRIC, "value": world * ops / (ms / 1e3) / 1e12, "unit": "TOPS",
            "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "int8",
            "data": "synthetic",
            "config": {"workload": PREFILL_WORKLOAD,
                       "parallelism": f"replicas: every GPU runs the whole sweep (x{world})",
                       "l2": "256 MB written before every GEMM (outside the timed events)",
                       "per_shape_us": {f"{m}x{k}x{n}": round(t * 1e3, 2)
                                        for (m, k, n), t in zip(PREFILL_SHAPES, per_shape)},
                       "per_shape_tops": {f"{m}x{k}x{n}": round(2 * m * n * k / (t / 1e3) / 1e12, 1)
                                          for (m, k, n), t in zip(PREFILL_SHAPES, per_shape)}},
            "roofline": {"bound": "tensor", "achieved": achieved, "peak": peak, "unit": "TOPS",
                         "frac": achieved / peak, "traffic": PREFILL_GEMM_TRAFFIC_BYTES,
                         "kernel": "gemm_w8a8_tc_kernel M=2048 K=N=8192 (int8 in, int8 out)",
                         "peak_kind": "2 x measured bf16 burst (B200 int8 dense rate = 2 x bf16)"
                                      if "bf16_tflops" in peaks else "2 x fallback bf16",
                         "nominal_peak": 4500.0, "frac_of_nominal": achieved / 4500.0,
                         "launch_us": gemm_s * 1e6},
            "e2e": {"value": world * ops / (ms_e2e / 1e3) / 1e12, "unit": "TOPS",
                    "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h},
            "gpu_launches": 2 * len(jobs) * args.steps,
            "clocks": clocks.summary(),
        }
        if cpu is not None:
            line["cpu_baseline"] = cpu
        print(json.dumps(line), flush=True)
    if world > 1:
        import torch.distributed as dist
        dist.barrier()
        dist.destroy_process_group()


# ---------------------------------------------------------------------------- LM-head latency
def lmhead_cpu_baseline(wq: np.ndarray, acc_step: np.ndarray, in_step: float, h: np.ndarray,
                        k: int, seconds: float) -> dict:
    """The LM head on the host cores: the C restatement (OpenMP over every core this process may
    use) of the static input quantisation, the int8 GEMV over the whole vocabulary and the
    top-k, timed over repeated tokens for about `seconds` (the reference's own host LM head,
    TransformerSession's fp32 fallback GEMV + Sampler::sample over V, is the same loop shape)."""
    sys.path.insert(0, str(ROOT))
    from oracle import oracle as O
    import ctypes as C
    lib = O.lib()
    cores = len(os.sched_getaffinity(0))
    lib.orc_set_threads(cores)
    T, K = h.shape
    V = wq.shape[0]
    x = np.ascontiguousarray(h, dtype=np.float32)
    w = np.ascontiguousarray(wq)
    st = np.ascontiguousarray(acc_step, dtype=np.float32)
    logits = np.empty((T, V), np.float32)
    q = np.empty((T, K), np.int8)
    val = np.empty((T, k), np.float32)
    idx = np.empty((T, k), np.int32)

    def run():
        lib.orc_lmhead_topk_omp(x.ctypes.data, T, K, V, w.ctypes.data, C.c_float(in_step),
                                st.ctypes.data, k, logits.ctypes.data, q.ctypes.data,
                                val.ctypes.data, idx.ctypes.data)

    run()
    n, t0 = 0, time.perf_counter()
    while time.perf_counter() - t0 < seconds or n < 3:
        run()
        n += 1
    us = (time.perf_counter() - t0) / n * 1e6
    return {"value": us, "unit": "us", "cores": cores, "kind": "port",
            "sample": f"{n} LM-head steps ({T} token(s), {K}x{V} int8 + top-{k}), C restatement, "
                      "OpenMP", "ids": idx[:, 0].tolist()}


LMHEAD_METRIC = ("LM-head latency per decode step (hidden state in HBM -> top-40 ids and argmax "
                 "on the host), vocab-sharded over n GPUs of one process")


def run_lmhead(args) -> None:
    """Qwen2.5-1.5B LM head (1536 x 151936, static int8 input, logits = acc * in_step * w_step)
    sharded over n = 1, 2, 4, ... up to --gpus devices driven by this one process
    (w8a8_lmhead_*).  Per step: device 0 quantises h and stores it into every shard's staging
    buffer, every shard runs its top-k GEMV, and device 0's merge kernel writes the argmax ids
    straight into pinned host memory (mapped; no separate copy).

    Two clocks, both CUDA events on GPU 0's stream:
      latency  from "h ready on GPU 0" to "ids in host memory".  A ~100 us GPU delay stands in
               for the decode step's layers before the LM head, during which the host issues
               the forward (as it does while a decode step's layers run), so the host's launch
               calls are not on the clock; the shards on other GPUs may start streaming their
               weights during that delay, as they would during the layers.
      e2e      the same forward with GPU 0 idle before it: the host's launch calls for all
               shards are on the clock.
    """
    if env_int("WORLD_SIZE", 1) > 1:
        raise SystemExit("--workload lmhead drives every GPU from one process; run it without "
                         "torchrun")
    sys.path.insert(0, str(ROOT))
    from romanaccio_b200 import Context, MultiDeviceLmHead, synth
    n_max = min(args.gpus, torch.cuda.device_count())
    ctxs = [Context(d) for d in range(n_max)]
    torch.cuda.set_device(0)
    K, V, k, T = synth.QWEN25_15B.hidden, synth.QWEN25_15B.vocab, 40, args.batch
    rng = np.random.default_rng(17)
    wq = rng.integers(-127, 128, size=(V, K), dtype=np.int16).astype(np.int8)
    w_step = (rng.random(V) * 0.02 / 127 + 1e-5)
    in_step = float(synth.activations(64, K, 23).abs().max()) / 127.0
    acc_step = (in_step * w_step).astype(np.float32)
    h = synth.activations(T, K, seed=5).cuda()
    ids_host = torch.empty((T,), dtype=torch.int32).pin_memory()
    counts = [n for n in (1, 2, 4, 8) if n <= n_max]
    # 256 MB written on every GPU between steps: no L2 holds any of its shard's weights at step
    # start
    flush = [torch.empty(256 << 20, dtype=torch.uint8, device=f"cuda:{d}") for d in range(n_max)]
    delay_cycles = 200_000  # ~100 us at 1.9 GHz
    result, ids_ref = {}, None
    stream = torch.cuda.current_stream()
    for n in counts:
        lm = MultiDeviceLmHead(ctxs[:n], wq, acc_step, in_step, max_tokens=max(T, 8), k_max=k)
        val = torch.empty((T, k), dtype=torch.float32, device="cuda")
        idx = torch.empty((T, k), dtype=torch.int32, device="cuda")
        for d in range(n):
            torch.cuda.synchronize(d)

        def step(delay: bool) -> float:
            for f in flush[:n]:
                f.fill_(1)
            if delay:
                torch.cuda._sleep(delay_cycles)
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record(stream)
            # the merge kernel stores the argmax ids straight into pinned host memory
            lm.forward(h, k, val, idx, ids_host)
            b.record(stream)
            b.synchronize()
            return a.elapsed_time(b) * 1e3

        for _ in range(args.warmup):
            step(True)
        lat = [step(True) for _ in range(args.steps)]
        e2e = [step(False) for _ in range(args.steps)]
        ids = ids_host.clone()
        if ids_ref is None:
            ids_ref = ids
        result[n] = {"us_median": statistics.median(lat), "us_min": min(lat),
                     "e2e_us_median": statistics.median(e2e),
                     "ids_equal_1gpu": bool(torch.equal(ids, ids_ref))}
        del lm
        for d in range(n):
            torch.cuda.synchronize(d)
    for c in ctxs:
        c.check()
    lat = [result[n]["us_median"] for n in counts]
    e2e_lat = [result[n]["e2e_us_median"] for n in counts]
    top = result[counts[-1]]
    line = {
        "metric": LMHEAD_METRIC, "value": top["us_median"], "unit": "us",
        "n_gpus": counts[-1], "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": top["us_median"] / 1e3, "higher_is_better": False,
        "scaling": "strong", "vs_baseline": None, "dtype": "int8", "data": "synthetic",
        "config": {"workload": f"LM head {K}x{V} top-{k} + argmax, T={T}",
                   "by_shards": {str(n): result[n] for n in counts},
                   "monotonic_decreasing": all(x > y for x, y in zip(lat, lat[1:])),
                   "e2e_monotonic_decreasing": all(x > y for x, y in zip(e2e_lat, e2e_lat[1:])),
                   "parallelism": "vocab-sharded, one process; activations and candidates cross "
                                  "NVLink by peer stores, device-memory counters in place of "
                                  "stream events",
                   "l2": "256 MB written on every GPU before every step",
                   "clock": "latency: h ready on GPU 0 (after a ~100 us GPU delay standing in "
                            "for the layers) -> ids in pinned host memory"},
        "e2e": {"value": top["e2e_us_median"], "unit": "us", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": T * 4},
        "gpu_launches": counts[-1] + 2,
    }
    if not args.no_cpu:
        cpu = lmhead_cpu_baseline(wq, acc_step, in_step, h.cpu().numpy(), k, args.cpu_seconds)
        cpu_ids = cpu.pop("ids")
        cpu["ids_equal_gpu"] = cpu_ids == ids_ref.tolist()
        line["cpu_baseline"] = cpu
    print(json.dumps(line), flush=True)


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--batch", type=int, default=1)
    ap.add_argument("--layers", type=int, default=None)
    ap.add_argument("--per-linear", action="store_true",
                    help="launch each linear separately instead of the persistent decode-chain "
                         "kernel (one cooperative launch per step)")
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--workload", choices=["decode", "prefill", "lmhead"], default="decode",
                    help="decode: the headline decode step; prefill: the int8 GEMM sweep; "
                         "lmhead: sharded LM-head latency over 1, 2, 4, 8 GPUs of one process")
    ap.add_argument("--no-cpu", action="store_true")
    ap.add_argument("--no-parity", action="store_true",
                    help="skip the oracle check of the measured step")
    ap.add_argument("--no-per-config", action="store_true",
                    help="skip the per-configuration records (configs 0, 1 at T=8/32, 2, 3, 4)")
    ap.add_argument("--config-steps", type=int, default=10,
                    help="timed steps of each per-configuration record")
    ap.add_argument("--cpu-seconds", type=float, default=10.0)
    args = ap.parse_args()
    if args.warmup < 3:
        raise SystemExit("--warmup must be >= 3")
    if args.workload == "prefill":
        run_prefill_reference(args) if args.impl == "reference" else run_prefill(args)
    elif args.workload == "lmhead":
        run_lmhead(args)
    elif args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
