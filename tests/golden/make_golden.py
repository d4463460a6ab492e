"""Generates the golden fixtures of tests/golden/ from the REFERENCE itself.

Run in a container that has the reference tree (read-only) at REF (default /root/reference):

    python tests/golden/make_golden.py [--ref /root/reference]

Sources of truth, all executed here rather than restated:
  * quant_linear_*.npz  -- build_single_conv_region / tile_int8_slice of
    src/LFM3/build_lfm3_int8_pkg.py:95-108, 171-224 (imported with its flatbuffer / compiler
    dependencies stubbed, since those only serve the .model patching).  The NVDLA-tiled weight
    bytes it writes are un-tiled with the inverse of its (0, 2, 3, 4, 1, 5) transpose.
  * boundary_*.npz      -- pack_npu_input_int8[_dyntok] / unpack_npu_output_int8[_dyntok] of
    src/LFM3/lfm3_v2.cpp (compiled by oracle/Makefile into oracle/_ref/libref.so).
  * requant_kat.npz     -- the CvtPrecision_QuantM expression as the reference's float64 torch
    simulation writes it, round(acc * (QuantM / 2^trunc)) clamped to +-Qmax
    (src/LFM3/attribute_int8_error.py:104-122), over hand-picked edge cases.
  * sampler_kat.npz     -- Sampler::sample greedy (oracle/_ref/libref.so) on the vector of
    src/eswin_runtime/tests/test_tokenizer_sampler.cpp:19-31 plus tie cases.
  * moe_route.npz       -- MoERouter::route (src/eswin_runtime/src/llm/moe_router.cpp:211-260,
    compiled into oracle/_ref/libref.so) on seeded gate logits (64 experts, top-6): raw
    softmax weights (norm_topk_prob = false), renormalised weights, and a gate bias.
"""
from __future__ import annotations

import argparse
import json
import sys
import types
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
ROOT = HERE.parent.parent
sys.path.insert(0, str(ROOT))

from oracle import oracle as O  # noqa: E402


class _Region:
    """Stand-in for the weight region the builder reads from a .model template."""

    def __init__(self, n_rows: int, k: int, slice_rows: int = 512):
        k_pad = ((k + 95) // 96) * 96
        self.n_slices = (n_rows + slice_rows - 1) // slice_rows
        self.offsets, self.contents, off = [], [], 0
        self.slice_rows = []
        for s in range(self.n_slices):
            m = min(slice_rows, n_rows - s * slice_rows)
            self.slice_rows.append(m)
            self.offsets += [off, off + m * k_pad]
            self.contents += ["weights", "quant_m"]
            off += m * k_pad + 2 * m
        self.size = off
        self.k_pad = k_pad


def import_builder(ref: Path):
    sys.path.insert(0, str(ref / "src" / "LFM3"))
    for name in ("backend", "backend.flatbuffer_emitter", "backend.dynamic_weight_binding"):
        sys.modules.setdefault(name, types.ModuleType(name))
    sys.modules["backend.flatbuffer_emitter"].ModelReader = object
    sys.modules["backend.flatbuffer_emitter"].ModelWriter = object
    sys.modules["backend.dynamic_weight_binding"].find_weight_regions = lambda m: None
    import build_lfm3_int8_pkg as builder  # noqa: E402
    return builder


def untile_int8(raw: bytes, m: int, k: int, k_pad: int) -> np.ndarray:
    """Inverse of reshape(M/8, 8, Kp/96, 3, 8, 4).transpose(0, 2, 3, 4, 1, 5)."""
    a = np.frombuffer(raw, dtype=np.int8).reshape(m // 8, k_pad // 96, 3, 8, 8, 4)
    return a.transpose(0, 4, 1, 2, 3, 5).reshape(m, k_pad)[:, :k].copy()


def seeded_inputs(n: int, k: int, seed: int):
    rng = np.random.default_rng(seed)
    w = (rng.standard_normal((n, k)) * 0.02).astype(np.float32)
    x = rng.standard_normal((64, k)).astype(np.float32)
    out_ch = rng.choice(k, size=max(1, k // 100), replace=False)
    x[:, out_ch] *= 20.0
    return w, x


def make_quant_linear(builder, n: int, k: int, trunc: int, seed: int, path: Path) -> None:
    w, x = seeded_inputs(n, k, seed)
    reg = _Region(n, k)
    buf, in_t, in_s, in_inv_smooth, out_step_chan = builder.build_single_conv_region(
        w, torch.from_numpy(x), None, trunc, cached_reg=reg)
    wq = np.empty((n, k), np.int8)
    qm = np.empty((n,), np.int16)
    for s in range(reg.n_slices):
        m = reg.slice_rows[s]
        r0 = s * 512
        wo, qo = reg.offsets[2 * s], reg.offsets[2 * s + 1]
        wq[r0:r0 + m] = untile_int8(buf[wo:wo + m * reg.k_pad], m, k, reg.k_pad)
        qm[r0:r0 + m] = np.frombuffer(buf[qo:qo + 2 * m], dtype=np.int16)
    np.savez_compressed(path, w=w, calib_x=x, trunc=np.int32(trunc), wq=wq, quant_m=qm,
                        in_thresh=np.float64(in_t), in_step=np.float64(in_s),
                        in_inv_smooth=in_inv_smooth.astype(np.float32),
                        out_step_chan=out_step_chan.astype(np.float32))
    print(f"{path.name}: N={n} K={k} trunc={trunc} in_t={in_t:.6f} qm[{qm.min()}, {qm.max()}]")


def make_boundary(path: Path, T: int, K: int, N: int, seed: int) -> None:
    rng = np.random.default_rng(seed)
    x = rng.standard_normal((T, K)).astype(np.float32)
    x[:, rng.choice(K, size=max(1, K // 100), replace=False)] *= 20.0
    # edge values: exact halves after scaling are produced by in_step = 1 on x = +-k.5
    x[0, :8] = np.array([0.5, 1.5, 2.5, -0.5, -1.5, 126.5, -126.5, 1000.0], np.float32)
    s = (rng.random(K).astype(np.float32) * 2.0 + 0.05).astype(np.float32)
    s[:8] = 1.0
    q_static = O.ref_pack(x, 1.0, s)
    q_static_nosmooth = O.ref_pack(x, 0.037, None)
    q_dyn, ratio = O.ref_pack_dyntok(x, 4.25, s)
    yq = rng.integers(-127, 128, size=(T, N)).astype(np.int8)
    osc = (rng.random(N).astype(np.float32) * 0.01 + 1e-4).astype(np.float32)
    y_static = O.ref_unpack(yq, 0.0123, osc, None)
    y_static_scalar = O.ref_unpack(yq, 0.0123, None, None)
    y_dyn = O.ref_unpack(yq, 0.0123, osc, ratio)
    y_dyn_scalar = O.ref_unpack(yq, 0.0123, None, ratio)
    yq16 = rng.integers(-32767, 32768, size=(T, N)).astype(np.int16)
    y16 = O.ref_unpack_i16(yq16, 0.0007, osc)
    np.savez_compressed(path, x=x, inv_smooth=s, q_static=q_static,
                        q_static_nosmooth=q_static_nosmooth, q_dyn=q_dyn, ratio=ratio, yq=yq,
                        out_step_chan=osc, y_static=y_static, y_static_scalar=y_static_scalar,
                        y_dyn=y_dyn, y_dyn_scalar=y_dyn_scalar, yq16=yq16, y16=y16)
    print(f"{path.name}: T={T} K={K} N={N}")


def make_requant_kat(path: Path) -> None:
    cases = []
    for trunc in (0, 1, 14, 15, 22, 23, 25, 26, 28):
        half = 1 << max(trunc - 1, 0)
        for qm in (1, 2, 3, 127, 4096, 32767):
            for acc in (0, 1, -1, half, -half, 3 * half, -3 * half, 2**31 - 1, -2**31, 127 << trunc,
                        (127 << trunc) + half, -(127 << trunc) - half, 1000, -1000, 123456789):
                acc = int(np.clip(acc, -2**31, 2**31 - 1))
                cases.append((acc, qm, trunc))
    acc = np.array([c[0] for c in cases], np.int64)
    qm = np.array([c[1] for c in cases], np.int64)
    tr = np.array([c[2] for c in cases], np.int64)
    out = {}
    for qmax in (127, 32767):
        a = torch.from_numpy(acc).double()
        scale = torch.from_numpy(qm).double() / torch.from_numpy((1 << tr).astype(np.float64))
        out[f"yq_{qmax}"] = torch.clamp(torch.round(a * scale), -float(qmax), float(qmax)).long().numpy()
    # CACC saturation known answer (src/eswin_simulator/tests/test_cmac_cacc.py:137-149):
    # QuantM = 1, trunc = 0 passes acc through; the SDP rule saturates symmetrically at +-127.
    cacc = np.array([-1000, -200, -128, 0, 50, 127, 200, 1000], np.int64)
    np.savez_compressed(path, acc=acc.astype(np.int32), quant_m=qm.astype(np.int16),
                        trunc=tr.astype(np.int32), cacc_acc=cacc.astype(np.int32), **out)
    print(f"{path.name}: {len(cases)} cases")


def make_sampler_kat(path: Path) -> None:
    rows = [
        np.array([1.0, 2.5, 0.5, 8.2, 3.1], np.float32),          # test_tokenizer_sampler.cpp:22
        np.array([3.0, 7.0, 7.0, 1.0, 7.0], np.float32),          # ties: lowest id wins
        np.array([-5.0, -1.0, -1.0, -3.0], np.float32),
        np.array([0.0, -0.0, 0.0], np.float32),
    ]
    rng = np.random.default_rng(7)
    big = rng.integers(-127, 128, size=4096).astype(np.float32) * 0.25  # int8-like logits, many ties
    rows.append(big)
    greedy = np.array([O.ref_greedy(r) for r in rows], np.int32)
    lens = np.array([len(r) for r in rows], np.int32)
    np.savez_compressed(path, logits=np.concatenate(rows), lens=lens, greedy=greedy)
    print(f"{path.name}: greedy={greedy.tolist()}")


def make_moe_route(path: Path) -> None:
    rng = np.random.default_rng(31)
    T, H, E, k = 6, 512, 64, 6
    hidden = rng.standard_normal((T, H)).astype(np.float32)
    gate_w = (rng.standard_normal((E, H)) * 0.02).astype(np.float32)
    bias = (rng.standard_normal(E) * 0.01).astype(np.float32)
    idx_raw, w_raw = O.ref_moe_route(hidden, gate_w, k)
    idx_norm, w_norm = O.ref_moe_route(hidden, gate_w, k, norm_topk=True, scaling=2.5)
    idx_bias, w_bias = O.ref_moe_route(hidden, gate_w, k, bias=bias)
    np.savez_compressed(path, hidden=hidden, gate_w=gate_w, bias=bias, k=np.int32(k),
                        idx_raw=idx_raw, w_raw=w_raw, idx_norm=idx_norm, w_norm=w_norm,
                        idx_bias=idx_bias, w_bias=w_bias)
    print(f"{path.name}: ids {idx_raw[0].tolist()}")


def make_norm_pack(path: Path) -> None:
    """fused_rms_norm_pack_dyntok_t1 and fused_post_op_residual_ffn_pack_mlp_t1 run by the
    reference on seeded rows (a multiple-of-4 width and one with a 3-element tail)."""
    rng = np.random.default_rng(41)
    out = {}
    for tag, C in (("c1536", 1536), ("c579", 579)):
        h = (rng.standard_normal(C) * 4).astype(np.float32)
        norm = (rng.standard_normal(C) * 0.3 + 1).astype(np.float32)
        smooth = (rng.random(C) * 2 + 0.05).astype(np.float32)
        op = (rng.standard_normal(C) * 6).astype(np.float32)
        post = (rng.standard_normal(C) * 0.2 + 1).astype(np.float32)
        ffn = (rng.random(C) * 25).astype(np.float32)
        q, ratio, u = O.ref_rmsnorm_pack_dyntok(h, norm, smooth, 7.5)
        m, q2 = O.ref_post_op_ffn_pack(op, post, h, ffn)
        out.update({f"{tag}_h": h, f"{tag}_norm": norm, f"{tag}_smooth": smooth,
                    f"{tag}_op": op, f"{tag}_post": post, f"{tag}_ffn": ffn, f"{tag}_q": q,
                    f"{tag}_ratio": np.float32(ratio), f"{tag}_u": u, f"{tag}_hmid": m,
                    f"{tag}_q2": q2})
    np.savez_compressed(path, in_thresh=np.float32(7.5), **out)
    print(f"{path.name}: ratio {out['c1536_ratio']}")


def make_sampler_seq(path: Path) -> None:
    """Token sequences drawn by the reference Sampler (full logits, seeded) for the candidate
    sampler's parity without the reference built."""
    rng = np.random.default_rng(61)
    V, S = 2000, 16
    logits = (rng.standard_normal((S, V)) * 3).astype(np.float32)
    history = np.argsort(-logits[0])[:10].astype(np.int32)
    cfgs = {"default": dict(temperature=0.7, top_k=40, top_p=0.9, min_p=0.05, repeat_penalty=1.15,
                            repeat_window=64, max_consecutive_duplicates=2, seed=1234),
            "greedy": dict(temperature=0.0, top_k=40, top_p=0.9, min_p=0.05, repeat_penalty=1.3,
                           repeat_window=8, max_consecutive_duplicates=2, seed=1)}
    out = {"logits": logits, "history": history}
    for name, c in cfgs.items():
        out[f"{name}_tokens"] = O.ref_sampler_run(c, history, logits)
        for key, val in c.items():
            out[f"{name}_{key}"] = np.asarray(val)
    np.savez_compressed(path, **out)
    print(f"{path.name}: default {out['default_tokens'][:6].tolist()}")


def make_nvdla_tiles(builder, path: Path) -> None:
    """The reference's NVDLA weight tiling (tile_int8_slice / tile_int16_slice) of seeded slices,
    with the row-major quantised weights computed from the same formula, for the package
    reader's un-tiling."""
    rng = np.random.default_rng(51)
    out = {}
    for tag, (m, k) in (("a", (512, 96)), ("b", (16, 200)), ("c", (24, 96))):
        w = rng.standard_normal((m, k)) * 0.05
        tiled, step = builder.tile_int8_slice(w)
        w64 = w.astype(np.float64)
        st = np.maximum(np.max(np.abs(w64), axis=1, keepdims=True), 1e-12) / 127.0
        q = np.clip(np.round(w64 / st), -127, 127).astype(np.int8)
        out[f"i8_{tag}_tiled"] = np.frombuffer(tiled, np.int8)
        out[f"i8_{tag}_q"] = q
        out[f"i8_{tag}_step"] = step
    for tag, (m, k) in (("a", (16, 100)), ("b", (8, 48))):
        w = rng.standard_normal((m, k)) * 0.05
        tiled, step = builder.tile_int16_slice(w)
        w64 = w.astype(np.float64)
        st = np.maximum(np.max(np.abs(w64), axis=1, keepdims=True), 1e-12) / 32767.0
        q = np.clip(np.round(w64 / st), -32767, 32767).astype(np.int16)
        out[f"i16_{tag}_tiled"] = np.frombuffer(tiled, np.int16)
        out[f"i16_{tag}_q"] = q
    np.savez_compressed(path, **out)
    print(f"{path.name}: {len(out)} arrays")


def make_emb_norm_pack(path: Path) -> None:
    """fused_emb_norm_broadcast_t1 (the LM head's input step) run by the reference on seeded
    final hidden states (widths 1536, 2048, 3840 and one with a 2-element tail), with
    emb_norm_scaled = weight * (1 / in_step) computed as the reference loader does in fp32."""
    rng = np.random.default_rng(43)
    out = {}
    for tag, C in (("c1536", 1536), ("c2048", 2048), ("c3840", 3840), ("c578", 578)):
        h = (rng.standard_normal(C) * 3).astype(np.float32)
        w = (rng.standard_normal(C) * 0.3 + 1).astype(np.float32)
        in_step = np.float32(0.031)
        emb = (w * (np.float32(1.0) / in_step)).astype(np.float32)
        q = O.ref_emb_norm_pack(h, emb)
        out.update({f"{tag}_h": h, f"{tag}_emb": emb, f"{tag}_q": q})
    np.savez_compressed(path, eps=np.float32(1e-5), **out)
    print(f"{path.name}: {len(out) // 3} rows")


def make_mini_package(builder, out_dir: Path) -> None:
    """A two-subgraph package in the reference's format (build_lfm3_int8_pkg.py:440-511): the
    weight regions come from the reference builder's own build_single_conv_region (NVDLA-tiled
    slices + QuantM at the stand-in template's offsets), quant_scales.json / quant_chan_scales.bin
    / weights_map.json are written the way its record_scale_entry and package loop write them,
    and region_offsets.json stands in for the loadable templates the engine reads the offsets
    from.  expected.npz keeps the builder's own returned values and the slices untiled here, for
    the ingest test to compare against."""
    out_dir.mkdir(exist_ok=True)
    chan_floats, subs, w_map, offs = [], {}, {}, {}
    blob = bytearray()
    exp = {}
    for name, n, k, trunc, seed in (("mini_l00_conv_in", 136, 160, 22, 51),
                                    ("mini_l00_attn_qkv", 520, 96, 23, 52)):
        w, x = seeded_inputs(n, k, seed)
        reg = _Region(n, k)
        buf, in_t, in_s, inv, osc = builder.build_single_conv_region(
            w, torch.from_numpy(x), None, trunc, cached_reg=reg)
        in_off = len(chan_floats)
        chan_floats.extend(np.asarray(inv, np.float32).tolist())
        out_off = len(chan_floats)
        chan_floats.extend(np.asarray(osc, np.float32).tolist())
        med = float(np.median(osc))
        subs[name] = {"input_dtype": "int8", "output_dtype": "int8",
                      "input_threshold": float(in_t), "input_step": float(in_s),
                      "output_threshold": med * 127.0, "output_step": med,
                      "in_smooth_offset": in_off, "in_smooth_count": int(k),
                      "out_step_offset": out_off, "out_step_count": int(n)}
        w_map[name] = {"layer": 0, "die": 0, "weight_offset": len(blob), "weight_size": len(buf)}
        offs[name] = {"offsets": list(map(int, reg.offsets)), "N": n, "K": k, "trunc": trunc}
        blob += buf
        wq = np.empty((n, k), np.int8)
        qm = np.empty((n,), np.int16)
        for sl in range(reg.n_slices):
            m = reg.slice_rows[sl]
            wo, qo = reg.offsets[2 * sl], reg.offsets[2 * sl + 1]
            wq[sl * 512:sl * 512 + m] = untile_int8(buf[wo:wo + m * reg.k_pad], m, k, reg.k_pad)
            qm[sl * 512:sl * 512 + m] = np.frombuffer(buf[qo:qo + 2 * m], dtype=np.int16)
        exp.update({f"{name}_wq": wq, f"{name}_qm": qm, f"{name}_inv": np.asarray(inv, np.float32),
                    f"{name}_osc": np.asarray(osc, np.float32), f"{name}_in_t": np.float64(in_t),
                    f"{name}_in_s": np.float64(in_s), f"{name}_x": x[:5].copy()})
    (out_dir / "die0.bin").write_bytes(bytes(blob))
    np.asarray(chan_floats, dtype=np.float32).tofile(str(out_dir / "quant_chan_scales.bin"))
    (out_dir / "quant_scales.json").write_text(json.dumps({"subgraphs": subs}, indent=2))
    (out_dir / "weights_map.json").write_text(json.dumps(w_map, indent=2))
    (out_dir / "region_offsets.json").write_text(json.dumps(offs, indent=2))
    np.savez_compressed(out_dir / "expected.npz", **exp)
    print(f"{out_dir.name}: {len(blob)} weight bytes, {len(chan_floats)} sidecar floats")


def make_mlp_w2(path: Path, ref: Path) -> None:
    """The int16 w2 stage of the SwiGLU MLP as the reference's own engine model computes it:
    attribute_int8_error.sim_mlp_npu (src/LFM3/attribute_int8_error.py:85-122) runs on seeded
    weights and tokens, and its last F.linear call (int16 activations m1_q against the int16 codes
    wq2) and the final clamp (the int16 outputs) are recorded as they happen.  QuantM of w2 is
    stored beside them (the same formula, :120)."""
    from torch.overrides import TorchFunctionMode
    import torch.nn.functional as F
    sys.path.insert(0, str(ref / "src" / "LFM3"))
    import attribute_int8_error as A  # noqa: E402

    class Record(TorchFunctionMode):
        def __init__(self):
            super().__init__()
            self.linear, self.clamp = [], []

        def __torch_function__(self, func, types, args=(), kwargs=None):
            out = func(*args, **(kwargs or {}))
            if func is F.linear:
                self.linear.append((args[0].detach().clone(), args[1].detach().clone()))
            elif func is torch.clamp:
                self.clamp.append(out.detach().clone())
            return out

    out = {}
    for tag, H, I, T, seed in (("a", 64, 96, 4, 61), ("b", 200, 328, 3, 62)):
        g = torch.Generator().manual_seed(seed)
        x = torch.randn((T, H), generator=g, dtype=torch.float64)
        w1 = torch.randn((I, H), generator=g, dtype=torch.float64) * 0.08
        w3 = torch.randn((I, H), generator=g, dtype=torch.float64) * 0.08
        w2 = torch.randn((H, I), generator=g, dtype=torch.float64) * 0.08
        c0 = x @ w1.T
        c1 = x @ w3.T
        m0 = F.silu(c0)
        m1 = m0 * c1
        y = m1 @ w2.T
        tbl = {"blob_info": {
            "input": {"int8_step": float(x.abs().max()) / 127.0},
            "/Conv_output_0": {"int16_step": float(c0.abs().max()) * 1.1 / 32767.0},
            "/Conv_1_output_0": {"int16_step": float(c1.abs().max()) * 1.1 / 32767.0},
            "/Sigmoid_output_0": {"int16_step": 1.0 / 32767.0},
            "/Mul_output_0": {"int16_step": float(m0.abs().max()) * 1.1 / 32767.0},
            "/Mul_1_output_0": {"int16_step": float(m1.abs().max()) * 1.1 / 32767.0},
            "output": {"int16_step": float(y.abs().max()) * 1.3 / 32767.0}}}
        rec = Record()
        with rec:
            y_ref = A.sim_mlp_npu(x.float(), w1.float(), w3.float(), w2.float(), tbl, True)
        m1_q, wq2 = rec.linear[-1]
        out_q = rec.clamp[-1]
        m1_s = tbl["blob_info"]["/Mul_1_output_0"]["int16_step"]
        out_s = tbl["blob_info"]["output"]["int16_step"]
        ws2 = w2.float().double().abs().amax(dim=1, keepdim=True).clamp(min=1e-12) / 32767.0
        qm2 = torch.round((m1_s * ws2[:, 0] / out_s) * (1 << 28))
        assert float(qm2.max()) <= 32767.0 and float(qm2.min()) >= 1.0
        out.update({f"{tag}_x": m1_q.numpy().astype(np.int16), f"{tag}_w": wq2.numpy().astype(np.int16),
                    f"{tag}_qm": qm2.numpy().astype(np.int16), f"{tag}_yq": out_q.numpy().astype(np.int16),
                    f"{tag}_y": y_ref.numpy().astype(np.float32), f"{tag}_out_s": np.float64(out_s)})
    np.savez_compressed(path, trunc=np.int32(28), **out)
    print(f"{path.name}: yq range [{out['a_yq'].min()}, {out['a_yq'].max()}]")


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref", default="/root/reference")
    ap.add_argument("--only", default=None, help="generate one fixture family (e.g. moe)")
    args = ap.parse_args()
    ref = Path(args.ref)
    O.build()
    if args.only == "moe":
        make_moe_route(HERE / "moe_route.npz")
        return
    if args.only == "norm":
        make_norm_pack(HERE / "norm_pack.npz")
        make_emb_norm_pack(HERE / "emb_norm_pack.npz")
        return
    if args.only == "sampler":
        make_sampler_seq(HERE / "sampler_seq.npz")
        return
    if args.only == "tiles":
        make_nvdla_tiles(import_builder(ref), HERE / "nvdla_tiles.npz")
        return
    if args.only == "package":
        make_mini_package(import_builder(ref), HERE / "pkg_mini")
        return
    if args.only == "mlp_w2":
        make_mlp_w2(HERE / "mlp_w2_int16.npz", ref)
        return
    builder = import_builder(ref)
    make_quant_linear(builder, 136, 160, 22, 11, HERE / "quant_linear_n136_k160_t22.npz")
    make_quant_linear(builder, 520, 96, 23, 12, HERE / "quant_linear_n520_k96_t23.npz")
    make_boundary(HERE / "boundary_t1.npz", 1, 576, 192, 21)
    make_boundary(HERE / "boundary_t5.npz", 5, 192, 64, 22)
    make_requant_kat(HERE / "requant_kat.npz")
    make_sampler_kat(HERE / "sampler_kat.npz")
    make_moe_route(HERE / "moe_route.npz")
    make_norm_pack(HERE / "norm_pack.npz")
    make_emb_norm_pack(HERE / "emb_norm_pack.npz")
    make_nvdla_tiles(builder, HERE / "nvdla_tiles.npz")
    make_mini_package(builder, HERE / "pkg_mini")
    make_mlp_w2(HERE / "mlp_w2_int16.npz", ref)
    make_sampler_seq(HERE / "sampler_seq.npz")


if __name__ == "__main__":
    main()
