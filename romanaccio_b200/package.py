"""Ingest of the reference's quantised-weight package (build_lfm3_int8_pkg.py:446-511).

A package directory holds `quant_scales.json` (one entry per subgraph: dtypes, input threshold /
step, output threshold / step, and offsets into the float sidecar), `quant_chan_scales.bin` (the
float32 sidecar: every subgraph's in_inv_smooth [K] and out_step_chan [N]) and per-die weight
blobs whose weight regions hold, per slice of 512 output channels, the NVDLA-tiled weights and
the int16 QuantM vector at offsets fixed by the region's loadable template.

  load_quant_scales      quant_scales.json + quant_chan_scales.bin -> {name: SubgraphScaleInfo}
                         with the defaults and the validity rule of parse_entry
                         (lfm3_v2.cpp:3743-3826)
  untile_int8 / _int16   NVDLA CMAC tiling -> row-major [N, K]; the inverse of tile_int8_slice /
                         tile_int16_slice (build_lfm3_int8_pkg.py:95-121; cmac.py:67-115)
  read_weight_region     one region's slices (weights + QuantM at the template's offsets) ->
                         (weights [N, K], QuantM [N]) ready for W8A8Linear
"""
from __future__ import annotations

import json
from pathlib import Path

import numpy as np

from ._lib import DTYPE_FP16, DTYPE_INT8, DTYPE_INT16
from .linear import SubgraphScaleInfo

SLICE_ROWS = 512  # output channels per weight slice of a region (build_lfm3_int8_pkg.py:216-217)


def parse_boundary_dtype(s: str) -> int:
    """parse_boundary_dtype (lfm3_v2.cpp:567-571): "int8", "int16", anything else fp16."""
    return DTYPE_INT8 if s == "int8" else DTYPE_INT16 if s == "int16" else DTYPE_FP16


def load_quant_scales(pkg_dir: str | Path) -> dict[str, SubgraphScaleInfo]:
    """Every subgraph entry of the package, as the engine's load_quant_scales parses it.

    Missing numbers take parse_entry's defaults (thresholds 1.0, steps 1/127); the per-channel
    vectors are slices of the sidecar when both offsets are present and in range, else None.
    Entries parse_entry would reject (no input_threshold, or neither smoothing nor a threshold
    different from 1) are left out.
    """
    pkg = Path(pkg_dir)
    root = json.loads((pkg / "quant_scales.json").read_text())
    if not isinstance(root, dict) or "subgraphs" not in root:
        raise ValueError("quant_scales.json has no 'subgraphs'")
    side_path = pkg / "quant_chan_scales.bin"
    side = np.empty(0, np.float32)
    if side_path.exists() and side_path.stat().st_size % 4 == 0:
        side = np.fromfile(side_path, dtype=np.float32)
    out: dict[str, SubgraphScaleInfo] = {}
    for name, v in root["subgraphs"].items():
        if not isinstance(v, dict):
            continue
        info = SubgraphScaleInfo(
            in_dtype=parse_boundary_dtype(v.get("input_dtype", "fp16")),
            out_dtype=parse_boundary_dtype(v.get("output_dtype", "fp16")),
            in_thresh=float(np.float32(v.get("input_threshold", 1.0))),
            in_step=float(np.float32(v.get("input_step", 1.0 / 127.0))),
            out_thresh=float(np.float32(v.get("output_threshold", 1.0))),
            out_step=float(np.float32(v.get("output_step", 1.0 / 127.0))))
        if side.size and "in_smooth_offset" in v and "out_step_offset" in v:
            io, ic = int(v["in_smooth_offset"]), int(v.get("in_smooth_count", 0))
            oo, oc = int(v["out_step_offset"]), int(v.get("out_step_count", 0))
            if io + ic <= side.size and oo + oc <= side.size:
                info.in_inv_smooth = side[io:io + ic].copy()
                info.out_step_chan = side[oo:oo + oc].copy()
        if "input_threshold" in v and (info.in_inv_smooth is not None
                                       or abs(info.in_thresh - 1.0) > 1e-5):
            out[name] = info
    return out


def _untile(raw, rows: int, k: int, k_group: int, inner: int, dtype) -> np.ndarray:
    if rows % 8:
        raise ValueError("NVDLA weight slices hold a multiple of 8 output channels")
    k_pad = -(-k // k_group) * k_group
    a = np.frombuffer(bytes(raw) if not isinstance(raw, np.ndarray) else raw.tobytes(),
                      dtype=dtype)
    if a.size != rows * k_pad:
        raise ValueError(f"slice holds {a.size} elements, expected {rows} x {k_pad}")
    # tiled axes: (rows/8, k_pad/k_group, 3, 8 channel-in-group, 8 rows, inner)
    a = a.reshape(rows // 8, k_pad // k_group, 3, 8, 8, inner)
    return a.transpose(0, 4, 1, 2, 3, 5).reshape(rows, k_pad)[:, :k].copy()


def untile_int8(raw, rows: int, k: int) -> np.ndarray:
    """Row-major int8 [rows, k] from a tile_int8_slice image (K padded to 96, atoms of 3x8x4)."""
    return _untile(raw, rows, k, 96, 4, np.int8)


def untile_int16(raw, rows: int, k: int) -> np.ndarray:
    """Row-major int16 [rows, k] from a tile_int16_slice image (K padded to 48, atoms of 3x8x2)."""
    return _untile(raw, rows, k, 48, 2, np.int16)


def read_weight_region(region: bytes, offsets: list[int], n: int, k: int,
                       int16_weights: bool = False) -> tuple[np.ndarray, np.ndarray]:
    """(weights [n, k], QuantM int16 [n]) of one weight region.

    offsets: the template's content offsets, two per slice of 512 output channels (weights, then
    QuantM), as build_single_conv_region writes them (build_lfm3_int8_pkg.py:216-222).
    """
    n_slices = -(-n // SLICE_ROWS)
    if len(offsets) < 2 * n_slices:
        raise ValueError(f"{n} channels need {2 * n_slices} region offsets")
    elem = 2 if int16_weights else 1
    k_pad = -(-k // (48 if int16_weights else 96)) * (48 if int16_weights else 96)
    ws, qms = [], []
    buf = memoryview(region)
    for s in range(n_slices):
        rows = min(SLICE_ROWS, n - s * SLICE_ROWS)
        w_raw = buf[offsets[2 * s]:offsets[2 * s] + rows * k_pad * elem]
        ws.append(untile_int16(w_raw, rows, k) if int16_weights else untile_int8(w_raw, rows, k))
        qms.append(np.frombuffer(buf[offsets[2 * s + 1]:offsets[2 * s + 1] + rows * 2],
                                 dtype=np.int16).copy())
    return np.concatenate(ws), np.concatenate(qms)
