"""TEST INFRASTRUCTURE ONLY: numpy front end of the CPU oracle (liboracle.so) and of the
reference's own C++ compiled from its sources (_ref/libref.so).

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline legs use this module, and
only as the checker / the timed CPU baseline.  The product (romanaccio_b200) never imports it.
"""
from __future__ import annotations

import ctypes as C
import subprocess
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
ORACLE_LIB = HERE / "liboracle.so"
REF_LIB = HERE / "_ref" / "libref.so"

_P, _I32, _I64, _F = C.c_void_p, C.c_int32, C.c_int64, C.c_float
_ORACLE_SIGS = {
    "orc_round_clamp": (C.c_int32, [_F, _F]),
    "orc_pack_static": (None, [_P, _I64, _I32, _I32, _F, _P, _P, _I64]),
    "orc_pack_dyntok": (None, [_P, _I64, _I32, _I32, _F, _P, _P, _I64, _P]),
    "orc_gemm_i32": (None, [_P, _I64, _P, _I64, _I32, _I32, _I32, _P, _I64]),
    "orc_requant_one": (C.c_int32, [_I32, _I32, _I32, _I32]),
    "orc_requant_f64_one": (C.c_int32, [_I32, _I32, _I32, _I32]),
    "orc_requant": (None, [_P, _I64, _I32, _I32, _P, _I32, _I32, _P, _I64]),
    "orc_requant_f64": (None, [_P, _I64, _I32, _I32, _P, _I32, _I32, _P, _I64]),
    "orc_unpack": (None, [_P, _I64, _I32, _I32, _I32, _P, _P, _F, _P, _I64]),
    "orc_dequant_acc": (None, [_P, _I64, _I32, _I32, _I32, _P, _P, _P, _I64]),
    "orc_topk": (None, [_P, _I64, _I32, _I32, _I32, _I32, _P, _P]),
    "orc_argmax": (C.c_int32, [_P, _I32]),
    "orc_moe_route": (None, [_P, _I64, _I32, _I32, _P, _P, _I32, _I32, _I32, _F, _P, _P]),
    "orc_moe_combine": (None, [_P, _I32, _I32, _I32, _I32, _I32, _P, _P, _P, _P]),
    "orc_rmsnorm_pack_dyntok": (None, [_P, _I64, _I32, _I32, _P, _P, _F, _F, _P, _I64, _P, _P,
                                       _I64]),
    "orc_post_op_ffn_pack": (None, [_P, _I64, _P, _P, _I64, _I32, _I32, _P, _F, _P, _I64, _P,
                                    _I64]),
    "orc_emb_norm_pack": (None, [_P, _I64, _I32, _I32, _P, _F, _P, _I64]),
    "orc_gemm_i16_requant": (None, [_P, _I64, _P, _I64, _I32, _I32, _I32, _P, _I32, _P, _I64]),
    "orc_num_threads": (C.c_int, []),
    "orc_set_threads": (None, [C.c_int]),
    "orc_linear_dyntok_omp": (None, [_P, _I32, _I32, _I32, _P, _P, _F, _P, _I32, _P, _P, _P, _P]),
    "orc_lmhead_topk_omp": (None, [_P, _I32, _I32, _I32, _P, _F, _P, _I32, _P, _P, _P, _P]),
    "orc_lmhead_topk_norm_omp": (None, [_P, _I32, _I32, _I32, _P, _P, _F, _P, _I32, _P, _P, _P,
                                        _P]),
    "orc_gemm_requant_omp": (None, [_P, _I32, _I32, _I32, _P, _P, _I32, _P]),
}
_REF_SIGS = {
    "ref_round_clamp_f32": (C.c_int32, [_F, _F]),
    "ref_pack_int8": (C.c_int, [_P, C.c_int, C.c_int, _F, _P, _P]),
    "ref_pack_int8_dyntok": (C.c_int, [_P, C.c_int, C.c_int, _F, _P, _P, _P]),
    "ref_unpack_int8": (C.c_int, [_P, C.c_int, C.c_int, _F, _P, _P, _P]),
    "ref_unpack_int16": (C.c_int, [_P, C.c_int, C.c_int, _F, _P, _P]),
    "ref_sampler_greedy": (C.c_int32, [_P, C.c_size_t]),
    "ref_rmsnorm_pack_dyntok": (C.c_int, [_P, C.c_int, _P, _P, _F, _F, _P, _P, _P]),
    "ref_post_op_ffn_pack": (C.c_int, [_P, _P, _P, _P, _P, _P, C.c_int, _F]),
    "ref_emb_norm_pack": (C.c_int, [_P, C.c_int, _P, _F, _P]),
    "ref_session_create": (_P, [C.c_int, C.c_int, _P]),
    "ref_session_lm_head": (C.c_int, [_P, _P, _P]),
    "ref_session_destroy": (None, [_P]),
    "ref_sampler_run": (C.c_int, [_F, C.c_int, _F, _F, _F, C.c_int, C.c_int, C.c_uint, _P,
                                  C.c_int, _P, C.c_int, C.c_size_t, _P]),
    "ref_moe_route": (C.c_int, [_P, C.c_int, C.c_int, _P, _P, C.c_int, C.c_int, C.c_int, _F, _P, _P]),
}

_orc = None
_ref = None


def build() -> None:
    """Builds liboracle.so (and _ref/libref.so when the reference tree is present)."""
    subprocess.run(["make", "-s", "-C", str(HERE)], check=True)


def _bind(path: Path, sigs: dict) -> C.CDLL:
    lib = C.CDLL(str(path))
    for name, (res, args) in sigs.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    return lib


def lib() -> C.CDLL:
    global _orc
    if _orc is None:
        if not ORACLE_LIB.exists():
            build()
        _orc = _bind(ORACLE_LIB, _ORACLE_SIGS)
    return _orc


def ref_available() -> bool:
    return REF_LIB.exists()


def ref() -> C.CDLL:
    global _ref
    if _ref is None:
        if not REF_LIB.exists():
            raise FileNotFoundError(f"{REF_LIB} was not built (needs the reference tree)")
        _ref = _bind(REF_LIB, _REF_SIGS)
    return _ref


def _p(a: np.ndarray | None):
    return None if a is None else a.ctypes.data


def _c(a, dtype):
    return None if a is None else np.ascontiguousarray(a, dtype=dtype)


# ------------------------------------------------------------------ restatement (liboracle)
def round_clamp(x: float, lim: float = 127.0) -> int:
    return int(lib().orc_round_clamp(x, lim))


def pack_static(x: np.ndarray, in_step: float, inv_smooth: np.ndarray | None = None) -> np.ndarray:
    x = _c(x, np.float32)
    T, K = x.shape
    s = _c(inv_smooth, np.float32)
    q = np.empty((T, K), np.int8)
    lib().orc_pack_static(_p(x), K, T, K, in_step, _p(s), _p(q), K)
    return q


def pack_dyntok(x: np.ndarray, in_thresh: float, inv_smooth: np.ndarray | None = None):
    x = _c(x, np.float32)
    T, K = x.shape
    s = _c(inv_smooth, np.float32)
    q = np.empty((T, K), np.int8)
    r = np.empty((T,), np.float32)
    lib().orc_pack_dyntok(_p(x), K, T, K, in_thresh, _p(s), _p(q), K, _p(r))
    return q, r


def gemm_i32(q: np.ndarray, w: np.ndarray) -> np.ndarray:
    q = _c(q, np.int8)
    w = _c(w, np.int8)
    T, K = q.shape
    N = w.shape[0]
    acc = np.empty((T, N), np.int32)
    lib().orc_gemm_i32(_p(q), K, _p(w), K, T, N, K, _p(acc), N)
    return acc


def requant(acc: np.ndarray, quant_m: np.ndarray, trunc: int, qmax: int = 127,
            f64: bool = False) -> np.ndarray:
    acc = _c(acc, np.int32)
    qm = _c(quant_m, np.int16)
    T, N = acc.shape
    yq = np.empty((T, N), np.int32)
    fn = lib().orc_requant_f64 if f64 else lib().orc_requant
    fn(_p(acc), N, T, N, _p(qm), trunc, qmax, _p(yq), N)
    return yq


def unpack(yq: np.ndarray, out_step: float, out_step_chan: np.ndarray | None = None,
           ratio: np.ndarray | None = None) -> np.ndarray:
    yq = _c(yq, np.int32)
    T, N = yq.shape
    osc = _c(out_step_chan, np.float32)
    r = _c(ratio, np.float32)
    y = np.empty((T, N), np.float32)
    lib().orc_unpack(_p(yq), N, T, N, 1 if r is not None else 0, _p(r), _p(osc), out_step, _p(y), N)
    return y


def dequant_acc(acc: np.ndarray, acc_step: np.ndarray, ratio: np.ndarray | None = None) -> np.ndarray:
    acc = _c(acc, np.int32)
    T, N = acc.shape
    st = _c(acc_step, np.float32)
    r = _c(ratio, np.float32)
    y = np.empty((T, N), np.float32)
    lib().orc_dequant_acc(_p(acc), N, T, N, 1 if r is not None else 0, _p(r), _p(st), _p(y), N)
    return y


def topk(logits: np.ndarray, k: int, id_offset: int = 0):
    lg = _c(logits, np.float32)
    T, V = lg.shape
    val = np.empty((T, k), np.float32)
    idx = np.empty((T, k), np.int32)
    lib().orc_topk(_p(lg), V, T, V, k, id_offset, _p(val), _p(idx))
    return val, idx


def argmax(logits_row: np.ndarray) -> int:
    lg = _c(logits_row, np.float32)
    return int(lib().orc_argmax(_p(lg), lg.shape[0]))


def moe_route(hidden: np.ndarray, gate_w: np.ndarray, k: int, bias: np.ndarray | None = None,
              norm_topk: bool = False, scaling: float = 1.0):
    """MoERouter::route for every row of hidden [T, H]: (expert ids [T, k], weights [T, k])."""
    h = _c(hidden, np.float32)
    gw = _c(gate_w, np.float32)
    b = _c(bias, np.float32)
    T, H = h.shape
    E = gw.shape[0]
    idx = np.empty((T, k), np.int32)
    w = np.empty((T, k), np.float32)
    lib().orc_moe_route(_p(h), H, T, H, _p(gw), _p(b), E, k, int(norm_topk), float(scaling),
                        _p(idx), _p(w))
    return idx, w


def moe_combine(yq: np.ndarray, idx: np.ndarray, w: np.ndarray, out_step_chan: np.ndarray,
                n_routed: int, slots: int) -> np.ndarray:
    """Weighted combine of the experts' requantised outputs yq [T*slots, H] into [T, H]."""
    y = _c(yq, np.int32)
    ix = _c(idx, np.int32)
    ww = _c(w, np.float32)
    osc = _c(out_step_chan, np.float32)
    T, k = ix.shape
    H = y.shape[1]
    out = np.empty((T, H), np.float32)
    lib().orc_moe_combine(_p(y), T, k, slots, n_routed, H, _p(ix), _p(ww), _p(osc), _p(out))
    return out


def moe_combine_ep(yq: np.ndarray, idx: np.ndarray, w: np.ndarray, out_step_chan: np.ndarray,
                   n_routed: int, slots: int, world: int) -> np.ndarray:
    """The expert-parallel combine: rank r sums, in slot order from 0.0f, the slots whose
    expert e has e % world == r (shared expert s is e = n_routed + s), each term
    float(yq) * (w * out_step_chan[e]) in fp32 as moe_combine; the layer output is the ranks'
    partials added in rank order from 0.0f (the reference's per-die sums added die after die,
    src/LFM2.5-8B-A1B/lfm2_moe.cpp:2190-2432, for world = 2)."""
    y = np.asarray(yq).astype(np.float32)
    ix = np.asarray(idx, np.int32)
    ww = np.asarray(w, np.float32)
    osc = np.asarray(out_step_chan, np.float32)
    T, k = ix.shape
    H = y.shape[1]
    out = np.zeros((T, H), np.float32)
    for r in range(world):
        part = np.zeros((T, H), np.float32)
        for t in range(T):
            for j in range(slots):
                e = int(ix[t, j]) if j < k else n_routed + (j - k)
                if e % world != r:
                    continue
                wj = ww[t, j] if j < k else np.float32(1.0)
                part[t] = part[t] + y[t * slots + j] * (np.float32(wj) * osc[e])
        out = out + part
    return out


def rmsnorm_pack_dyntok(h: np.ndarray, norm: np.ndarray, smooth: np.ndarray, in_thresh: float,
                        eps: float = 1e-5):
    """fused_rms_norm_pack_dyntok_t1 per row of h [T, C] -> (q [T, C], ratio [T], u_out [T, C])."""
    hh = _c(h, np.float32)
    T, Cn = hh.shape
    q = np.empty((T, Cn), np.int8)
    ratio = np.empty(T, np.float32)
    u = np.empty((T, Cn), np.float32)
    lib().orc_rmsnorm_pack_dyntok(_p(hh), Cn, T, Cn, _p(_c(norm, np.float32)),
                                  _p(_c(smooth, np.float32)), float(in_thresh), float(eps), _p(q),
                                  Cn, _p(ratio), _p(u), Cn)
    return q, ratio, u


def gemm_i16_requant(x: np.ndarray, w: np.ndarray, quant_m: np.ndarray, trunc: int) -> np.ndarray:
    """The MLP's w2 stage: int16 x [T, K] against int16 codes w [N, K], QuantM requant to int16."""
    xx = _c(x, np.int16)
    ww = _c(w, np.int16)
    T, K = xx.shape
    N = ww.shape[0]
    y = np.empty((T, N), np.int16)
    lib().orc_gemm_i16_requant(_p(xx), K, _p(ww), K, T, K, N, _p(_c(quant_m, np.int16)), int(trunc),
                               _p(y), N)
    return y


def emb_norm_pack(h: np.ndarray, emb_norm_scaled: np.ndarray, eps: float = 1e-5) -> np.ndarray:
    """fused_emb_norm_broadcast_t1 per row of h [T, C] -> q [T, C] int8."""
    hh = _c(h, np.float32)
    T, Cn = hh.shape
    q = np.empty((T, Cn), np.int8)
    lib().orc_emb_norm_pack(_p(hh), Cn, T, Cn, _p(_c(emb_norm_scaled, np.float32)), float(eps),
                            _p(q), Cn)
    return q


def ref_emb_norm_pack(h_row: np.ndarray, emb_norm_scaled: np.ndarray, eps: float = 1e-5):
    """The reference's fused_emb_norm_broadcast_t1 on one row (compiled from its source)."""
    hh = _c(h_row, np.float32)
    q = np.empty(hh.shape[0], np.int8)
    rc = ref().ref_emb_norm_pack(_p(hh), hh.shape[0], _p(_c(emb_norm_scaled, np.float32)),
                                 float(eps), _p(q))
    if rc != 0:
        raise RuntimeError(f"ref_emb_norm_pack returned {rc}")
    return q


def post_op_ffn_pack(op_out: np.ndarray, post_norm: np.ndarray, h: np.ndarray,
                     ffn_scaled: np.ndarray, eps: float = 1e-5):
    """fused_post_op_residual_ffn_pack_mlp_t1 per row -> (h_mid [T, C], q [T, C])."""
    o = _c(op_out, np.float32)
    hh = _c(h, np.float32)
    T, Cn = o.shape
    m = np.empty((T, Cn), np.float32)
    q = np.empty((T, Cn), np.int8)
    lib().orc_post_op_ffn_pack(_p(o), Cn, _p(_c(post_norm, np.float32)), _p(hh), Cn, T, Cn,
                               _p(_c(ffn_scaled, np.float32)), float(eps), _p(m), Cn, _p(q), Cn)
    return m, q


def ref_rmsnorm_pack_dyntok(h_row, norm, smooth, in_thresh: float, eps: float = 1e-5):
    hh = _c(h_row, np.float32)
    Cn = hh.shape[0]
    q = np.empty(Cn, np.int8)
    ratio = np.empty(1, np.float32)
    u = np.empty(Cn, np.float32)
    assert ref().ref_rmsnorm_pack_dyntok(_p(hh), Cn, _p(_c(norm, np.float32)),
                                         _p(_c(smooth, np.float32)), float(in_thresh), float(eps),
                                         _p(q), _p(ratio), _p(u)) == 0
    return q, ratio[0], u


def ref_post_op_ffn_pack(op_row, post_norm, h_row, ffn_scaled, eps: float = 1e-5):
    o = _c(op_row, np.float32)
    Cn = o.shape[0]
    m = np.empty(Cn, np.float32)
    q = np.empty(Cn, np.int8)
    assert ref().ref_post_op_ffn_pack(_p(o), _p(_c(post_norm, np.float32)), _p(_c(h_row, np.float32)),
                                      _p(m), _p(_c(ffn_scaled, np.float32)), _p(q), Cn,
                                      float(eps)) == 0
    return m, q


def linear(x: np.ndarray, wq: np.ndarray, quant_m: np.ndarray, trunc: int, out_step_chan: np.ndarray,
           inv_smooth: np.ndarray | None, in_thresh: float | None = None, in_step: float | None = None,
           out_step: float = 0.0, qmax: int = 127):
    """Full boundary: pack (dyntok when in_thresh is given, else static) -> GEMM -> requant ->
    unpack.  Returns (q, ratio or None, acc, yq, y)."""
    if in_thresh is not None:
        q, r = pack_dyntok(x, in_thresh, inv_smooth)
    else:
        q, r = pack_static(x, in_step, inv_smooth), None
    acc = gemm_i32(q, wq)
    yq = requant(acc, quant_m, trunc, qmax)
    y = unpack(yq, out_step, out_step_chan, r)
    return q, r, acc, yq, y


# ------------------------------------------------------------------ reference C++ (_ref)
def ref_round_clamp(x: float, lim: float = 127.0) -> int:
    return int(ref().ref_round_clamp_f32(x, lim))


def ref_pack(x: np.ndarray, in_step: float, inv_smooth: np.ndarray | None = None) -> np.ndarray:
    x = _c(x, np.float32)
    T, K = x.shape
    s = _c(inv_smooth, np.float32)
    q = np.empty((T, K), np.int8)
    assert ref().ref_pack_int8(_p(x), T, K, in_step, _p(s), _p(q)) == 0
    return q


def ref_pack_dyntok(x: np.ndarray, in_thresh: float, inv_smooth: np.ndarray | None = None):
    x = _c(x, np.float32)
    T, K = x.shape
    s = _c(inv_smooth, np.float32)
    q = np.empty((T, K), np.int8)
    r = np.empty((max(T, 1),), np.float32)
    assert ref().ref_pack_int8_dyntok(_p(x), T, K, in_thresh, _p(s), _p(q), _p(r)) == 0
    return q, r[:T]


def ref_unpack(yq: np.ndarray, out_step: float, out_step_chan: np.ndarray | None = None,
               ratio: np.ndarray | None = None) -> np.ndarray:
    yq = _c(yq, np.int8)
    T, N = yq.shape
    osc = _c(out_step_chan, np.float32)
    r = _c(ratio, np.float32)
    y = np.empty((T, N), np.float32)
    assert ref().ref_unpack_int8(_p(yq), T, N, out_step, _p(osc), _p(r), _p(y)) == 0
    return y


def ref_unpack_i16(yq: np.ndarray, out_step: float, out_step_chan: np.ndarray | None = None) -> np.ndarray:
    yq = _c(yq, np.int16)
    T, N = yq.shape
    osc = _c(out_step_chan, np.float32)
    y = np.empty((T, N), np.float32)
    assert ref().ref_unpack_int16(_p(yq), T, N, out_step, _p(osc), _p(y)) == 0
    return y


def ref_greedy(logits_row: np.ndarray) -> int:
    lg = np.array(logits_row, dtype=np.float32, copy=True)
    return int(ref().ref_sampler_greedy(_p(lg), lg.shape[0]))


def ref_sampler_run(params: dict, history, logits: np.ndarray) -> np.ndarray:
    """The reference Sampler (sampler.cpp:83-179) over S steps of full logits [S, V]: accepts
    `history`, then samples each step and accepts the sampled token."""
    lg = np.ascontiguousarray(logits, dtype=np.float32)
    S, V = lg.shape
    h = np.ascontiguousarray(np.asarray(history, dtype=np.int32))
    out = np.empty(S, np.int32)
    assert ref().ref_sampler_run(
        params["temperature"], params["top_k"], params["top_p"], params["min_p"],
        params["repeat_penalty"], params["repeat_window"], params["max_consecutive_duplicates"],
        params["seed"], _p(h), h.shape[0], _p(lg), S, V, _p(out)) == 0
    return out


def ref_moe_route(hidden: np.ndarray, gate_w: np.ndarray, k: int, bias: np.ndarray | None = None,
                  norm_topk: bool = False, scaling: float = 1.0):
    """The reference's MoERouter::route (compiled from its sources) on every row of hidden."""
    h = _c(hidden, np.float32)
    gw = _c(gate_w, np.float32)
    b = _c(bias, np.float32)
    T, H = h.shape
    idx = np.empty((T, k), np.int32)
    w = np.empty((T, k), np.float32)
    rc = ref().ref_moe_route(_p(h), T, H, _p(gw), _p(b), gw.shape[0], k, int(norm_topk),
                             float(scaling), _p(idx), _p(w))
    if rc != 0:
        raise RuntimeError(f"ref_moe_route failed ({rc})")
    return idx, w


class DecodeOracle:
    """One decode step of a linear stack + LM head through the oracle's OpenMP C restatement
    (src/LFM3/lfm3_v2.cpp pack / unpack, cmac.py:300-383 GEMM, attribute_int8_error.py:104-122
    requant; the same arithmetic as the CUDA path): dyntok pack -> int32 GEMM -> QuantM requant ->
    unpack per linear, each linear reading the previous one's output (o the q slice of qkv, down
    the gate slice of gate_up), then the LM head with its top-k: lm = (wq, acc_step, in_step) for
    a static pack, or (wq, acc_step, in_step, emb_norm_scaled, eps) for the RMSNorm pack of
    fused_emb_norm_broadcast_t1 (src/LFM3/lfm3_v2.cpp:810-831).  Used as the checker of the GPU
    step and, timed, as the CPU baseline."""

    def __init__(self, params, lm, T: int, shape, k: int = 40):
        import os
        self.C = C
        self.lib = lib()
        # every host core this process may run on (launchers such as torchrun export
        # OMP_NUM_THREADS=1 to their workers)
        self.lib.orc_set_threads(len(os.sched_getaffinity(0)))
        self.cores = int(self.lib.orc_num_threads())
        self.T, self.shape, self.k = T, shape, k
        self.bufs = {name: np.empty((T, N), np.float32) for (name, K, N, _) in shape.subgraphs()}
        self.qbuf = np.empty((T, max(kk for (_, kk, _, _) in shape.subgraphs())), np.int8)
        self.ratio = np.empty((T,), np.float32)
        self.wq_lm, self.acc_step_lm, self.in_step_lm = lm[:3]
        self.emb_lm = (np.ascontiguousarray(lm[3], np.float32), float(lm[4])) if len(lm) > 3 else None
        V = self.wq_lm.shape[0]
        self.logits = np.empty((T, V), np.float32)
        self.val = np.empty((T, k), np.float32)
        self.idx = np.empty((T, k), np.int32)
        self.qlm = np.empty((T, shape.hidden), np.int8)
        self.prepared = []
        for name, prm in params:
            self.prepared.append((name, prm.wq.shape[1], prm.wq.shape[0], np.ascontiguousarray(prm.wq),
                                  np.ascontiguousarray(prm.in_inv_smooth, np.float32), prm.in_thresh,
                                  np.ascontiguousarray(prm.quant_m), prm.trunc,
                                  np.ascontiguousarray(prm.out_step_chan, np.float32)))

    def run(self, x0: np.ndarray):
        """Returns (final hidden state [T, hidden], top-k values [T, k], top-k ids [T, k])."""
        C, lib, shape, bufs = self.C, self.lib, self.shape, self.bufs

        def p(a):
            return a.ctypes.data

        x = np.ascontiguousarray(x0, dtype=np.float32)
        for (name, K, N, wq, inv, thr, qm, tr, osc) in self.prepared:
            if name == "o":
                x = np.ascontiguousarray(bufs["qkv"][:, :shape.q])
            elif name == "down":
                x = np.ascontiguousarray(bufs["gate_up"][:, :shape.ffn])
            elif name == "gate_up":
                x = bufs["o"]
            y = bufs[name]
            lib.orc_linear_dyntok_omp(p(x), self.T, K, N, p(wq), p(inv), C.c_float(thr), p(qm),
                                      tr, p(osc), p(y), p(self.qbuf), p(self.ratio))
            x = bufs["down"] if name == "down" else x
        V = self.wq_lm.shape[0]
        if self.emb_lm is not None:
            lib.orc_lmhead_topk_norm_omp(p(bufs["down"]), self.T, shape.hidden, V, p(self.wq_lm),
                                         p(self.emb_lm[0]), C.c_float(self.emb_lm[1]),
                                         p(self.acc_step_lm), self.k, p(self.logits),
                                         p(self.qlm), p(self.val), p(self.idx))
        else:
            lib.orc_lmhead_topk_omp(p(bufs["down"]), self.T, shape.hidden, V, p(self.wq_lm),
                                    C.c_float(self.in_step_lm), p(self.acc_step_lm), self.k,
                                    p(self.logits), p(self.qlm), p(self.val), p(self.idx))
        return bufs["down"].copy(), self.val.copy(), self.idx.copy()


class ReferenceDecode:
    """One decode step through the reference's own C++ wherever the reference has CPU code for it
    (TIMED BASELINE ONLY, compiled from its sources into _ref/libref.so): per linear its
    pack_npu_input_int8_dyntok (src/LFM3/lfm3_v2.cpp:1050-1141, OpenMP), the NPU's int8 GEMM and
    QuantM requant (no CPU code in the reference: the C restatement, OpenMP) and its
    unpack_npu_output_int8_dyntok (:1143-1183); then TransformerSession's host LM head
    (transformer_session.cpp:597-612, fp32 rows, OpenMP) and Sampler::sample (sampler.cpp:83-179,
    greedy) over the whole vocabulary.  params / lm as DecodeOracle; the LM head runs on the fp32
    rows wq * w_step (what its host fallback holds)."""

    def __init__(self, params, lm_f32_rows: np.ndarray, T: int, shape):
        import os
        self.C = C
        self.lib, self.ref = lib(), ref()
        self.lib.orc_set_threads(len(os.sched_getaffinity(0)))
        self.cores = int(self.lib.orc_num_threads())
        if T != 1:
            raise ValueError("the reference's host LM head takes one hidden state per call")
        self.T, self.shape = T, shape
        self.bufs = {name: np.empty((T, N), np.float32) for (name, K, N, _) in shape.subgraphs()}
        self.q = np.empty((T, max(kk for (_, kk, _, _) in shape.subgraphs())), np.int8)
        self.yq = np.empty((T, max(n for (_, _, n, _) in shape.subgraphs())), np.int8)
        self.ratio = np.empty((T,), np.float32)
        V, K = lm_f32_rows.shape
        w = np.ascontiguousarray(lm_f32_rows, np.float32)
        self.session = self.ref.ref_session_create(K, V, _p(w))
        self.logits = np.empty(V, np.float32)
        self.V = V
        self.prepared = [(name, prm.wq.shape[1], prm.wq.shape[0], np.ascontiguousarray(prm.wq),
                          np.ascontiguousarray(prm.in_inv_smooth, np.float32), prm.in_thresh,
                          np.ascontiguousarray(prm.quant_m), prm.trunc,
                          np.ascontiguousarray(prm.out_step_chan, np.float32))
                         for name, prm in params]
        self.seconds = {"pack": 0.0, "gemm_requant": 0.0, "unpack": 0.0, "lm_head": 0.0,
                        "sampler": 0.0}

    def run(self, x0: np.ndarray) -> int:
        import time
        ref, lib, shape, bufs, clk = self.ref, self.lib, self.shape, self.bufs, time.perf_counter
        x = np.ascontiguousarray(x0, dtype=np.float32)
        for (name, K, N, wq, inv, thr, qm, tr, osc) in self.prepared:
            if name == "o":
                x = np.ascontiguousarray(bufs["qkv"][:, :shape.q])
            elif name == "down":
                x = np.ascontiguousarray(bufs["gate_up"][:, :shape.ffn])
            elif name == "gate_up":
                x = bufs["o"]
            t0 = clk()
            ref.ref_pack_int8_dyntok(_p(x), self.T, K, float(thr), _p(inv), _p(self.q), _p(self.ratio))
            t1 = clk()
            lib.orc_gemm_requant_omp(_p(self.q), self.T, K, N, _p(wq), _p(qm), tr, _p(self.yq))
            t2 = clk()
            ref.ref_unpack_int8(_p(self.yq), self.T, N, 0.0, _p(osc), _p(self.ratio), _p(bufs[name]))
            t3 = clk()
            self.seconds["pack"] += t1 - t0
            self.seconds["gemm_requant"] += t2 - t1
            self.seconds["unpack"] += t3 - t2
            x = bufs["down"] if name == "down" else x
        t0 = clk()
        ref.ref_session_lm_head(self.session, _p(bufs["down"]), _p(self.logits))
        t1 = clk()
        tok = int(ref.ref_sampler_greedy(_p(self.logits), self.V))
        self.seconds["sampler"] += clk() - t1
        self.seconds["lm_head"] += t1 - t0
        return tok

    def close(self) -> None:
        if getattr(self, "session", None):
            self.ref.ref_session_destroy(self.session)
            self.session = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

