"""numpy front of the CPU oracle (liboracle.so) — TEST INFRASTRUCTURE ONLY.

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg import
this module, as the checker; the product path (kern-k3-pp-prefill_b200/k3moe.py
over libk3moe.so) never does.  See k3oracle.h for what each function restates.
"""
from __future__ import annotations

import ctypes
import os

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB = os.path.join(HERE, "liboracle.so")
REF_DIR = os.path.join(HERE, "_ref")

_lib = None


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(LIB):
            raise RuntimeError(f"{LIB} missing: run `make -C oracle`")
        _lib = ctypes.CDLL(LIB)
        _lib.orc_mx8_exponent.restype = ctypes.c_int
        _lib.orc_mx8_exponent.argtypes = [ctypes.c_float]
        _lib.orc_mx8_exponent_ocp.restype = ctypes.c_int
        _lib.orc_mx8_exponent_ocp.argtypes = [ctypes.c_float]
        _lib.orc_f32_to_e4m3_sat.restype = ctypes.c_uint8
        _lib.orc_f32_to_e4m3_sat.argtypes = [ctypes.c_float]
        _lib.orc_e4m3_to_f32.restype = ctypes.c_float
        _lib.orc_e4m3_to_f32.argtypes = [ctypes.c_uint8]
        _lib.orc_set_threads.restype = ctypes.c_int
        _lib.orc_set_threads.argtypes = [ctypes.c_int]
        _lib.orc_synth_f32.argtypes = [ctypes.c_uint64, ctypes.c_longlong, ctypes.c_longlong, ctypes.c_int,
                                       ctypes.c_float, ctypes.c_void_p]
        _lib.orc_quant_mxfp4.argtypes = [ctypes.c_void_p, ctypes.c_longlong, ctypes.c_int, ctypes.c_void_p,
                                         ctypes.c_void_p]
    return _lib


def _p(a: np.ndarray):
    assert a.flags["C_CONTIGUOUS"], "oracle arrays must be C-contiguous"
    return ctypes.c_void_p(a.ctypes.data)


def bf16_bits(x_f32: np.ndarray) -> np.ndarray:
    """f32 -> bf16 bit patterns (round to nearest even)."""
    u = np.ascontiguousarray(x_f32, dtype=np.float32).view(np.uint32).astype(np.uint64)
    u = u + 0x7FFF + ((u >> 16) & 1)
    return (u >> 16).astype(np.uint16)


def bf16_to_f32(b: np.ndarray) -> np.ndarray:
    return (np.ascontiguousarray(b, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


def set_threads(n: int = 0) -> int:
    return lib().orc_set_threads(n)


def topk(S: np.ndarray, bias: np.ndarray, rs_bits: int, K: int):
    S = np.ascontiguousarray(S, dtype=np.float32)
    T, E = S.shape
    idx = np.empty((T, K), np.int32)
    wts = np.empty((T, K), np.float32)
    lib().orc_topk(_p(S), ctypes.c_int(E), _p(np.ascontiguousarray(bias, np.float32)), ctypes.c_uint16(rs_bits),
                   ctypes.c_int(T), ctypes.c_int(E), ctypes.c_int(K), _p(idx), _p(wts))
    return idx, wts


def max_ctas(R, K, E, shared, tile=128):
    rows = R * K + (R if shared else 0)
    return E + (1 if shared else 0) + -(-rows // tile)


def tables(idx: np.ndarray, E: int, first: int = 0, shared: int = 0, tile: int = 128):
    idx = np.ascontiguousarray(idx, np.int32)
    R, K = idx.shape
    mc = max_ctas(R, K, E, shared, tile)
    out = dict(
        counts=np.zeros(E + shared, np.int32),
        cta_batch=np.full(mc, -7, np.int32),
        cta_limit=np.full(mc, -7, np.int32),
        meta=np.zeros(4, np.int32),
        route_map=np.full(mc * tile, -7, np.int32),
        exp2perm=np.empty((R, K), np.int32),
    )
    lib().orc_tables(_p(idx), R, K, first, E, shared, tile, _p(out["counts"]), _p(out["cta_batch"]),
                     _p(out["cta_limit"]), _p(out["meta"]), _p(out["route_map"]), _p(out["exp2perm"]))
    out["max_ctas"] = mc
    out["cap_rows"] = mc * tile
    return out


def quant_mxfp8(x_bits: np.ndarray, tiled: bool = False):
    x_bits = np.ascontiguousarray(x_bits, np.uint16)
    rows, cols = x_bits.shape
    q = np.empty((rows, cols), np.uint8)
    sf = (np.zeros(-(-rows // 128) * -(-cols // 128) * 512, np.uint8) if tiled
          else np.empty((rows, cols // 32), np.uint8))
    lib().orc_quant_mxfp8(_p(x_bits), cols, rows, cols, _p(q), _p(sf), int(tiled))
    return q, sf


def quant_permute(x_bits: np.ndarray, exp2perm: np.ndarray, meta: np.ndarray, cap_rows: int):
    x_bits = np.ascontiguousarray(x_bits, np.uint16)
    R, H = x_bits.shape
    K = exp2perm.shape[1]
    qp = np.zeros((cap_rows, H), np.uint8)
    sfp = np.zeros(cap_rows * H // 32, np.uint8)
    lib().orc_quant_permute(_p(x_bits), H, R, H, K, _p(np.ascontiguousarray(exp2perm, np.int32)),
                            _p(np.ascontiguousarray(meta, np.int32)), _p(qp), _p(sfp))
    return qp, sfp


def quant_mxfp4(w: np.ndarray):
    w = np.ascontiguousarray(w, np.float32)
    rows, K = w.shape
    packed = np.empty((rows, K // 2), np.uint8)
    sf = np.zeros(-(-rows // 128) * (K // 128) * 512, np.uint8)
    lib().orc_quant_mxfp4(_p(w), rows, K, _p(packed), _p(sf))
    return packed, sf


def synth_f32(seed: int, rows: int, K: int, sd: float, row0: int = 0):
    out = np.empty((rows, K), np.float32)
    lib().orc_synth_f32(seed, row0, rows, K, sd, _p(out))
    return out


def combine(fc2_bits, exp2perm, wts, meta, T, K, out_rows=None):
    fc2_bits = np.ascontiguousarray(fc2_bits, np.uint16)
    cols = fc2_bits.shape[1]
    out_rows = out_rows or T
    out = np.empty((out_rows, cols), np.uint16)
    meta_p = _p(np.ascontiguousarray(meta, np.int32)) if meta is not None else None
    lib().orc_combine(_p(fc2_bits), _p(np.ascontiguousarray(exp2perm, np.int32)),
                      _p(np.ascontiguousarray(wts, np.float32)), meta_p, _p(out), cols, T, out_rows, K, cols)
    return out


def fc1(w13, w13_sf, qp, sfp, cta_batch, cta_limit, c0, c1, H, I, out_q=None, out_sf=None, act=0):
    """act: 0 SwiGLU, 1 K3's SiTU."""
    cap = qp.shape[0]
    out_q = np.zeros((cap, I), np.uint8) if out_q is None else out_q
    out_sf = np.zeros(cap * I // 32, np.uint8) if out_sf is None else out_sf
    lib().orc_fc1_act(_p(w13), _p(w13_sf), _p(qp), _p(sfp), _p(np.ascontiguousarray(cta_batch, np.int32)),
                      _p(np.ascontiguousarray(cta_limit, np.int32)), c0, c1, H, I, _p(out_q), _p(out_sf), act)
    return out_q, out_sf


def fc2(w2, w2_sf, fc1_q, fc1_sf, cta_batch, cta_limit, c0, c1, H, I, out=None):
    cap = fc1_q.shape[0]
    out = np.zeros((cap, H), np.uint16) if out is None else out
    lib().orc_fc2(_p(w2), _p(w2_sf), _p(fc1_q), _p(fc1_sf), _p(np.ascontiguousarray(cta_batch, np.int32)),
                  _p(np.ascontiguousarray(cta_limit, np.int32)), c0, c1, H, I, _p(out))
    return out


E4M3_TABLE = None


def e4m3_to_f32(q: np.ndarray) -> np.ndarray:
    global E4M3_TABLE
    if E4M3_TABLE is None:
        E4M3_TABLE = np.array([lib().orc_e4m3_to_f32(i) for i in range(256)], np.float32)
    return E4M3_TABLE[q]


def t128_rows(buf: np.ndarray, rows, K: int) -> np.ndarray:
    """Rows of a tile-major E4M3 operand (128 x 128 tiles, see k3oracle.h) as row-major [len(rows), K]."""
    flat = np.ascontiguousarray(buf).reshape(-1)
    r = np.asarray(rows, np.int64)[:, None]
    k = np.arange(K, dtype=np.int64)[None, :]
    off = ((r // 128) * (K // 128) + k // 128) * 16384 + (r % 128) * 128 + k % 128
    return flat[off]


def dequant_rows(q: np.ndarray, sf_tiled: np.ndarray, rows: np.ndarray) -> np.ndarray:
    """MXFP8 rows of a tile-major operand (tiled scales) -> f32 [len(rows), cols]."""
    cols = q.shape[1]
    kbn, kg4 = cols // 32, -(-cols // 128)
    r = rows.astype(np.int64)[:, None]
    kb = np.arange(kbn, dtype=np.int64)[None, :]
    off = ((r // 128) * kg4 + kb // 4) * 512 + (r % 32) * 16 + ((r % 128) // 32) * 4 + kb % 4
    s = np.ldexp(np.float32(1.0), sf_tiled[off].astype(np.int32) - 127).astype(np.float32)
    v = e4m3_to_f32(t128_rows(q, rows, cols)).reshape(len(rows), kbn, 32)
    return (v * s[:, :, None]).reshape(len(rows), cols)


def moe_forward(S, bias, rs_bits, x_bits, w13, w13_sf, w2, w2_sf, E, K, H, I, shared, act=0):
    """The whole layer on the CPU (small configs): returns (out bf16 bits, intermediates)."""
    T = x_bits.shape[0]
    idx, wts = topk(S, bias, rs_bits, K)
    tb = tables(idx, E, 0, shared)
    qp, sfp = quant_permute(x_bits, tb["exp2perm"], tb["meta"], tb["cap_rows"])
    nne = int(tb["meta"][0])
    f1q, f1sf = fc1(w13, w13_sf, qp, sfp, tb["cta_batch"], tb["cta_limit"], 0, nne, H, I, act=act)
    y = fc2(w2, w2_sf, f1q, f1sf, tb["cta_batch"], tb["cta_limit"], 0, nne, H, I)
    out = combine(y, tb["exp2perm"], wts, tb["meta"], T, K)
    return out, dict(idx=idx, wts=wts, tables=tb, q_perm=qp, sf_perm=sfp, fc1_q=f1q, fc1_sf=f1sf, fc2=y)


def situ(g: np.ndarray, u: np.ndarray) -> np.ndarray:
    """K3's shared-expert activation in float64 (harness/k3/ref.h:97-101; source/k3_moe_front.cu:76-83):
    4 tanh(g/4) * sigmoid(g) * 25 tanh(u/25), g and u as given (land them to bf16 first where the kernel does)."""
    g = np.asarray(g, np.float64)
    u = np.asarray(u, np.float64)
    return 4.0 * np.tanh(g / 4.0) / (1.0 + np.exp(-g)) * 25.0 * np.tanh(u / 25.0)


def strided_tables(idx: np.ndarray, first: int, stride: int, local: int, tile: int = 16):
    """Routing tables of a rank holding experts first + j * stride (j < local): the decode front's
    (source/k3_moe_front.cu:119-176), an expert's rows in token order.  Picks of other ranks' experts get
    exp2perm -1."""
    idx = np.asarray(idx, np.int64)
    d = idx - first
    mine = (d >= 0) & (d % stride == 0) & (d // stride < local)
    loc = np.where(mine, d // stride, -1).astype(np.int32)
    return tables(loc, local, 0, 0, tile)
