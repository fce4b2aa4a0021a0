"""Python host mirror of the k3moe C ABI (include/k3moe.h).

The reference drives its MoE through manifest ops (scripts/k3_moe_bmm.py:55-173:
`moe_route`, `moe_fc1`, `moe_fc2`, `moe_finalize`); this module exposes the same
steps as functions over torch CUDA tensors, each a thin call into
``libk3moe.so`` (the sm_100a kernels).  Torch is used only for device memory and
streams.  There is no fallback: if the library is missing or a call fails, an
exception is raised.
"""
from __future__ import annotations

import ctypes
import os
from dataclasses import dataclass

import torch

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libk3moe.so")

_ERRORS = {
    -1: "invalid argument",
    -2: "workspace too small",
    -3: "CUDA driver tensor-map entry unavailable",
    -4: "tensor map could not be encoded (alignment / size)",
    -5: "kernel launch failed",
    -6: "device reported an error",
    -7: "size beyond the fixed scratch of the allocation-free entry",
}

# (name, restype, argtypes) of every exported entry point; tests check the
# library exports exactly what include/k3moe.h declares.
_P, _I, _L, _U64, _F, _SZ = ctypes.c_void_p, ctypes.c_int, ctypes.c_longlong, ctypes.c_uint64, ctypes.c_float, ctypes.c_size_t
SIGNATURES = {
    "k3moe_abi_version": (_I, []),
    "k3moe_route_topk": (_I, [_P, _I, _P, _P, _I, _I, _I, _P, _P, _P]),
    "k3moe_route_scratch_bytes": (_SZ, [_I, _I, _I]),
    "k3moe_route_tables": (_I, [_P, _I, _I, _I, _I, _I, _I, _P, _P, _P, _P, _P, _P, _P, _P]),
    "k3moe_max_ctas": (_I, [_I, _I, _I, _I, _I]),
    "k3moe_quant_mxfp8": (_I, [_P, _I, _I, _I, _P, _P, _I, _P]),
    "k3moe_quant_permute": (_I, [_P, _I, _I, _I, _I, _P, _P, _P, _P, _P]),
    "k3moe_fc1": (_I, [_P, _P, _P, _P, _P, _P, _P, _P, _P, _I, _I, _I, _I, _I, _P, _P]),
    "k3moe_fc2": (_I, [_P, _P, _P, _P, _P, _P, _P, _P, _I, _I, _I, _I, _I, _P, _P]),
    "k3moe_combine": (_I, [_P, _P, _P, _P, _P, _I, _I, _I, _I, _I, _P]),
    "k3moe_quant_mxfp4": (_I, [_P, _L, _I, _P, _P, _P]),
    "k3moe_synth_mxfp4": (_I, [_U64, _L, _L, _I, _F, _P, _P, _P]),
    "k3moe_layer_workspace_size": (_SZ, [_I, _I, _I, _I, _I, _I]),
    "k3moe_layer_forward": (_I, [_P, _P, _SZ, _P]),
    "k3moe_layer_forward_events": (_I, [_P, _P, _SZ, _P, _P, _I]),
    "k3moe_layer_workspace_offsets": (_I, [_I, _I, _I, _I, _I, _I, _P]),
    "k3moe_read_error": (_I, [_P, _P, _I, _P]),
    "k3moe_set_trace": (_I, [_P]),
    "k3moe_route_tables_noalloc": (_I, [_P, _I, _I, _I, _I, _I, _I, _P, _P, _P, _P, _P, _P, _P]),
    "k3moe_fc2_to_rows": (_I, [_P, _P, _P, _P, _P, _P, _P, _P, _P, _I, _I, _I, _I, _I, _P, _P]),
    "k3moe_fc1_act": (_I, [_P, _P, _P, _P, _P, _P, _P, _P, _P, _I, _I, _I, _I, _I, _P, _I, _P]),
    "k3moe_ep_row_stride": (_I, [_I]),
    "k3moe_ep_pack": (_I, [_P, _I, _I, _I, _I, _P, _P, _I, _I, _P, _I, _P]),
    "k3moe_ep_ids": (_I, [_P, _I, _I, _I, _P, _P]),
    "k3moe_ep_unpack": (_I, [_P, _I, _I, _I, _P, _P, _P, _P]),
    "k3moe_combine_ep": (_I, [_P, _P, _P, _P, _I, _P, _I, _I, _I, _I, _P]),
    "k3moe_ep_pair_row_stride": (_I, [_I, _I]),
    "k3moe_fc2_cols": (_I, [_P, _P, _P, _P, _P, _P, _P, _P, _P, _I, _I, _I, _I, _I, _I, _I, _I, _I, _P, _P]),
    "k3moe_combine_ep_chunked": (_I, [_P, _L, _I, _P, _P, _P, _L, _I, _P, _I, _I, _I, _I, _I, _P]),
    "k3moe_ep_pairs": (_I, [_P, _I, _I, _I, _P, _P]),
    "k3moe_ep_pack_pairs": (_I, [_P, _I, _I, _I, _I, _P, _P, _P, _I, _I, _P, _I, _P]),
    "k3moe_ep_ids_k": (_I, [_P, _I, _I, _I, _I, _P, _P]),
    "k3moe_ep_unpack_k": (_I, [_P, _I, _I, _I, _I, _P, _P, _P, _P]),
    "k3moe_ep_return_rows": (_I, [_P, _I, _I, _P, _P]),
    "k3moe_import_mxfp4": (_I, [_P, _P, _I, _I, _I, _I, _P, _P, _P]),
    "k3moe_gemm_tensor_maps": (_I, [_I, _P, _P, _I, _I, _I, _I, _P, _P]),
    "k3moe_ep_pack_pairs_to": (_I, [_P, _I, _I, _I, _I, _P, _P, _P, _I, _P, _I, _P]),
    "k3moe_ep_row_ptrs": (_I, [_P, _I, _I, _P, _I, _P, _P, ctypes.c_int64, _P, _P, _P, _P]),
    "k3moe_fc2_to_ptrs": (_I, [_P, _P, _P, _P, _P, _P, _P, _P, _I, _I, _I, _I, _I, _P, _P]),
    "k3moe_ep_signal": (_I, [_P, _I, _I, _I, ctypes.c_uint32, _P]),
    "k3moe_ep_wait": (_I, [_P, _I, _I, ctypes.c_uint32, _U64, _P, _P]),
    "k3moe_ipc_export": (_I, [_P, _P, _P]),
    "k3moe_ipc_import": (_I, [_P, _U64, _P]),
    "k3moe_ipc_release": (_I, [_P, _U64]),
    "k3moe_router_gemm": (_I, [_P, _I, _P, _I, _I, _I, _I, _P, _I, _P, _P]),
    "k3moe_ep_peer_bytes": (_SZ, [_P]),
    "k3moe_ep_workspace_bytes": (_SZ, [_P]),
    "k3moe_ep_create": (_I, [_P, _P, _P, _P, _P, _P, _P, _P, _P, _SZ, _P, _P]),
    "k3moe_ep_forward": (_I, [_P, _P, _I, _P, _P, _P, _I, _I, _P, _I, _P]),
    "k3moe_ep_forward_events": (_I, [_P, _P, _I, _P, _P, _P, _I, _I, _P, _I, _P, _P, _I]),
    "k3moe_ep_errors": (_P, [_P]),
    "k3moe_ep_counts": (_P, [_P]),
    "k3moe_ep_expert_rows": (_P, [_P]),
    "k3moe_ep_meta": (_P, [_P]),
    "k3moe_ep_destroy": (None, [_P]),
}

TRACE_FIELDS = ["producer", "producer_wait_stage", "mma", "mma_wait_loaded", "mma_wait_drained", "epilogue",
                "epilogue_wait_acc", "units"]


def set_trace(buf):
    """Enable GEMM role counters into a zeroed uint64 device tensor of 32 entries (None disables)."""
    _check(lib().k3moe_set_trace(_p(buf)), "set_trace")


class K3MoeError(RuntimeError):
    pass


_lib = None


def lib() -> ctypes.CDLL:
    """Load libk3moe.so (raises if it is missing: there is no CPU path)."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise K3MoeError(f"{LIB_PATH} is missing: build it with `python __graft_entry__.py` (build())")
        _lib = ctypes.CDLL(LIB_PATH)
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(_lib, name)
            fn.restype = res
            fn.argtypes = args
    return _lib


def _check(rc: int, what: str) -> None:
    if rc != 0:
        raise K3MoeError(f"{what}: {_ERRORS.get(rc, rc)} ({rc})")


def _p(t) -> int | None:
    return None if t is None else t.data_ptr()


def _stream(stream=None) -> int:
    s = stream if stream is not None else torch.cuda.current_stream()
    return s.cuda_stream


class k3moe_layer_args(ctypes.Structure):
    _fields_ = [
        ("T", ctypes.c_int), ("H", ctypes.c_int), ("I", ctypes.c_int), ("E", ctypes.c_int), ("K", ctypes.c_int),
        ("shared", ctypes.c_int),
        ("S", ctypes.c_void_p), ("lds", ctypes.c_int),
        ("bias", ctypes.c_void_p), ("rs", ctypes.c_void_p),
        ("x", ctypes.c_void_p), ("ldx", ctypes.c_int),
        ("w13", ctypes.c_void_p), ("w13_sf", ctypes.c_void_p),
        ("w2", ctypes.c_void_p), ("w2_sf", ctypes.c_void_p),
        ("out", ctypes.c_void_p), ("ldo", ctypes.c_int),
        ("activation", ctypes.c_int),
    ]


ACT_SWIGLU, ACT_SITU = 0, 1


class k3moe_ep_config(ctypes.Structure):
    """include/k3moe.h k3moe_ep_config: one rank's part of the device-resident expert-parallel layer."""
    _fields_ = [
        ("world", ctypes.c_int), ("rank", ctypes.c_int), ("H", ctypes.c_int), ("I", ctypes.c_int),
        ("E", ctypes.c_int), ("K", ctypes.c_int), ("shared", ctypes.c_int), ("max_tokens", ctypes.c_int),
        ("activation", ctypes.c_int), ("wait_budget_ns", ctypes.c_uint64),
    ]


# ------------------------------------------------------------------ steps
def route_topk(S: torch.Tensor, bias: torch.Tensor, rs: torch.Tensor, K: int, E: int | None = None, stream=None):
    """Router top-k (kern_k3g_router_topk semantics): returns (idx int32 [T,K], wts f32 [T,K])."""
    T = S.shape[0]
    E = E or S.shape[1]
    idx = torch.empty((T, K), dtype=torch.int32, device=S.device)
    wts = torch.empty((T, K), dtype=torch.float32, device=S.device)
    _check(lib().k3moe_route_topk(_p(S), S.stride(0), _p(bias), _p(rs), T, E, K, _p(idx), _p(wts), _stream(stream)),
           "route_topk")
    return idx, wts


def router_gemm(x: torch.Tensor, w: torch.Tensor, err: torch.Tensor | None = None, stream=None) -> torch.Tensor:
    """S = x . w^T in f32 (x bf16 [T, H], w bf16 [E, H]): the router logits (k3moe_router_gemm)."""
    T, H = x.shape
    E = w.shape[0]
    S = torch.empty((T, E), dtype=torch.float32, device=x.device)
    _check(lib().k3moe_router_gemm(_p(x), x.stride(0), _p(w), w.stride(0), T, E, H, _p(S), S.stride(0), _p(err),
                                   _stream(stream)), "router_gemm")
    return S


@dataclass
class Tables:
    counts: torch.Tensor
    cta_batch: torch.Tensor
    cta_limit: torch.Tensor
    meta: torch.Tensor          # [num_non_exiting, total_padded, shared_base, 0]
    route_map: torch.Tensor
    exp2perm: torch.Tensor
    max_ctas: int
    cap_rows: int


def route_tables(idx: torch.Tensor, E: int, first: int = 0, shared: int = 0, tile: int = 128, stream=None) -> Tables:
    R, K = idx.shape
    L = lib()
    max_ctas = L.k3moe_max_ctas(R, K, E, shared, tile)
    cap = max_ctas * tile
    dev = idx.device
    scratch = torch.empty(L.k3moe_route_scratch_bytes(R, E, shared), dtype=torch.uint8, device=dev)
    t = Tables(
        counts=torch.empty(E + shared, dtype=torch.int32, device=dev),
        cta_batch=torch.empty(max_ctas, dtype=torch.int32, device=dev),
        cta_limit=torch.empty(max_ctas, dtype=torch.int32, device=dev),
        meta=torch.zeros(4, dtype=torch.int32, device=dev),
        route_map=torch.empty(cap, dtype=torch.int32, device=dev),
        exp2perm=torch.empty((R, K), dtype=torch.int32, device=dev),
        max_ctas=max_ctas, cap_rows=cap)
    _check(L.k3moe_route_tables(_p(idx), R, K, first, E, shared, tile, _p(scratch), _p(t.counts), _p(t.cta_batch),
                                _p(t.cta_limit), _p(t.meta), _p(t.route_map), _p(t.exp2perm), _stream(stream)),
           "route_tables")
    return t


NOALLOC_MAX_ROWS, NOALLOC_MAX_EXPERTS = 16384, 1025  # include/k3moe.h


def route_tables_noalloc(idx: torch.Tensor, E: int, first: int = 0, shared: int = 0, tile: int = 128,
                         stream=None, out: Tables | None = None) -> Tables:
    """route_tables() through k3moe_route_tables_noalloc: the library allocates nothing (its scratch is a fixed
    array in the library; see include/k3moe.h).  `out` may hold preallocated output tables."""
    R, K = idx.shape
    L = lib()
    max_ctas = L.k3moe_max_ctas(R, K, E, shared, tile)
    cap = max_ctas * tile
    dev = idx.device
    t = out or Tables(
        counts=torch.empty(E + shared, dtype=torch.int32, device=dev),
        cta_batch=torch.empty(max_ctas, dtype=torch.int32, device=dev),
        cta_limit=torch.empty(max_ctas, dtype=torch.int32, device=dev),
        meta=torch.zeros(4, dtype=torch.int32, device=dev),
        route_map=torch.empty(cap, dtype=torch.int32, device=dev),
        exp2perm=torch.empty((R, K), dtype=torch.int32, device=dev),
        max_ctas=max_ctas, cap_rows=cap)
    _check(L.k3moe_route_tables_noalloc(_p(idx), R, K, first, E, shared, tile, _p(t.counts), _p(t.cta_batch),
                                        _p(t.cta_limit), _p(t.meta), _p(t.route_map), _p(t.exp2perm),
                                        _stream(stream)), "route_tables_noalloc")
    return t


def quant_mxfp8(x: torch.Tensor, tiled_sf: bool = False, stream=None):
    rows, cols = x.shape
    q = torch.empty((rows, cols), dtype=torch.uint8, device=x.device)
    if tiled_sf:
        sf = torch.zeros((-(-rows // 128)) * (-(-cols // 128)) * 512, dtype=torch.uint8, device=x.device)
    else:
        sf = torch.empty((rows, cols // 32), dtype=torch.uint8, device=x.device)
    _check(lib().k3moe_quant_mxfp8(_p(x), x.stride(0), rows, cols, _p(q), _p(sf), int(tiled_sf), _stream(stream)),
           "quant_mxfp8")
    return q, sf


def quant_permute(x: torch.Tensor, tables: Tables, stream=None):
    R, H = x.shape
    K = tables.exp2perm.shape[1]
    qp = torch.empty((tables.cap_rows, H), dtype=torch.uint8, device=x.device)
    sfp = torch.zeros(tables.cap_rows * H // 32, dtype=torch.uint8, device=x.device)
    _check(lib().k3moe_quant_permute(_p(x), x.stride(0), R, H, K, _p(tables.exp2perm), _p(tables.meta), _p(qp),
                                     _p(sfp), _stream(stream)), "quant_permute")
    return qp, sfp


def fc1(w13, w13_sf, qp, sfp, tables: Tables, H: int, I: int, n_experts: int, err: torch.Tensor, stream=None,
        activation: int = ACT_SWIGLU):
    cap = tables.cap_rows
    out_q = torch.zeros((cap, I), dtype=torch.uint8, device=qp.device)
    out_sf = torch.zeros(cap * I // 32, dtype=torch.uint8, device=qp.device)
    _check(lib().k3moe_fc1_act(_p(w13), _p(w13_sf), _p(qp), _p(sfp), _p(tables.cta_batch), _p(tables.cta_limit),
                               _p(tables.meta), _p(out_q), _p(out_sf), H, I, n_experts, cap, tables.max_ctas, _p(err),
                               activation, _stream(stream)), "fc1")
    return out_q, out_sf


def fc2(w2, w2_sf, fc1_q, fc1_sf, tables: Tables, H: int, I: int, n_experts: int, err: torch.Tensor, stream=None):
    cap = tables.cap_rows
    out = torch.zeros((cap, H), dtype=torch.bfloat16, device=fc1_q.device)
    _check(lib().k3moe_fc2(_p(w2), _p(w2_sf), _p(fc1_q), _p(fc1_sf), _p(tables.cta_batch), _p(tables.cta_limit),
                           _p(tables.meta), _p(out), H, I, n_experts, cap, tables.max_ctas, _p(err), _stream(stream)),
           "fc2")
    return out


def combine(fc2_out, tables: Tables, wts, T: int, out_rows: int | None = None, stream=None):
    out_rows = out_rows or T
    H = fc2_out.shape[1]
    K = tables.exp2perm.shape[1]
    out = torch.empty((out_rows, H), dtype=torch.bfloat16, device=fc2_out.device)
    _check(lib().k3moe_combine(_p(fc2_out), _p(tables.exp2perm), _p(wts), _p(tables.meta), _p(out), H, T, out_rows,
                               K, H, _stream(stream)), "combine")
    return out


def quant_mxfp4(w: torch.Tensor, stream=None):
    """fp32 [rows, K] -> (packed uint8 [rows, K/2], tiled scales)."""
    rows, K = w.shape
    packed = torch.empty((rows, K // 2), dtype=torch.uint8, device=w.device)
    sf = torch.zeros((-(-rows // 128)) * (K // 128) * 512, dtype=torch.uint8, device=w.device)
    _check(lib().k3moe_quant_mxfp4(_p(w), rows, K, _p(packed), _p(sf), _stream(stream)), "quant_mxfp4")
    return packed, sf


def import_mxfp4(packed_rows: torch.Tensor, scale_rows: torch.Tensor, experts: int, gated: bool, stream=None):
    """A checkpoint's MXFP4 expert tensors (row-major `weight_packed` [experts*n, K/2] and `weight_scale`
    [experts*n, K/32], FC1 as [w3 (up); w1 (gate)] with gated=True) -> (packed tile-major, scales tiled), the
    layout the grouped GEMMs read (k3moe_import_mxfp4)."""
    rows, half = packed_rows.shape
    K = half * 2
    n = rows // experts
    packed = torch.empty((rows, half), dtype=torch.uint8, device=packed_rows.device)
    sf = torch.empty(rows * K // 32, dtype=torch.uint8, device=packed_rows.device)
    _check(lib().k3moe_import_mxfp4(_p(packed_rows), _p(scale_rows), experts, n, K, int(gated), _p(packed), _p(sf),
                                    _stream(stream)), "import_mxfp4")
    return packed, sf


def synth_mxfp4(seed: int, rows: int, K: int, sd: float, device="cuda", row0: int = 0, packed=None, sf=None,
                stream=None):
    """Synthetic MXFP4 weights of stream `seed`, rows [row0, row0 + rows)."""
    if packed is None:
        packed = torch.empty((rows, K // 2), dtype=torch.uint8, device=device)
    if sf is None:
        sf = torch.zeros((-(-rows // 128)) * (K // 128) * 512, dtype=torch.uint8, device=device)
    _check(lib().k3moe_synth_mxfp4(seed, row0, rows, K, sd, _p(packed), _p(sf), _stream(stream)), "synth_mxfp4")
    return packed, sf


def read_error(err: torch.Tensor, clear: bool = True, stream=None):
    out = (ctypes.c_uint32 * 2)()
    rc = lib().k3moe_read_error(_p(err), ctypes.cast(out, ctypes.c_void_p), int(clear), _stream(stream))
    return rc, (out[0], out[1])


# ------------------------------------------------------------------ the layer
OFFSET_NAMES = ["idx", "wts", "counts", "cta_batch", "cta_limit", "meta", "route_map", "exp2perm", "q_perm",
                "sf_perm", "fc1_q", "fc1_sf", "fc2", "err"]


class MoELayer:
    """One routed-MoE layer over resident MXFP4 weights (all experts on this GPU).

    Weights: w13 [E+shared, 2I, H/2] packed E2M1 ([gate; up] rows), w2 [E+shared, H, I/2],
    scales tiled over the flattened rows.  forward() runs top-k -> tables -> MXFP8 permute ->
    FC1 (SwiGLU or K3's SiTU, MXFP8) -> FC2 -> combine through k3moe_layer_forward.
    """

    def __init__(self, H, I, E, K, shared, w13, w13_sf, w2, w2_sf, bias, rs, max_tokens, device="cuda",
                 activation=ACT_SWIGLU):
        self.H, self.I, self.E, self.K, self.shared = H, I, E, K, int(shared)
        self.activation = activation
        self.w13, self.w13_sf, self.w2, self.w2_sf = w13, w13_sf, w2, w2_sf
        self.bias, self.rs = bias, rs
        self.max_tokens = max_tokens
        self.ws_bytes = lib().k3moe_layer_workspace_size(max_tokens, H, I, E, K, self.shared)
        if self.ws_bytes == 0:
            raise K3MoeError("bad layer dimensions")
        self.ws = torch.empty(self.ws_bytes, dtype=torch.uint8, device=device)

    def args(self, S, x, out, T=None):
        T = T or x.shape[0]
        a = k3moe_layer_args()
        a.T, a.H, a.I, a.E, a.K, a.shared = T, self.H, self.I, self.E, self.K, self.shared
        a.S, a.lds = S.data_ptr(), S.stride(0)
        a.bias, a.rs = self.bias.data_ptr(), self.rs.data_ptr()
        a.x, a.ldx = x.data_ptr(), x.stride(0)
        a.w13, a.w13_sf, a.w2, a.w2_sf = (self.w13.data_ptr(), self.w13_sf.data_ptr(), self.w2.data_ptr(),
                                          self.w2_sf.data_ptr())
        a.out, a.ldo = out.data_ptr(), out.stride(0)
        a.activation = self.activation
        return a

    def forward(self, S, x, out=None, stream=None):
        T = x.shape[0]
        if T > self.max_tokens:
            raise K3MoeError(f"{T} rows > max_tokens {self.max_tokens}")
        if out is None:
            out = torch.empty((T, self.H), dtype=torch.bfloat16, device=x.device)
        a = self.args(S, x, out, T)
        _check(lib().k3moe_layer_forward(ctypes.byref(a), self.ws.data_ptr(), self.ws_bytes, _stream(stream)),
               "layer_forward")
        return out

    STAGES = ["topk", "tables", "permute", "fc1", "fc2", "combine"]

    def forward_events(self, S, x, out, events, stream=None):
        """forward() recording torch.cuda.Event objects before each stage and after the last (7 events)."""
        T = x.shape[0]
        a = self.args(S, x, out, T)
        arr = (ctypes.c_void_p * len(events))(*[e.cuda_event for e in events])
        _check(lib().k3moe_layer_forward_events(ctypes.byref(a), self.ws.data_ptr(), self.ws_bytes, _stream(stream),
                                                ctypes.cast(arr, ctypes.c_void_p), len(events)), "layer_forward")
        return out

    def offsets(self, T=None):
        T = T or self.max_tokens
        arr = (ctypes.c_size_t * 14)()
        _check(lib().k3moe_layer_workspace_offsets(T, self.H, self.I, self.E, self.K, self.shared,
                                                   ctypes.cast(arr, ctypes.c_void_p)), "offsets")
        return dict(zip(OFFSET_NAMES, list(arr)))

    def check_device_error(self, T=None, stream=None):
        off = self.offsets(T)["err"]
        rc, words = read_error(self.ws[off:off + 8], clear=True, stream=stream)
        if rc != 0:
            raise K3MoeError(f"device error words {words[0]:#x} {words[1]:#x}")
