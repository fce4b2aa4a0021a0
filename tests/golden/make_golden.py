"""Make tests/golden/router_topk_ref.npz with the reference's own CPU reference.

The reference's router top-k reference (harness/k3/ref.h `ref_router_topk`,
EXPERTS = 896, TOPK = 16, sigmoid in double, 16 sequential max passes, ties to
the smaller expert) is compiled from where it lies in the reference tree into
oracle/_ref/libk3ref.so by oracle/Makefile.  Inputs follow the reference
harness's router case (harness/k3/harness.cu:697-710): S ~ N(0, 2), bias ~
N(0, 0.1), experts 40 and 41 forced to an exact tie inside the top-16 (S = 6,
bias = 0.5), rs = 2.5; they are regenerated from the stored seeds with numpy's
PCG64, so only the outputs are stored.

Run where the reference tree exists:  make -C oracle && python tests/golden/make_golden.py
"""
import ctypes
import os

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
LIB = os.path.join(ROOT, "oracle", "_ref", "libk3ref.so")
SIZES = [1, 2, 8, 64]
E, K = 896, 16


def inputs(B, seed):
    rng = np.random.default_rng(seed)
    S = (rng.standard_normal((B, E)) * 2.0).astype(np.float32)
    bias = (rng.standard_normal(E) * 0.1).astype(np.float32)
    bias[40] = bias[41] = 0.5
    S[:, 40] = S[:, 41] = 6.0
    return S, bias


RS_BITS = 0x4020  # bf16 2.5
SITU_ROWS, SITU_N = 4, 768


def situ_inputs():
    rng = np.random.default_rng(4242)
    p = np.empty((SITU_ROWS, 2 * SITU_N), np.float32)
    p[:, :SITU_N] = rng.uniform(-12, 12, (SITU_ROWS, SITU_N))
    p[:, SITU_N:] = rng.uniform(-60, 60, (SITU_ROWS, SITU_N))
    p[0, :16] = 0.0
    p[1, SITU_N:SITU_N + 16] = 0.0
    return p


def main():
    lib = ctypes.CDLL(LIB)
    assert lib.k3ref_experts() == E and lib.k3ref_topk() == K
    out = {"sizes": np.array(SIZES, np.int32), "rs_bits": np.array([RS_BITS], np.uint16)}
    for B in SIZES:
        S, bias = inputs(B, 1000 + B)
        idx = np.empty((B, K), np.int32)
        wts = np.empty((B, K), np.float32)
        rs = np.array([RS_BITS], np.uint16)
        lib.k3ref_router_topk(S.ctypes.data_as(ctypes.c_void_p), bias.ctypes.data_as(ctypes.c_void_p),
                              rs.ctypes.data_as(ctypes.c_void_p), idx.ctypes.data_as(ctypes.c_void_p),
                              wts.ctypes.data_as(ctypes.c_void_p), ctypes.c_int(B))
        out[f"idx_{B}"] = idx
        out[f"wts_{B}"] = wts
    np.savez_compressed(os.path.join(HERE, "router_topk_ref.npz"), **out)
    print("wrote", os.path.join(HERE, "router_topk_ref.npz"))

    # K3's shared-expert SiTU with its bf16 landings (harness/k3/ref.h:614-622, `ref_land_situ`): gate | up
    # f32 rows of one rank's shared width (768), values spread over the tanh knees (|g| up to 12, |u| up to
    # 60) plus exact zeros; regenerated from the seed, only the outputs stored
    B, n = SITU_ROWS, SITU_N
    p = situ_inputs()
    act = np.empty((B, n), np.uint16)
    lib.k3ref_land_situ(p.ctypes.data_as(ctypes.c_void_p), act.ctypes.data_as(ctypes.c_void_p), ctypes.c_int(n),
                        ctypes.c_int(B))
    np.savez_compressed(os.path.join(HERE, "land_situ_ref.npz"), act=act)
    print("wrote", os.path.join(HERE, "land_situ_ref.npz"))


if __name__ == "__main__":
    main()
