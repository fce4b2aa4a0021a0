"""CPU tests of the C ABI boundary (no GPU work is launched): the library
loads, exports every entry point include/k3moe.h declares, and rejects bad
arguments before touching the device."""
import ctypes
import os
import re
import subprocess

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "k3moe.h")


@pytest.fixture(scope="module")
def lib():
    import __graft_entry__

    __graft_entry__.build()
    import k3moe

    return k3moe.lib()


def declared():
    src = open(HEADER).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return sorted(set(re.findall(r"\b(k3moe_\w+)\s*\(", src)))


def test_header_declares_entries():
    names = declared()
    assert "k3moe_layer_forward" in names and "k3moe_fc1" in names and len(names) >= 15


def test_library_exports_every_declared_symbol(lib):
    import k3moe

    nm = subprocess.run(["nm", "-D", "--defined-only", k3moe.LIB_PATH], capture_output=True, text=True).stdout
    exported = set(re.findall(r" T (k3moe_\w+)", nm))
    missing = [n for n in declared() if n not in exported]
    assert not missing, f"declared but not exported: {missing}"
    # every declared entry is also bound (with its signature) by the Python mirror
    assert sorted(k3moe.SIGNATURES) == declared()


def test_pure_host_entries(lib):
    assert lib.k3moe_abi_version() == 1
    assert lib.k3moe_max_ctas(8192, 8, 896, 1, 128) == 897 + (8192 * 9 + 127) // 128
    ws = lib.k3moe_layer_workspace_size(8192, 7168, 2048, 896, 8, 1)
    assert ws > 3 * 10 ** 9
    off = (ctypes.c_size_t * 14)()
    assert lib.k3moe_layer_workspace_offsets(8192, 7168, 2048, 896, 8, 1, ctypes.cast(off, ctypes.c_void_p)) == 0
    assert list(off) == sorted(off) and off[-1] < ws


def test_bad_arguments_rejected_without_device_work(lib):
    # K not a power of two / too many experts / bad widths: rejected before any launch
    assert lib.k3moe_route_topk(None, 896, None, None, 8, 896, 3, None, None, None) == -1
    assert lib.k3moe_route_topk(None, 2048, None, None, 8, 2048, 8, None, None, None) == -1
    assert lib.k3moe_quant_mxfp8(None, 100, 4, 100, None, None, 0, None) == -1
    assert lib.k3moe_layer_forward(None, None, 0, None) == -1


def test_ep_and_gemm_argument_checks(lib):
    # the pair-row stride: E4M3 row, scales, K int16 ids, 16-byte rows
    assert lib.k3moe_ep_pair_row_stride(7168, 8) == 7408
    assert lib.k3moe_ep_pair_row_stride(7168, 16) == 7424
    assert lib.k3moe_ep_pair_row_stride(7168, 17) == 0 and lib.k3moe_ep_pair_row_stride(100, 8) == 0
    # more ranks than a warp's lanes, K out of range, a stride too small for the ids: rejected before any launch
    assert lib.k3moe_ep_pairs(None, 4, 8, 33, None, None) == -1
    assert lib.k3moe_ep_pairs(None, 4, 17, 8, None, None) == -1
    assert lib.k3moe_ep_pack_pairs(None, 7168, 4, 7168, 8, None, None, None, 1, 0, None, 7392, None) == -1
    assert lib.k3moe_ep_ids_k(None, 7392, 4, 7168, 8, None, None) == -1
    assert lib.k3moe_ep_unpack_k(None, 7408, 4, 7168, 0, None, None, None, None) == -1
    assert lib.k3moe_ep_return_rows(None, 4, 8, None, None) == -1
    # FC2 column slices: not on 256-column blocks, past H, a row stride shorter than the slice
    args = [None] * 9
    assert lib.k3moe_fc2_cols(*args, 1024, 128, 256, 7168, 2048, 8, 1024, 8, 0, None, None) == -1
    assert lib.k3moe_fc2_cols(*args, 1024, 7168, 256, 7168, 2048, 8, 1024, 8, 0, None, None) == -1
    assert lib.k3moe_fc2_cols(*args, 128, 0, 256, 7168, 2048, 8, 1024, 8, 0, None, None) == -1
    # the GEMM outputs must start 32-byte aligned (the epilogues store 32 bytes at a time)
    assert lib.k3moe_fc2(None, None, None, None, None, None, None, 16, 7168, 2048, 8, 1024, 8, None, None) == -1
    assert lib.k3moe_combine_ep_chunked(None, 0, 100, None, None, None, 0, 0, None, 7168, 4, 8, 7168, 1000,
                                        None) == -1


def test_noalloc_limits_match_the_header():
    """The Python mirror's limits of the allocation-free entry are the header's, and the fixed array (513 KB,
    2 x 256-byte-rounded [R/256][E + shared] int tables) is exactly the scratch of the largest call."""
    import os
    import re

    import k3moe

    hdr = open(os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "include", "k3moe.h")).read()
    rows = int(re.search(r"#define K3MOE_NOALLOC_MAX_ROWS (\d+)", hdr).group(1))
    experts = int(re.search(r"#define K3MOE_NOALLOC_MAX_EXPERTS (\d+)", hdr).group(1))
    assert (rows, experts) == (k3moe.NOALLOC_MAX_ROWS, k3moe.NOALLOC_MAX_EXPERTS)
    assert k3moe.lib().k3moe_route_scratch_bytes(rows, experts - 1, 1) == 2 * -(-(rows // 256) * experts * 4 // 256) * 256
    assert k3moe.lib().k3moe_route_scratch_bytes(rows, experts - 1, 1) == 524800


def _ep_cfg(**kw):
    import k3moe

    c = dict(world=8, rank=3, H=7168, I=2048, E=896, K=8, shared=1, max_tokens=8192, activation=0,
             wait_budget_ns=0)
    c.update(kw)
    return k3moe.k3moe_ep_config(**c)


def test_ep_step_buffer_sizes(lib):
    """The device-resident step's peer buffer: (W + 1) regions of max_tokens rows (E4M3 | UE8M0 | int16 ids |
    int32 return index, 16-byte rows), the return buffer of max_tokens * K bf16 rows, 256 bytes of counts and
    of flags, each part 256-byte aligned."""
    c = _ep_cfg()
    stride = -(-(7168 + 7168 // 32 + 2 * 8 + 4) // 16) * 16
    assert stride == 7424
    recv = 9 * 8192 * stride
    back_off = -(-recv // 256) * 256
    counts_off = back_off + -(-(8192 * 8 * 7168 * 2) // 256) * 256
    assert lib.k3moe_ep_peer_bytes(ctypes.byref(c)) == counts_off + 512
    # K = 1: the return index after one int16 id is moved to the next 4-byte boundary (7392 + 2 -> 7396)
    c1 = _ep_cfg(K=1, world=2, rank=0, E=16, max_tokens=64)
    recv1 = 3 * 64 * -(-(7396 + 4) // 16) * 16
    assert lib.k3moe_ep_peer_bytes(ctypes.byref(c1)) == -(-recv1 // 256) * 256 + 64 * 7168 * 2 + 512
    ws = lib.k3moe_ep_workspace_bytes(ctypes.byref(c))
    # the GEMM operands dominate: every pick a rank can receive (8 sources x 8192 tokens x 8 picks + the shared
    # rows), padded to 128 an expert, in MXFP8 (H + H/32) and FC1's output (I + I/32)
    cap = (112 + 1 + -(-(8 * 8192 * 8 + 8192) // 128)) * 128
    assert ws > cap * (7168 + 224 + 2048 + 64)
    assert ws < cap * (7168 + 224 + 2048 + 64 + 8) + 2 ** 28


def test_ep_step_rejects_bad_configurations_without_device_work(lib):
    bad = [dict(world=0), dict(world=17), dict(rank=8), dict(E=900), dict(K=3), dict(K=32), dict(H=1000),
           dict(I=100), dict(max_tokens=0), dict(activation=2), dict(E=2048, world=8)]
    for kw in bad:
        c = _ep_cfg(**kw)
        assert lib.k3moe_ep_peer_bytes(ctypes.byref(c)) == 0, kw
        assert lib.k3moe_ep_workspace_bytes(ctypes.byref(c)) == 0, kw
        out = ctypes.c_void_p()
        assert lib.k3moe_ep_create(ctypes.byref(c), None, None, None, None, None, None, None, None, 0, None,
                                   ctypes.byref(out)) == -1, kw
    assert lib.k3moe_ep_peer_bytes(None) == 0
    # a valid configuration with missing buffers is refused before any device call
    out = ctypes.c_void_p()
    assert lib.k3moe_ep_create(ctypes.byref(_ep_cfg()), None, None, None, None, None, None, None, None, 0, None,
                               ctypes.byref(out)) == -1
    assert lib.k3moe_ep_forward(None, None, 896, None, None, None, 7168, 8, None, 7168, None) == -1
    assert lib.k3moe_ep_errors(None) is None
