"""The allocation-free routing-table entry (k3moe_route_tables_noalloc).

Some callers cannot allocate device memory -- a host runtime that owns every
device buffer and hands each call a fixed list, or a latency-critical loop
that cannot pay for cudaMalloc's possible device-wide synchronisation.  For
them the library keeps the table builder's scratch in a fixed array of its
own.  These tests call that entry through the C ABI and check its tables
against the ordinary entry (which takes caller scratch): the tables are
integers, so they must match exactly, on two calls in a row (the second call
reuses the array the first one left behind).  The file runs last so that a
failure here never hides the rest of the suite."""
import ctypes

import numpy as np
import pytest
import torch

import k3moe

pytestmark = pytest.mark.gpu


def _ids(R, K, E_total, seed):
    rng = np.random.default_rng(seed)
    return np.stack([rng.choice(E_total, K, replace=False) for _ in range(R)]).astype(np.int32)


def _same(a: k3moe.Tables, b: k3moe.Tables):
    n = int(b.meta[0])
    assert torch.equal(a.meta[:3], b.meta[:3])
    assert torch.equal(a.counts, b.counts)
    assert torch.equal(a.cta_batch[:n], b.cta_batch[:n])
    assert torch.equal(a.cta_limit[:n], b.cta_limit[:n])
    assert torch.equal(a.exp2perm, b.exp2perm)
    assert torch.equal(a.route_map[:int(b.meta[1])], b.route_map[:int(b.meta[1])])


def test_noalloc_tables_match_two_calls_in_a_row(dev):
    ids1 = torch.from_numpy(_ids(8192, 8, 896, 1)).to(dev)
    ids2 = torch.from_numpy(_ids(300, 8, 896, 2)).to(dev)
    # call 1: a prefill chunk with every expert local and the shared expert;
    # call 2, right after it: a different size and an expert-parallel slice, over the scratch call 1 left
    got1 = k3moe.route_tables_noalloc(ids1, 896, 0, 1)
    got2 = k3moe.route_tables_noalloc(ids2, 112, 224, 0)
    ref1 = k3moe.route_tables(ids1, 896, 0, 1)
    ref2 = k3moe.route_tables(ids2, 112, 224, 0)
    torch.cuda.synchronize()
    _same(got1, ref1)
    _same(got2, ref2)


def test_noalloc_rejects_sizes_beyond_its_scratch(dev):
    lib = k3moe.lib()
    ids = torch.zeros((k3moe.NOALLOC_MAX_ROWS + 1, 1), dtype=torch.int32, device=dev)
    out = torch.empty(1 << 20, dtype=torch.int32, device=dev)  # never written: the call is refused first
    p = ctypes.c_void_p(out.data_ptr())
    s = torch.cuda.current_stream().cuda_stream
    rc = lib.k3moe_route_tables_noalloc(ids.data_ptr(), ids.shape[0], 1, 0, 16, 0, 128, p, p, p, p, p, p, s)
    assert rc == -7
    rc = lib.k3moe_route_tables_noalloc(ids.data_ptr(), 128, 1, 0, k3moe.NOALLOC_MAX_EXPERTS, 1, 128, p, p, p, p,
                                        p, p, s)
    assert rc == -7


def test_noalloc_at_its_limits(dev):
    """The largest call the fixed array takes (K3MOE_NOALLOC_MAX_ROWS rows, K3MOE_NOALLOC_MAX_EXPERTS local
    experts with the shared expert): its second scratch table ends exactly at the end of the array."""
    R, E = k3moe.NOALLOC_MAX_ROWS, k3moe.NOALLOC_MAX_EXPERTS - 1
    ids = torch.from_numpy(_ids(R, 8, E, 3)).to(dev)
    got = k3moe.route_tables_noalloc(ids, E, 0, 1)
    ref = k3moe.route_tables(ids, E, 0, 1)
    torch.cuda.synchronize()
    _same(got, ref)
