"""Bit parity with the reference's own kernels, built from its sources for
sm_100a (oracle/_ref) and run on the same GPU over identical seeded inputs.

Pinned here: router top-k ids and weights (kern_k3g_router_topk,
source/k3_prefill_glue.cu:504-557), MXFP8 bytes and scales in both layouts
(kern_k3_moe_quant, source/k3_moe_prefill.cu:66-95; kern_k3_mxfp8_quant,
source/k3_mxfp8.cu:20-54), the EP-slice routing tables (kern_k3_moe_route_count
/ _tables / _scatter, source/k3_moe_prefill.cu:97-204) and the combine
(kern_k3_moe_finalize, source/k3_moe_prefill.cu:206-234)."""
import numpy as np
import pytest
import torch

import k3moe
import oracle
import refkern as rk

pytestmark = pytest.mark.gpu

REF_TOPK, REF_E = 16, 896


def _t(a, dev):
    return torch.from_numpy(np.ascontiguousarray(a)).to(dev)


def _need(module):
    if not rk.available(module):
        pytest.fail(f"oracle/_ref/{module}.cubin missing (build it with `make -C oracle` where the reference tree is)")


@pytest.mark.parametrize("B", [1, 2, 8, 64, 4096])
def test_router_topk_bit_exact_with_reference(dev, B):
    _need("k3_prefill_glue")
    rng = np.random.default_rng(B)
    S = (rng.standard_normal((B, REF_E)) * 2).astype(np.float32)
    bias = (rng.standard_normal(REF_E) * 0.1).astype(np.float32)
    bias[40] = bias[41] = 0.5
    S[:, 40] = S[:, 41] = 6.0
    rs = _t(oracle.bf16_bits(np.array([2.5], np.float32)), dev).view(torch.bfloat16)
    dS, db = _t(S, dev), _t(bias, dev)
    ridx = torch.full((B, REF_TOPK), -7, dtype=torch.int32, device=dev)
    rw = torch.full((B, REF_TOPK), -7.0, dtype=torch.float32, device=dev)
    f = rk.function("k3_prefill_glue", "kern_k3g_router_topk")
    rk.launch(f, ((B + 3) // 4, 1, 1), (128, 1, 1), [rk.P(dS), rk.P(db), rk.P(rs), rk.P(ridx), rk.P(rw), rk.I(B)])
    idx16, w16 = k3moe.route_topk(dS, db, rs, 16)
    torch.cuda.synchronize()
    assert torch.equal(idx16, ridx)
    assert torch.equal(w16.view(torch.int32), rw.view(torch.int32))
    # top-8: the first 8 of the reference's top-16 (one total order)
    idx8, _ = k3moe.route_topk(dS, db, rs, 8)
    assert torch.equal(idx8, ridx[:, :8])


@pytest.mark.parametrize("rows,cols", [(1, 3584), (64, 3584), (1000, 7168), (8192, 7168)])
def test_quant_linear_bit_exact_with_reference(dev, rows, cols):
    _need("k3_moe_prefill")
    rng = np.random.default_rng(rows + cols)
    x = (rng.standard_normal((rows, cols)) * np.exp(rng.uniform(-6, 6, (rows, 1)))).astype(np.float32)
    xb = _t(oracle.bf16_bits(x), dev).view(torch.bfloat16)
    rq = torch.full((rows, cols), 0x5A, dtype=torch.uint8, device=dev)
    rsf = torch.full((rows, cols // 32), 0x5A, dtype=torch.uint8, device=dev)
    f = rk.function("k3_moe_prefill", "kern_k3_moe_quant")
    grid = (-(-rows * cols // 32 // 256), 1, 1)
    rk.launch(f, grid, (256, 1, 1), [rk.P(xb), rk.P(rq), rk.P(rsf), rk.I(rows), rk.I(cols)])
    q, sf = k3moe.quant_mxfp8(xb, tiled_sf=False)
    torch.cuda.synchronize()
    assert torch.equal(q, rq)
    assert torch.equal(sf, rsf)


@pytest.mark.parametrize("rows,cols", [(130, 3584), (4096, 7168)])
def test_quant_tiled_bit_exact_with_reference(dev, rows, cols):
    _need("k3_mxfp8")
    rng = np.random.default_rng(rows * 3 + cols)
    x = (rng.standard_normal((rows, cols)) * np.exp(rng.uniform(-6, 6, (rows, 1)))).astype(np.float32)
    xb = _t(oracle.bf16_bits(x), dev).view(torch.bfloat16)
    nsf = -(-rows // 128) * -(-cols // 128) * 512
    rq = torch.zeros((rows, cols), dtype=torch.uint8, device=dev)
    rsf = torch.zeros(nsf, dtype=torch.uint8, device=dev)
    f = rk.function("k3_mxfp8", "kern_k3_mxfp8_quant")
    rk.launch(f, (296, 1, 1), (256, 1, 1), [rk.P(xb), rk.I(cols), rk.P(rq), rk.P(rsf), rk.I(rows), rk.I(cols)])
    q, sf = k3moe.quant_mxfp8(xb, tiled_sf=True)
    torch.cuda.synchronize()
    assert torch.equal(q, rq)
    assert torch.equal(sf[:nsf], rsf)  # rows past `rows` in the last atom are zero on both sides


@pytest.mark.parametrize("T,E,rank,tile", [(1, 64, 0, 128), (48, 56, 3, 128), (300, 64, 7, 128), (4096, 56, 1, 64),
                                           (8192, 64, 13, 128)])
def test_route_tables_bit_exact_with_reference(dev, T, E, rank, tile):
    _need("k3_moe_prefill")
    rng = np.random.default_rng(T + 31 * rank)
    total = 896
    idx = np.stack([rng.choice(total, REF_TOPK, replace=False) for _ in range(T)]).astype(np.int32)
    first = rank * E
    # make some tokens pick mostly local experts (as the reference's d1 harness does)
    for t in range(0, T, 4):
        idx[t] = first + rng.choice(E, REF_TOPK, replace=False)
    didx = _t(idx, dev)
    blocks = -(-T // 256)
    ctas_max = E + -(-T * REF_TOPK // tile)
    bc = torch.zeros(blocks * E, dtype=torch.int32, device=dev)
    boff = torch.zeros(blocks * E, dtype=torch.int32, device=dev)
    cb = torch.full((ctas_max,), -7, dtype=torch.int32, device=dev)
    cl = torch.full((ctas_max,), -7, dtype=torch.int32, device=dev)
    nne = torch.full((1,), -7, dtype=torch.int32, device=dev)
    tp = torch.full((1,), -7, dtype=torch.int32, device=dev)
    rmap = torch.full((ctas_max * tile,), -7, dtype=torch.int32, device=dev)
    e2p = torch.full((T, REF_TOPK), -7, dtype=torch.int32, device=dev)
    m = "k3_moe_prefill"
    rk.launch(rk.function(m, "kern_k3_moe_route_count"), (blocks, 1, 1), (256, 1, 1),
              [rk.P(didx), rk.I(T), rk.I(rank), rk.I(E), rk.P(bc)])
    rk.launch(rk.function(m, "kern_k3_moe_route_tables"), (1, 1, 1), (1024, 1, 1),
              [rk.P(bc), rk.I(blocks), rk.I(E), rk.I(tile), rk.P(boff), rk.P(cb), rk.P(cl), rk.P(nne), rk.P(tp),
               rk.P(rmap)])
    rk.launch(rk.function(m, "kern_k3_moe_route_scatter"), (blocks, 1, 1), (256, 1, 1),
              [rk.P(didx), rk.P(boff), rk.I(T), rk.I(rank), rk.I(E), rk.P(rmap), rk.P(e2p)])
    t = k3moe.route_tables(didx, E, first, 0, tile)
    torch.cuda.synchronize()
    n = int(nne.item())
    assert int(t.meta[0]) == n and int(t.meta[1]) == int(tp.item())
    assert torch.equal(t.cta_batch[:n], cb[:n])
    assert torch.equal(t.cta_limit[:n], cl[:n])
    assert torch.equal(t.exp2perm, e2p)
    assert torch.equal(t.route_map[:n * tile], rmap[:n * tile])


@pytest.mark.parametrize("T,out_rows,cols", [(1, 1, 3584), (37, 64, 3584), (512, 512, 7168)])
def test_combine_bit_exact_with_reference(dev, T, out_rows, cols):
    _need("k3_moe_prefill")
    rng = np.random.default_rng(T + cols)
    idx = np.stack([rng.choice(896, REF_TOPK, replace=False) for _ in range(T)]).astype(np.int32)
    t = k3moe.route_tables(_t(idx, dev), 448, 0, 0)  # half the experts local: the rest are -1 picks
    fc2 = _t(oracle.bf16_bits(rng.standard_normal((t.cap_rows, cols)).astype(np.float32)), dev).view(torch.bfloat16)
    wts = _t(rng.uniform(0, 0.3, (T, REF_TOPK)).astype(np.float32), dev)
    ref = torch.full((out_rows, cols), 7, dtype=torch.bfloat16, device=dev)
    f = rk.function("k3_moe_prefill", "kern_k3_moe_finalize")
    rk.launch(f, (out_rows, 1, 1), (cols // 8, 1, 1), [rk.P(fc2), rk.P(t.exp2perm), rk.P(wts), rk.P(ref), rk.I(T),
                                                       rk.I(cols)])
    out = torch.empty((out_rows, cols), dtype=torch.bfloat16, device=dev)
    rc = k3moe.lib().k3moe_combine(fc2.data_ptr(), t.exp2perm.data_ptr(), wts.data_ptr(), None, out.data_ptr(), cols,
                                   T, out_rows, REF_TOPK, cols, torch.cuda.current_stream().cuda_stream)
    assert rc == 0
    torch.cuda.synchronize()
    assert torch.equal(out.view(torch.int16), ref.view(torch.int16))
