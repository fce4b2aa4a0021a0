"""The grouped GEMMs and the weight re-layout as module entries of k3moe_module.cubin (kern_k3_moe_fc1,
kern_k3_moe_fc2, kern_k3_moe_w_tiles, kern_k3_moe_sf_tiles), bound by name through the driver API with the
reference ops' parameter lists (scripts/k3_moe_bmm.py:131-134, 167-169; the shuffles' lists,
source/k3_moe_prefill.cu:242-259), against the C-ABI entries on the same inputs: byte equality."""
import ctypes
import os

import numpy as np
import pytest
import torch

import k3moe
import refkern as rk

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
MOD = os.path.join(ROOT, "kern-k3-pp-prefill_b200", "k3moe_module.cubin")
GEMM_THREADS, GEMM_SMEM = 384, 204032  # K3MOE_GEMM_THREADS / K3MOE_GEMM_SMEM_BYTES (include/k3moe.h)


def _F(v):
    return ctypes.c_float(v)


def _setup(dev, T, H, I, E, K, shared, seed):
    g = torch.Generator(device=dev)
    g.manual_seed(seed)
    S = torch.randn((T, E), generator=g, device=dev)
    bias = torch.rand(E, generator=g, device=dev) * 0.2 - 0.1
    rs = torch.tensor([1.0], dtype=torch.bfloat16, device=dev)
    x = torch.randn((T, H), generator=g, device=dev).to(torch.bfloat16)
    ne = E + shared
    w13, w13_sf = k3moe.synth_mxfp4(seed + 1, ne * 2 * I, H, 0.02, device=dev)
    w2, w2_sf = k3moe.synth_mxfp4(seed + 2, ne * H, I, 0.02, device=dev)
    idx, _ = k3moe.route_topk(S, bias, rs, K)
    tb = k3moe.route_tables(idx, E, 0, shared)
    qp, sfp = k3moe.quant_permute(x, tb)
    return dict(w13=w13, w13_sf=w13_sf, w2=w2, w2_sf=w2_sf, tb=tb, qp=qp, sfp=sfp, ne=ne)


def _maps(mode, w, act, ne, H, I, cap, dev):
    maps = torch.zeros(256, dtype=torch.uint8, device=dev)  # K3MOE_GEMM_MAPS_BYTES
    rc = k3moe.lib().k3moe_gemm_tensor_maps(mode, w.data_ptr(), act.data_ptr(), ne, H, I, cap, maps.data_ptr(),
                                            k3moe._stream())
    assert rc == 0, f"k3moe_gemm_tensor_maps = {rc}"
    return maps


@pytest.mark.parametrize("cfg", [dict(T=333, H=1024, I=512, E=32, K=8, shared=1),
                                 dict(T=200, H=7168, I=2048, E=8, K=4, shared=1),
                                 dict(T=64, H=2048, I=256, E=4, K=2, shared=0)])
@pytest.mark.parametrize("act", [0, 1])
def test_module_fc1_fc2_equal_c_abi(dev, cfg, act):
    H, I = cfg["H"], cfg["I"]
    d = _setup(dev, **cfg, seed=31 + act)
    tb, ne = d["tb"], d["ne"]
    cap = tb.cap_rows
    err = torch.zeros(4, dtype=torch.int32, device=dev)
    # the C ABI
    f1q, f1sf = k3moe.fc1(d["w13"], d["w13_sf"], d["qp"], d["sfp"], tb, H, I, ne, err, activation=act)
    y = k3moe.fc2(d["w2"], d["w2_sf"], f1q, f1sf, tb, H, I, ne, err)
    # the module entries, through the driver API
    sms = torch.cuda.get_device_properties(dev).multi_processor_count
    m1 = _maps(0, d["w13"], d["qp"], ne, H, I, cap, dev)
    alpha = torch.full((ne,), 4.0, device=dev)
    beta = torch.full((ne,), 25.0, device=dev)
    out_q = torch.zeros((cap, I), dtype=torch.uint8, device=dev)
    out_sf = torch.zeros(cap * I // 32, dtype=torch.uint8, device=dev)
    merr = torch.zeros(4, dtype=torch.int32, device=dev)
    nne, tp = tb.meta[0:1], tb.meta[1:2]
    f = rk.function(MOD, "kern_k3_moe_fc1")
    rk.allow_smem(f, GEMM_SMEM)
    rk.launch(f, (sms, 1, 1), (GEMM_THREADS, 1, 1),
              [rk.P(d["w13"]), rk.P(d["w13_sf"]), rk.P(d["qp"]), rk.P(d["sfp"]), rk.P(out_q), rk.P(out_sf),
               rk.P(tb.route_map), rk.P(alpha), rk.P(beta), rk.P(nne), rk.P(tp), rk.P(tb.cta_batch),
               rk.P(tb.cta_limit), rk.I(2 * I), rk.I(H), rk.I(ne), rk.I(cap), rk.I(tb.max_ctas), rk.I(act),
               rk.P(m1), rk.P(merr)], smem=GEMM_SMEM)
    m2 = _maps(1, d["w2"], out_q, ne, H, I, cap, dev)
    out = torch.zeros((cap, H), dtype=torch.bfloat16, device=dev)
    f = rk.function(MOD, "kern_k3_moe_fc2")
    rk.allow_smem(f, GEMM_SMEM)
    rk.launch(f, (sms, 1, 1), (GEMM_THREADS, 1, 1),
              [rk.P(d["w2"]), rk.P(d["w2_sf"]), rk.P(out_q), rk.P(out_sf), rk.P(out), rk.P(nne), rk.P(tp),
               rk.P(tb.cta_batch), rk.P(tb.cta_limit), rk.I(H), rk.I(I), rk.I(ne), rk.I(cap), rk.I(tb.max_ctas),
               rk.P(m2), rk.P(merr)], smem=GEMM_SMEM)
    torch.cuda.synchronize()
    assert err[:2].tolist() == [0, 0] and merr[:2].tolist() == [0, 0]
    assert torch.equal(out_q, f1q), "FC1 E4M3 bytes differ"
    assert torch.equal(out_sf, f1sf), "FC1 scales differ"
    assert torch.equal(out.view(torch.int16), y.view(torch.int16)), "FC2 bf16 output differs"


def test_module_gemm_rejects_bad_arguments(dev):
    """A module launch has no host checks: bad shapes set the error word and write nothing."""
    d = _setup(dev, T=64, H=1024, I=256, E=4, K=2, shared=0, seed=5)
    tb, ne = d["tb"], d["ne"]
    cap = tb.cap_rows
    m1 = _maps(0, d["w13"], d["qp"], ne, 1024, 256, cap, dev)
    out_q = torch.full((cap, 256), 0x5A, dtype=torch.uint8, device=dev)
    out_sf = torch.full((cap * 256 // 32,), 0x5A, dtype=torch.uint8, device=dev)
    merr = torch.zeros(4, dtype=torch.int32, device=dev)
    f = rk.function(MOD, "kern_k3_moe_fc1")
    rk.allow_smem(f, GEMM_SMEM)
    rk.launch(f, (4, 1, 1), (GEMM_THREADS, 1, 1),
              [rk.P(d["w13"]), rk.P(d["w13_sf"]), rk.P(d["qp"]), rk.P(d["sfp"]), rk.P(out_q), rk.P(out_sf),
               rk.P(tb.route_map), rk.P(out_q), rk.P(out_q), rk.P(tb.meta[0:1]), rk.P(tb.meta[1:2]),
               rk.P(tb.cta_batch), rk.P(tb.cta_limit), rk.I(2 * 256 + 128), rk.I(1024), rk.I(ne), rk.I(cap),
               rk.I(tb.max_ctas), rk.I(0), rk.P(m1), rk.P(merr)], smem=GEMM_SMEM)
    torch.cuda.synchronize()
    assert int(merr[0].item()) & 8, "the bad-argument bit is not set"
    assert bool((out_q == 0x5A).all()) and bool((out_sf == 0x5A).all()), "an output was written"


@pytest.mark.parametrize("experts,n,K,gated", [(3, 256, 512, 1), (2, 7168, 2048, 0)])
def test_module_weight_tiles_equal_c_abi(dev, experts, n, K, gated):
    rng = np.random.default_rng(experts * n + K)
    w = torch.from_numpy(rng.integers(0, 256, (experts * n, K // 2), dtype=np.uint8)).to(dev)
    s = torch.from_numpy(rng.integers(0, 256, (experts * n, K // 32), dtype=np.uint8)).to(dev)
    ref_p, ref_s = k3moe.import_mxfp4(w, s, experts, bool(gated))
    out_p = torch.empty_like(ref_p).fill_(0x5A)
    out_s = torch.empty_like(ref_s).fill_(0x5A)
    total = experts * n * K // 32
    rk.launch(rk.function(MOD, "kern_k3_moe_w_tiles"), ((total + 255) // 256, 1, 1), (256, 1, 1),
              [rk.P(w), rk.P(out_p), rk.I(experts), rk.I(n), rk.I(K // 2), rk.I(gated)])
    total = experts * n * K // 128
    rk.launch(rk.function(MOD, "kern_k3_moe_sf_tiles"), ((total + 255) // 256, 1, 1), (256, 1, 1),
              [rk.P(s), rk.P(out_s), rk.I(experts), rk.I(n), rk.I(K // 32), rk.I(gated)])
    torch.cuda.synchronize()
    assert torch.equal(out_p, ref_p) and torch.equal(out_s, ref_s)


@pytest.mark.parametrize("T,H,E,K,shared", [(333, 1024, 32, 8, 1), (64, 7168, 896, 8, 0)])
def test_module_quant_permute_equal_c_abi(dev, T, H, E, K, shared):
    g = torch.Generator(device=dev)
    g.manual_seed(T + H)
    S = torch.randn((T, E), generator=g, device=dev)
    bias = torch.zeros(E, device=dev)
    rs = torch.tensor([1.0], dtype=torch.bfloat16, device=dev)
    x = torch.randn((T, H), generator=g, device=dev).to(torch.bfloat16)
    idx, _ = k3moe.route_topk(S, bias, rs, K)
    tb = k3moe.route_tables(idx, E, 0, shared)
    qp = torch.zeros((tb.cap_rows, H), dtype=torch.uint8, device=dev)
    sfp = torch.zeros(tb.cap_rows * H // 32, dtype=torch.uint8, device=dev)
    rc = k3moe.lib().k3moe_quant_permute(x.data_ptr(), H, T, H, K, tb.exp2perm.data_ptr(), tb.meta.data_ptr(),
                                         qp.data_ptr(), sfp.data_ptr(), k3moe._stream())
    assert rc == 0
    oq = torch.zeros_like(qp)
    osf = torch.zeros_like(sfp)
    rk.launch(rk.function(MOD, "kern_k3_moe_quant_permute"), (148, 1, 1), (256, 1, 1),
              [rk.P(x), rk.I(H), rk.I(T), rk.I(H), rk.I(K), rk.P(tb.exp2perm), rk.P(tb.meta), rk.P(oq), rk.P(osf)])
    torch.cuda.synchronize()
    assert torch.equal(oq, qp) and torch.equal(osf, sfp)
