"""The drop-in module (kern-k3-pp-prefill_b200/k3moe_module.cubin): each entry,
bound by name and launched with the reference manifest's geometry, against the
same entry of the reference's module built from source (oracle/_ref), on the
same inputs into output buffers poisoned the same way: byte equality."""
import os

import numpy as np
import pytest
import torch

import oracle
import refkern as rk

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
MOD = os.path.join(ROOT, "kern-k3-pp-prefill_b200", "k3moe_module.cubin")
TOPK, E, LATENT = 16, 896, 3584


def _t(a, dev):
    return torch.from_numpy(np.ascontiguousarray(a)).to(dev)


def _poison(shape, dtype, dev):
    t = torch.empty(shape, dtype=dtype, device=dev)
    t.view(torch.uint8).fill_(0x5A)
    return t


def _both(ref_module, entry, grid, block, make_args):
    """Launch the reference entry and ours on argument sets built by make_args(); return both sets."""
    ra, oa = make_args(), make_args()
    rk.launch(rk.function(ref_module, entry), grid, block, ra[0])
    rk.launch(rk.function(MOD, entry), grid, block, oa[0])
    torch.cuda.synchronize()
    return ra[1], oa[1]


@pytest.mark.parametrize("rows,cols", [(1, 3584), (333, 7168), (8192, 3584)])
def test_moe_quant(dev, rows, cols):
    rng = np.random.default_rng(rows)
    x = _t(oracle.bf16_bits((rng.standard_normal((rows, cols)) * np.exp(rng.uniform(-5, 5, (rows, 1))))
                            .astype(np.float32)), dev).view(torch.bfloat16)

    def mk():
        q, sf = _poison((rows, cols), torch.uint8, dev), _poison((rows, cols // 32), torch.uint8, dev)
        return [rk.P(x), rk.P(q), rk.P(sf), rk.I(rows), rk.I(cols)], (q, sf)

    (rq, rsf), (q, sf) = _both("k3_moe_prefill", "kern_k3_moe_quant", (-(-rows * cols // 32 // 256), 1, 1),
                               (256, 1, 1), mk)
    assert torch.equal(q, rq) and torch.equal(sf, rsf)


@pytest.mark.parametrize("rows,cols", [(130, 3584), (1000, 7168)])
def test_mxfp8_quant(dev, rows, cols):
    rng = np.random.default_rng(cols + rows)
    x = _t(oracle.bf16_bits(rng.standard_normal((rows, cols)).astype(np.float32)), dev).view(torch.bfloat16)
    nsf = -(-rows // 128) * -(-cols // 128) * 512

    def mk():
        q, sf = _poison((rows, cols), torch.uint8, dev), _poison(nsf, torch.uint8, dev)
        return [rk.P(x), rk.I(cols), rk.P(q), rk.P(sf), rk.I(rows), rk.I(cols)], (q, sf)

    (rq, rsf), (q, sf) = _both("k3_mxfp8", "kern_k3_mxfp8_quant", (148, 1, 1), (256, 1, 1), mk)
    assert torch.equal(q, rq) and torch.equal(sf, rsf)


@pytest.mark.parametrize("B", [1, 7, 64, 2048])
def test_router_topk(dev, B):
    rng = np.random.default_rng(B + 3)
    S = _t((rng.standard_normal((B, E)) * 2).astype(np.float32), dev)
    bias = _t((rng.standard_normal(E) * 0.1).astype(np.float32), dev)
    rs = _t(oracle.bf16_bits(np.array([2.5], np.float32)), dev).view(torch.bfloat16)

    def mk():
        idx, w = _poison((B, TOPK), torch.int32, dev), _poison((B, TOPK), torch.float32, dev)
        return [rk.P(S), rk.P(bias), rk.P(rs), rk.P(idx), rk.P(w), rk.I(B)], (idx, w)

    (ri, rw), (i, w) = _both("k3_prefill_glue", "kern_k3g_router_topk", (-(-B // 4), 1, 1), (128, 1, 1), mk)
    assert torch.equal(i, ri) and torch.equal(w.view(torch.int32), rw.view(torch.int32))


@pytest.mark.parametrize("T,El,rank,tile", [(48, 56, 3, 128), (4096, 64, 5, 64), (1, 16, 0, 128)])
def test_route_count_tables_scatter(dev, T, El, rank, tile):
    rng = np.random.default_rng(T + El)
    ids_np = np.stack([rng.choice(E, TOPK, replace=False) for _ in range(T)]).astype(np.int32)
    for t in range(0, T, 3):
        ids_np[t] = rank * El + rng.choice(El, TOPK, replace=False)
    ids = _t(ids_np, dev)
    blocks = -(-T // 256)
    ctas = El + -(-T * TOPK // tile)
    outs = {}
    for name, mod in (("ref", "k3_moe_prefill"), ("ours", MOD)):
        bc = _poison(blocks * El, torch.int32, dev)
        bo = _poison(blocks * El, torch.int32, dev)
        cb, cl = _poison(ctas, torch.int32, dev), _poison(ctas, torch.int32, dev)
        nne, tp = _poison(1, torch.int32, dev), _poison(1, torch.int32, dev)
        rmap, e2p = _poison(ctas * tile, torch.int32, dev), _poison((T, TOPK), torch.int32, dev)
        rk.launch(rk.function(mod, "kern_k3_moe_route_count"), (blocks, 1, 1), (256, 1, 1),
                  [rk.P(ids), rk.I(T), rk.I(rank), rk.I(El), rk.P(bc)])
        rk.launch(rk.function(mod, "kern_k3_moe_route_tables"), (1, 1, 1), (1024, 1, 1),
                  [rk.P(bc), rk.I(blocks), rk.I(El), rk.I(tile), rk.P(bo), rk.P(cb), rk.P(cl), rk.P(nne), rk.P(tp),
                   rk.P(rmap)])
        rk.launch(rk.function(mod, "kern_k3_moe_route_scatter"), (blocks, 1, 1), (256, 1, 1),
                  [rk.P(ids), rk.P(bo), rk.I(T), rk.I(rank), rk.I(El), rk.P(rmap), rk.P(e2p)])
        torch.cuda.synchronize()
        outs[name] = [bc, bo, cb, cl, nne, tp, rmap, e2p]
    for a, b in zip(outs["ref"], outs["ours"]):
        assert torch.equal(a, b)


def _fc2_inputs(T, cols, dev, seed):
    rng = np.random.default_rng(seed)
    idx = np.stack([rng.choice(E, TOPK, replace=False) for _ in range(T)]).astype(np.int32)
    e2p = np.where(idx % 3 == 0, -1, np.arange(T * TOPK).reshape(T, TOPK)).astype(np.int32)  # some foreign picks
    fc2 = oracle.bf16_bits(rng.standard_normal((T * TOPK, cols)).astype(np.float32))
    wts = rng.uniform(0, 0.3, (T, TOPK)).astype(np.float32)
    gamma = oracle.bf16_bits(rng.uniform(0.5, 1.5, cols).astype(np.float32))
    return (_t(fc2, dev).view(torch.bfloat16), _t(e2p, dev), _t(wts, dev),
            _t(gamma, dev).view(torch.bfloat16))


@pytest.mark.parametrize("T,rows,cols", [(37, 64, 3584), (300, 300, 7168)])
def test_finalize(dev, T, rows, cols):
    fc2, e2p, wts, _ = _fc2_inputs(T, cols, dev, T)

    def mk():
        out = _poison((rows, cols), torch.bfloat16, dev)
        return [rk.P(fc2), rk.P(e2p), rk.P(wts), rk.P(out), rk.I(T), rk.I(cols)], out

    ro, o = _both("k3_moe_prefill", "kern_k3_moe_finalize", (rows, 1, 1), (cols // 8, 1, 1), mk)
    assert torch.equal(o.view(torch.int16), ro.view(torch.int16))


@pytest.mark.parametrize("T,rows", [(5, 8), (512, 512)])
def test_finalize_rms(dev, T, rows):
    cols = LATENT
    fc2, e2p, wts, gamma = _fc2_inputs(T, cols, dev, T + 1)

    def mk_glue():
        out = _poison((rows, cols), torch.bfloat16, dev)
        return [rk.P(fc2), rk.P(e2p), rk.P(wts), rk.P(gamma), rk.P(out), rk.I(T), rk.I(cols)], out

    ro, o = _both("k3_prefill_glue", "kern_k3g_finalize_rms", (rows, 1, 1), (cols // 8, 1, 1), mk_glue)
    assert torch.equal(o.view(torch.int16), ro.view(torch.int16))
    # the route module's variant writes the first LATENT columns of ldo-wide rows (only that entry of the
    # module runs here; its grid-barrier router entry is not launched)
    ldo = cols + 256

    def mk_route():
        out = _poison((rows, ldo), torch.bfloat16, dev)
        return [rk.P(fc2), rk.P(e2p), rk.P(wts), rk.P(gamma), rk.P(out), rk.I(ldo), rk.I(T)], out

    ro, o = _both("k3_moe_route", "kern_k3g_moe_finalize_rms", (rows, 1, 1), (cols // 8, 1, 1), mk_route)
    assert torch.equal(o.view(torch.int16), ro.view(torch.int16))


# kern_k3g_moe_route's sync words (source/k3_moe_route.cu:317-333): barrier words, two routing tables, counters
ROUTE_TABLE = E * (1 + 8192 // 256 + 8192 // 32)
ROUTE_SYNC_WORDS = 64 + 2 * ROUTE_TABLE + 2
SHARED_W = 6144


@pytest.mark.parametrize("Bs", [(64, 200), (300, 2048)])
def test_fused_route(dev, Bs):
    """The fused prefill front, two calls in a row on one sync buffer (the second on the other parity's
    table), each launched cooperatively so every block of the grid barrier is resident; all eleven outputs
    byte-equal to the reference entry's."""
    rng = np.random.default_rng(sum(Bs))
    ldx, ldgu, ldact = LATENT + 64, 2 * SHARED_W + 128, SHARED_W + 64
    bias = _t(rng.uniform(-0.1, 0.1, E).astype(np.float32), dev)
    rs = _t(oracle.bf16_bits(np.array([2.5], np.float32)), dev).view(torch.bfloat16)
    ins = []
    for B in Bs:
        S = _t(rng.standard_normal((B, E)).astype(np.float32), dev)
        x = _t(oracle.bf16_bits(rng.standard_normal((B, ldx)).astype(np.float32)), dev).view(torch.bfloat16)
        gu = _t(oracle.bf16_bits((3.0 * rng.standard_normal((B, ldgu))).astype(np.float32)), dev).view(torch.bfloat16)
        ins.append((B, S, x, gu))

    def run(module):
        f_init = rk.function(module, "kern_k3g_moe_route_init")
        f = rk.function(module, "kern_k3g_moe_route")
        sync = _poison((ROUTE_SYNC_WORDS,), torch.int32, dev)
        rk.launch(f_init, (64, 1, 1), (1024, 1, 1), [rk.P(sync)])
        outs = []
        for B, S, x, gu in ins:
            ctas = E + (B * TOPK + 127) // 128
            o = dict(q=_poison((B, LATENT), torch.uint8, dev), sf=_poison((B, LATENT // 32), torch.uint8, dev),
                     idx=_poison((B, TOPK), torch.int32, dev), wts=_poison((B, TOPK), torch.float32, dev),
                     act=_poison((B, ldact), torch.bfloat16, dev), cta_batch=_poison((ctas,), torch.int32, dev),
                     cta_limit=_poison((ctas,), torch.int32, dev), nne=_poison((1,), torch.int32, dev),
                     tp=_poison((1,), torch.int32, dev), route_map=_poison((ctas * 128,), torch.int32, dev),
                     exp2perm=_poison((B, TOPK), torch.int32, dev))
            args = [rk.P(S), rk.P(bias), rk.P(rs), rk.P(x), rk.I(ldx), rk.P(gu), rk.I(ldgu), rk.P(o["q"]),
                    rk.P(o["sf"]), rk.P(o["idx"]), rk.P(o["wts"]), rk.P(o["act"]), rk.I(ldact), rk.P(sync),
                    rk.P(o["cta_batch"]), rk.P(o["cta_limit"]), rk.P(o["nne"]), rk.P(o["tp"]), rk.P(o["route_map"]),
                    rk.P(o["exp2perm"]), rk.I(128), rk.I(B)]
            rk.launch_cooperative(f, (64 if B <= 256 else 288, 1, 1), (512, 1, 1), args)
            torch.cuda.synchronize()
            outs.append(o)
        return outs, sync

    ref, _ = run("k3_moe_route")
    got, sync = run(MOD)
    assert int(sync[1].item()) == 0, "a grid-barrier wait ran out"
    for call, (r, g) in enumerate(zip(ref, got)):
        for name in r:
            assert torch.equal(r[name].view(torch.uint8), g[name].view(torch.uint8)), f"call {call}: {name} differs"


@pytest.mark.parametrize("experts,n,K,gated", [(3, 256, 3584, 1), (2, 7168, 512, 0), (1, 64, 256, 1)])
def test_weight_shuffles(dev, experts, n, K, gated):
    """The load-time re-layouts of the checkpoint's MXFP4 rows (packed bytes) and their scales."""
    rng = np.random.default_rng(experts * n + K)
    row_bytes, kg = K // 2, K // 32
    w = _t(rng.integers(0, 256, (experts * n, row_bytes), dtype=np.uint8), dev)
    s = _t(rng.integers(0, 256, (experts * n, kg), dtype=np.uint8), dev)

    def mk_w():
        out = _poison((experts * n, row_bytes), torch.uint8, dev)
        return [rk.P(w), rk.P(out), rk.I(experts), rk.I(n), rk.I(row_bytes), rk.I(gated)], out

    total = experts * n * row_bytes // 16
    ro, o = _both("k3_moe_prefill", "kern_k3_moe_w_shuffle", ((total + 255) // 256, 1, 1), (256, 1, 1), mk_w)
    assert torch.equal(o, ro)

    def mk_sf():
        out = _poison((experts * n * kg,), torch.uint8, dev)
        return [rk.P(s), rk.P(out), rk.I(experts), rk.I(n), rk.I(kg), rk.I(gated)], out

    total = experts * n * kg
    ro, o = _both("k3_moe_prefill", "kern_k3_moe_sf_shuffle", ((total + 255) // 256, 1, 1), (256, 1, 1), mk_sf)
    assert torch.equal(o, ro)


FRONT_LDS, FRONT_SH, FRONT_STRIDE, FRONT_NSH = 6016, 768, 8, 7168
FRONT_LOCAL, FRONT_READERS, FRONT_TILE = E // FRONT_STRIDE, FRONT_NSH // 64, 16
FRONT_SMEM = 1024 + 2 * (FRONT_SH // 64) * 64 * 128 + 64 * 64 * 2
FC1_W, FC1_SF = 2 * 3072 * (LATENT // 2), 2 * 3072 * (LATENT // 32)
FRONT_CTAS = 256


@pytest.fixture(scope="module")
def front_weights(dev):
    """The shared expert's down projection [NSH, SH] bf16 and FC1 buffers the prefetcher reads (contents unused)."""
    rng = np.random.default_rng(77)
    wsh = _t(oracle.bf16_bits((0.05 * rng.standard_normal((FRONT_NSH, FRONT_SH))).astype(np.float32)),
             dev).view(torch.bfloat16)
    w13 = torch.zeros(FRONT_LOCAL * FC1_W, dtype=torch.uint8, device=dev)
    w13_sf = torch.zeros(FRONT_LOCAL * FC1_SF, dtype=torch.uint8, device=dev)
    return wsh, w13, w13_sf


def _front_inputs(T, ties, seed, dev):
    rng = np.random.default_rng(seed)
    if ties:  # many equal scores: the tie rule (smaller expert first) decides the picks
        S = (rng.integers(-6, 7, (T, FRONT_LDS)) * 0.5).astype(np.float32)
        bias = np.zeros(E, np.float32)
    else:
        S = rng.uniform(-4, 4, (T, FRONT_LDS)).astype(np.float32)
        bias = rng.uniform(-0.1, 0.1, E).astype(np.float32)
    return S, bias


def _front_run(module, calls, weights, dev):
    """Launch `module`'s kern_k3_moe_front once per (T, S, bias, rs_bits, first) in order, on one set of
    carries (ready, ids, done) zeroed once before the first call, as the manifest keeps them."""
    wsh, w13, w13_sf = weights
    f = rk.function(module, "kern_k3_moe_front")
    rk.allow_smem(f, FRONT_SMEM)
    ready = torch.zeros(FRONT_READERS * 64, dtype=torch.int32, device=dev)
    ids = torch.zeros(FRONT_READERS * 64, dtype=torch.int32, device=dev)
    done = torch.zeros(1, dtype=torch.int32, device=dev)
    outs = []
    for T, S, bias, rs_bits, first in calls:
        S_d, bias_d = _t(S, dev), _t(bias, dev)
        rs = _t(np.array([rs_bits], np.uint16), dev).view(torch.bfloat16)
        o = dict(idx=_poison((T, TOPK), torch.int32, dev), wts=_poison((T, TOPK), torch.float32, dev),
                 q=_poison((T, LATENT), torch.uint8, dev), sf=_poison((T, LATENT // 32), torch.uint8, dev),
                 act=_poison((T, FRONT_SH), torch.bfloat16, dev),
                 cta_batch=_poison((FRONT_CTAS,), torch.int32, dev), cta_limit=_poison((FRONT_CTAS,), torch.int32, dev),
                 nne=_poison((1,), torch.int32, dev), tp=_poison((1,), torch.int32, dev),
                 route_map=_poison((FRONT_CTAS * FRONT_TILE,), torch.int32, dev),
                 exp2perm=_poison((T, TOPK), torch.int32, dev), sh_out=_poison((T, FRONT_NSH), torch.bfloat16, dev))
        args = [rk.P(S_d), rk.P(bias_d), rk.P(rs), rk.P(o["idx"]), rk.P(o["wts"]), rk.P(o["q"]), rk.P(o["sf"]),
                rk.P(o["act"]), rk.P(ready), rk.P(ids), rk.P(done), rk.P(o["cta_batch"]), rk.P(o["cta_limit"]),
                rk.P(o["nne"]), rk.P(o["tp"]), rk.P(o["route_map"]), rk.P(o["exp2perm"]), rk.P(wsh),
                rk.P(o["sh_out"]), rk.P(w13), rk.P(w13_sf), rk.I(first), rk.I(T)]
        rk.launch(f, (T + FRONT_READERS, 1, 1), (1024, 1, 1), args, smem=FRONT_SMEM)
        torch.cuda.synchronize()
        o["carries"] = (int(ready.abs().sum().item()), int(ids.abs().sum().item()), int(done.item()))
        outs.append({k: (v.cpu() if isinstance(v, torch.Tensor) else v) for k, v in o.items()})
    return outs


@pytest.mark.parametrize("ties", [0, 1])
def test_decode_front(dev, front_weights, ties):
    """kern_k3_moe_front over a run of calls (1-64 rows, several ranks' expert slices) on one set of carries:
    picks, weights, the latent's MXFP8, the SiTU row and the shared expert's down projection byte-equal to
    the reference entry's; the routing tables equal to the oracle's (an expert's rows in token order) and
    to the reference's up to the order of an expert's rows (it places rows by shared-memory atomics);
    every carry back to zero after each call."""
    rs_bits = 0x4020  # 2.5
    calls = []
    for n, (T, first) in enumerate([(1, 0), (8, 3), (24, 7), (48, 1), (64, 0), (17, 5)]):
        S, bias = _front_inputs(T, ties, 1000 * ties + n, dev)
        calls.append((T, S, bias, rs_bits, first))
    ref = _front_run("k3_moe_front", calls, front_weights, dev)
    got = _front_run(MOD, calls, front_weights, dev)
    wsh = front_weights[0].float().cpu()
    for (T, S, bias, _, first), r, g in zip(calls, ref, got):
        tag = f"T={T} first={first}"
        assert g["carries"] == (0, 0, 0), f"{tag}: carries left set {g['carries']}"
        assert r["carries"] == (0, 0, 0), f"{tag}: reference carries {r['carries']}"
        for name in ("idx", "wts", "q", "sf", "act", "sh_out", "nne", "tp"):
            assert torch.equal(r[name].view(torch.uint8), g[name].view(torch.uint8)), f"{tag}: {name} differs"
        nne, tp = int(g["nne"][0]), int(g["tp"][0])
        assert torch.equal(r["cta_batch"][:nne], g["cta_batch"][:nne]) and torch.equal(r["cta_limit"][:nne],
                                                                                       g["cta_limit"][:nne])
        # the oracle: picks, the SiTU row, token-ordered tables, the projection in f32
        idx_o, wts_o = oracle.topk(S[:, :E], bias, rs_bits, TOPK)
        assert np.array_equal(g["idx"].numpy(), idx_o), tag
        # the host's expf and the device's differ by an ulp now and then: weights to 2e-6 (bit-equal to the
        # reference entry above)
        np.testing.assert_allclose(g["wts"].numpy(), wts_o, rtol=2e-6, atol=0, err_msg=tag)
        q_o, sf_o = oracle.quant_mxfp8(oracle.bf16_bits(S[:, E:E + LATENT]))
        assert np.array_equal(g["q"].numpy(), q_o) and np.array_equal(g["sf"].numpy(), sf_o), tag
        land = lambda a: oracle.bf16_to_f32(oracle.bf16_bits(a))  # noqa: E731
        gate, up = S[:, E + LATENT:E + LATENT + FRONT_SH], S[:, E + LATENT + FRONT_SH:E + LATENT + 2 * FRONT_SH]
        act_o = oracle.situ(land(gate), land(up))
        act_g = g["act"].float().numpy()
        assert np.allclose(act_g, act_o, rtol=1.6e-2, atol=1e-3), f"{tag}: SiTU off the oracle"
        tb = oracle.strided_tables(idx_o, first, FRONT_STRIDE, FRONT_LOCAL, FRONT_TILE)
        assert nne == tb["meta"][0] and tp == tb["meta"][1], tag
        assert np.array_equal(g["cta_batch"][:nne].numpy(), tb["cta_batch"][:nne]), tag
        assert np.array_equal(g["cta_limit"][:nne].numpy(), tb["cta_limit"][:nne]), tag
        assert np.array_equal(g["route_map"][:tp].numpy(), tb["route_map"][:tp]), tag
        assert np.array_equal(g["exp2perm"].numpy(), tb["exp2perm"]), tag
        # the reference's tables: the same rows per expert in another order
        e2r, rmr, cb = r["exp2perm"].numpy().ravel(), r["route_map"].numpy(), r["cta_batch"].numpy()
        e2g = g["exp2perm"].numpy().ravel()
        for i in range(T * TOPK):
            assert (e2r[i] < 0) == (e2g[i] < 0), f"{tag}: pick {i}"
            if e2r[i] >= 0:
                assert rmr[e2r[i]] == i // TOPK and cb[e2r[i] // FRONT_TILE] == cb[e2g[i] // FRONT_TILE], f"{tag}: {i}"
        pad = np.ones(tp, bool)
        pad[e2g[e2g >= 0]] = False
        assert (rmr[:tp][pad] == 0).all(), f"{tag}: reference padding rows"
        want = act_g.astype(np.float32) @ wsh.numpy().T
        got_sh = g["sh_out"].float().numpy()
        assert np.allclose(got_sh, want, rtol=1e-2, atol=2e-2 * np.abs(want).max()), f"{tag}: projection"


def test_decode_front_latency(dev, front_weights, capsys):
    """Device time of kern_k3_moe_front against the reference entry, 40 back-to-back launches a CUDA graph
    (the step's launches, S resident in L2 as the front GEMM leaves it), best of 9 replays; printed, not
    asserted (the numbers are quoted in the design notes).  Carries must be zero after every replay."""
    wsh, w13, w13_sf = front_weights
    rows = []
    for T in (1, 8, 16, 32, 64):
        S, bias = _front_inputs(T, 0, 500 + T, dev)
        line = [T]
        for module in ("k3_moe_front", MOD):
            f = rk.function(module, "kern_k3_moe_front")
            rk.allow_smem(f, FRONT_SMEM)
            ready = torch.zeros(FRONT_READERS * 64, dtype=torch.int32, device=dev)
            ids = torch.zeros_like(ready)
            done = torch.zeros(1, dtype=torch.int32, device=dev)
            S_d, b_d = _t(S, dev), _t(bias, dev)
            rs = _t(np.array([0x4020], np.uint16), dev).view(torch.bfloat16)
            o = [torch.zeros(n, dtype=torch.int32, device=dev) for n in
                 (T * TOPK, T * TOPK, T * LATENT // 4, T * LATENT // 128, T * FRONT_SH // 2, FRONT_CTAS, FRONT_CTAS,
                  1, 1, FRONT_CTAS * FRONT_TILE, T * TOPK, T * FRONT_NSH // 2)]
            args = [rk.P(S_d), rk.P(b_d), rk.P(rs)] + [rk.P(x) for x in o[:5]] + [rk.P(ready), rk.P(ids), rk.P(done)] + \
                   [rk.P(x) for x in o[5:11]] + [rk.P(wsh), rk.P(o[11]), rk.P(w13), rk.P(w13_sf), rk.I(0), rk.I(T)]
            grid = (T + FRONT_READERS, 1, 1)
            for _ in range(3):
                rk.launch(f, grid, (1024, 1, 1), args, smem=FRONT_SMEM)
            torch.cuda.synchronize()
            side = torch.cuda.Stream()
            g = torch.cuda.CUDAGraph()
            with torch.cuda.stream(side):
                with torch.cuda.graph(g, stream=side):
                    for _ in range(40):
                        rk.launch(f, grid, (1024, 1, 1), args, smem=FRONT_SMEM)
            g.replay()
            torch.cuda.synchronize()
            best = float("inf")
            for _ in range(9):
                e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                e0.record()
                g.replay()
                e1.record()
                e1.synchronize()
                best = min(best, e0.elapsed_time(e1) * 1e3 / 40)
            g.reset()
            assert int(done.item()) == 0 and int(ready.abs().sum()) == 0 and int(ids.abs().sum()) == 0, module
            line.append(best)
        rows.append(line)
    with capsys.disabled():
        print("\nkern_k3_moe_front device time a launch (us): rows, reference, k3moe")
        for T, r, k in rows:
            print(f"  {T:3d}  {r:7.2f}  {k:7.2f}")


@pytest.mark.parametrize("B,n", [(1, 768), (37, 6144), (5, 1032)])
def test_situ(dev, B, n):
    """kern_k3g_situ: K3's shared-expert SiTU on bf16 [gate | up] rows, byte-equal to the reference entry,
    including gates below -87 (where the reference leaves its fast reciprocal for the IEEE one)."""
    rng = np.random.default_rng(B * n)
    p = (4.0 * rng.standard_normal((B, 2 * n))).astype(np.float32)
    p[:, : min(16, n)] = -100.0
    pb = _t(oracle.bf16_bits(p), dev).view(torch.bfloat16)

    def mk():
        out = _poison((B, n), torch.bfloat16, dev)
        return [rk.P(pb), rk.P(out), rk.I(n), rk.I(B)], out

    grid = (B, -(-n // 2048), 1)
    ro, o = _both("k3_prefill_glue", "kern_k3g_situ", grid, (256, 1, 1), mk)
    assert torch.equal(o.view(torch.int16), ro.view(torch.int16))
    land = oracle.bf16_to_f32(oracle.bf16_bits(p))
    want = oracle.situ(land[:, :n], land[:, n:])
    assert np.allclose(o.float().cpu().numpy(), want, rtol=1.6e-2, atol=1e-3)


@pytest.mark.parametrize("B", [1, 7, 64])
def test_decode_router_topk(dev, B):
    """kern_k3_router_topk (the decode router's entry, one block a row): ids and weight bits byte-equal to the
    reference entry's."""
    rng = np.random.default_rng(100 + B)
    S = _t((2.0 * rng.standard_normal((B, E))).astype(np.float32), dev)
    bias = _t(rng.uniform(-0.1, 0.1, E).astype(np.float32), dev)
    rs = _t(oracle.bf16_bits(np.array([2.5], np.float32)), dev).view(torch.bfloat16)

    def mk():
        i, w = _poison((B, TOPK), torch.int32, dev), _poison((B, TOPK), torch.float32, dev)
        return [rk.P(S), rk.P(bias), rk.P(rs), rk.P(i), rk.P(w), rk.I(B)], (i, w)

    (ri, rw), (i, w) = _both("k3_router_argmax", "kern_k3_router_topk", (B, 1, 1), (1024, 1, 1), mk)
    assert torch.equal(i, ri) and torch.equal(w.view(torch.int32), rw.view(torch.int32))
