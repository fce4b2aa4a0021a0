"""GPU parity of the bandwidth kernels against the CPU oracle, through the C ABI.

Integer / byte outputs (top-k ids, tables, MXFP8 and MXFP4 bytes and scales,
the combine's bf16 bits) must match bit for bit."""
import numpy as np
import pytest
import torch

import cases
import k3moe
import oracle

pytestmark = pytest.mark.gpu


def _t(a, dev):
    return torch.from_numpy(np.ascontiguousarray(a)).to(dev)


@pytest.mark.parametrize("T,E,K,rs", [(1, 896, 8, 2.5), (64, 896, 8, 2.5), (300, 896, 16, 1.0), (128, 16, 4, 1.0),
                                      (2048, 256, 8, 2.5), (8192, 896, 8, 2.5)])
def test_topk_matches_oracle(dev, T, E, K, rs):
    rng = np.random.default_rng(T * 7 + E)
    S = rng.standard_normal((T, E), dtype=np.float32)
    bias = rng.uniform(-0.1, 0.1, E).astype(np.float32)
    rs_bits = int(oracle.bf16_bits(np.array([rs], np.float32))[0])
    ref_idx, ref_w = oracle.topk(S, bias, rs_bits, K)
    idx, w = k3moe.route_topk(_t(S, dev), _t(bias, dev), _t(np.array([rs_bits], np.uint16), dev).view(torch.bfloat16), K)
    idx, w = idx.cpu().numpy(), w.cpu().numpy()
    assert np.array_equal(idx, ref_idx), f"{(idx != ref_idx).any(1).sum()} rows differ"
    np.testing.assert_allclose(w, ref_w, rtol=2e-6, atol=0)


def test_topk_forced_tie_takes_smaller_expert(dev):
    # the reference harness pins "tie -> smaller e" with equal keys at experts 40/41 (harness/k3/harness.cu:697-709)
    T, E, K = 8, 896, 16
    rng = np.random.default_rng(5)
    S = (rng.standard_normal((T, E)) * 2).astype(np.float32)
    bias = (rng.standard_normal(E) * 0.1).astype(np.float32)
    bias[40] = bias[41] = 0.5
    S[:, 40] = S[:, 41] = 6.0
    rs_bits = int(oracle.bf16_bits(np.array([2.5], np.float32))[0])
    idx, _ = k3moe.route_topk(_t(S, dev), _t(bias, dev), _t(np.array([rs_bits], np.uint16), dev).view(torch.bfloat16), K)
    idx = idx.cpu().numpy()
    for row in idx:
        assert list(row).index(40) + 1 == list(row).index(41)


@pytest.mark.parametrize("R,K,E,first,shared", [(1, 8, 896, 0, 0), (300, 8, 896, 0, 1), (8192, 8, 896, 0, 1),
                                                (1000, 16, 64, 128, 0), (513, 4, 16, 0, 0), (4096, 8, 112, 224, 0)])
def test_tables_match_oracle(dev, R, K, E, first, shared):
    rng = np.random.default_rng(R + E)
    E_total = max(first + E + 37, 896)
    idx = np.stack([rng.choice(E_total, K, replace=False) for _ in range(R)]).astype(np.int32)
    ref = oracle.tables(idx, E, first, shared)
    t = k3moe.route_tables(_t(idx, dev), E, first, shared)
    nne = int(ref["meta"][0])
    assert t.max_ctas == ref["max_ctas"]
    assert np.array_equal(t.meta.cpu().numpy()[:3], ref["meta"][:3])
    assert np.array_equal(t.counts.cpu().numpy(), ref["counts"])
    assert np.array_equal(t.cta_batch.cpu().numpy()[:nne], ref["cta_batch"][:nne])
    assert np.array_equal(t.cta_limit.cpu().numpy()[:nne], ref["cta_limit"][:nne])
    assert np.array_equal(t.exp2perm.cpu().numpy(), ref["exp2perm"])
    tp = int(ref["meta"][1])
    assert np.array_equal(t.route_map.cpu().numpy()[:tp], ref["route_map"][:tp])


@pytest.mark.parametrize("rows,cols,tiled", [(1, 256, 0), (130, 1024, 0), (130, 1024, 1), (4096, 7168, 0),
                                             (4096, 7168, 1), (257, 3584, 1)])
def test_quant_mxfp8_bit_exact(dev, rows, cols, tiled):
    rng = np.random.default_rng(rows + cols)
    x = (rng.standard_normal((rows, cols)) * np.exp(rng.uniform(-8, 8, (rows, 1)))).astype(np.float32)
    x[0, :32] = 0.0          # an all-zero group: exponent 0
    x[-1, 32:64] = 448.0      # an exact power-of-two quotient
    xb = oracle.bf16_bits(x)
    ref_q, ref_sf = oracle.quant_mxfp8(xb, tiled=bool(tiled))
    q, sf = k3moe.quant_mxfp8(_t(xb, dev).view(torch.bfloat16), tiled_sf=bool(tiled))
    assert np.array_equal(q.cpu().numpy(), ref_q)
    if tiled:
        # only the bytes of real rows are defined
        kg4 = -(-cols // 128)
        r = np.arange(rows)[:, None]
        kb = np.arange(cols // 32)[None, :]
        off = ((r // 128) * kg4 + kb // 4) * 512 + (r % 32) * 16 + ((r % 128) // 32) * 4 + kb % 4
        assert np.array_equal(sf.cpu().numpy()[off], ref_sf[off])
    else:
        assert np.array_equal(sf.cpu().numpy(), ref_sf)


def test_quant_mxfp8_every_bf16_amax(dev):
    # every positive finite bf16 as a group's amax (the rest of the group a fixed pattern below it)
    amax_bits = np.arange(0x0001, 0x7F80, dtype=np.uint32)
    amax = oracle.bf16_to_f32(amax_bits.astype(np.uint16))
    frac = np.linspace(-1, 1, 31, dtype=np.float32)
    x = np.concatenate([amax[:, None], amax[:, None] * frac[None, :]], axis=1)
    cols = 256
    n = x.shape[0]
    rows = -(-n // 8)
    buf = np.zeros((rows * 8, 32), np.float32)
    buf[:n] = x
    xb = oracle.bf16_bits(buf.reshape(rows, cols))
    ref_q, ref_sf = oracle.quant_mxfp8(xb, tiled=False)
    q, sf = k3moe.quant_mxfp8(_t(xb, dev).view(torch.bfloat16), tiled_sf=False)
    assert np.array_equal(sf.cpu().numpy(), ref_sf)
    assert np.array_equal(q.cpu().numpy(), ref_q)


@pytest.mark.parametrize("T,H,E,K,shared", [(128, 1024, 16, 4, 0), (300, 7168, 896, 8, 1)])
def test_quant_permute_bit_exact(dev, T, H, E, K, shared):
    rng = np.random.default_rng(T)
    idx = np.stack([rng.choice(E, K, replace=False) for _ in range(T)]).astype(np.int32)
    xb = oracle.bf16_bits(rng.standard_normal((T, H)).astype(np.float32))
    ref = oracle.tables(idx, E, 0, shared)
    ref_q, ref_sf = oracle.quant_permute(xb, ref["exp2perm"], ref["meta"], ref["cap_rows"])
    t = k3moe.route_tables(_t(idx, dev), E, 0, shared)
    qp, sfp = k3moe.quant_permute(_t(xb, dev).view(torch.bfloat16), t)
    rows = np.unique(ref["exp2perm"][ref["exp2perm"] >= 0])
    if shared:
        rows = np.concatenate([rows, ref["meta"][2] + np.arange(T)])
    qp = qp.cpu().numpy()
    assert np.array_equal(oracle.t128_rows(qp, rows, H), oracle.t128_rows(ref_q, rows, H))
    sfp = sfp.cpu().numpy()
    kg4 = H // 128
    r = rows[:, None].astype(np.int64)
    kb = np.arange(H // 32)[None, :]
    off = ((r // 128) * kg4 + kb // 4) * 512 + (r % 32) * 16 + ((r % 128) // 32) * 4 + kb % 4
    assert np.array_equal(sfp[off], ref_sf[off])


@pytest.mark.parametrize("T,H,E,K,shared,out_rows", [(64, 7168, 896, 8, 1, 64), (100, 1024, 16, 4, 0, 128)])
def test_combine_bit_exact(dev, T, H, E, K, shared, out_rows):
    rng = np.random.default_rng(T + H)
    idx = np.stack([rng.choice(E, K, replace=False) for _ in range(T)]).astype(np.int32)
    idx[0, 1] = E + 5  # a foreign expert: exp2perm -1, skipped
    tb = oracle.tables(idx, E, 0, shared)
    cap = tb["cap_rows"]
    fc2 = oracle.bf16_bits(rng.standard_normal((cap, H)).astype(np.float32))
    wts = rng.uniform(0, 0.5, (T, K)).astype(np.float32)
    ref = oracle.combine(fc2, tb["exp2perm"], wts, tb["meta"], T, K, out_rows)
    t = k3moe.route_tables(_t(idx, dev), E, 0, shared)
    out = k3moe.combine(_t(fc2, dev).view(torch.bfloat16), t, _t(wts, dev), T, out_rows)
    assert np.array_equal(out.view(torch.int16).cpu().numpy().view(np.uint16), ref)


@pytest.mark.parametrize("rows,K", [(256, 1024), (384, 7168), (7168, 2048)])
def test_quant_mxfp4_bit_exact(dev, rows, K):
    rng = np.random.default_rng(rows)
    w = rng.normal(0, 0.02, (rows, K)).astype(np.float32)
    w[0, :32] = 0.0
    w[1, :32] = np.array([0.25, 0.75, 1.25, 1.75, 2.5, 3.5, 5.0, 7.9] * 4, np.float32)  # E2M1 ties, saturation
    ref_p, ref_sf = oracle.quant_mxfp4(w)
    p, sf = k3moe.quant_mxfp4(_t(w, dev))
    assert np.array_equal(p.cpu().numpy(), ref_p)
    assert np.array_equal(sf.cpu().numpy(), ref_sf)


def test_synth_mxfp4_matches_host_stream(dev):
    rows, K, seed = 256, 2048, 1234
    w = oracle.synth_f32(seed, rows, K, 0.02, row0=128)
    ref_p, ref_sf = oracle.quant_mxfp4(w)
    p, sf = k3moe.synth_mxfp4(seed, rows, K, 0.02, device=dev, row0=128)
    assert np.array_equal(p.cpu().numpy(), ref_p)
    assert np.array_equal(sf.cpu().numpy(), ref_sf)
