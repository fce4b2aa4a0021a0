"""Each step of the expert-parallel layer on one GPU against its oracle-built
counterpart (tests/ep_oracle_ops.py), on the same inputs: the send plan, the
packed wire rows, the received ids, the unpacked GEMM operand, FC1+FC2 with
rows stored in receive order, and the owner-side combine."""
import numpy as np
import pytest
import torch

import cases
import ep_oracle_ops
import k3moe
import k3moe_ep
import oracle

pytestmark = pytest.mark.gpu

H, I, E, K, SH, W = 1024, 512, 16, 4, 1, 2
El = E // W


@pytest.fixture(scope="module")
def setup(dev):
    c = cases.make_case(T=200, H=H, I=I, E=E, K=K, shared=SH, rs=2.5, seed=7)
    g = cases.to_device(c, dev)
    gops, oops = k3moe_ep.GpuOps(dev), ep_oracle_ops.OracleOps()
    return c, g, gops, oops


def _np(t):
    return t.detach().cpu().numpy()


def test_pack_plan_ids(setup):
    c, g, gops, oops = setup
    idx, wts = gops.topk(g["S"], g["bias"], g["rs"], K)
    plan_g = gops.tables((idx // El).to(torch.int32).reshape(-1, 1).contiguous(), W, 1)
    plan_o = oops.tables((idx // El).to(torch.int32).reshape(-1, 1).cpu(), W, 1)
    assert np.array_equal(_np(plan_g.exp2perm), _np(plan_o.exp2perm))
    assert np.array_equal(_np(plan_g.counts), _np(plan_o.counts))
    n = c.T * K
    sg = gops.pack(g["x"], idx, plan_g.exp2perm.reshape(c.T, K), El, n)
    so = oops.pack(g["x"].cpu(), idx.cpu(), plan_o.exp2perm.reshape(c.T, K), El, n)
    used = H + H // 32 + 4
    assert np.array_equal(_np(sg)[:, :used], _np(so)[:, :used])
    ids_g = gops.ids(sg, n, H)
    ids_o = oops.ids(so, n, H)
    assert np.array_equal(_np(ids_g), _np(ids_o))


def test_unpack_ffn_combine(setup):
    c, g, gops, oops = setup
    # rows as if received: every pick of this rank's tokens that lands on rank 0's experts, then the shared rows
    idx, wts = gops.topk(g["S"], g["bias"], g["rs"], K)
    plan = gops.tables((idx // El).to(torch.int32).reshape(-1, 1).contiguous(), W, 1)
    send_pos = plan.exp2perm.reshape(c.T, K)
    n = c.T * K
    sent = gops.pack(g["x"], idx, send_pos, El, n)
    r0 = int(plan.counts[0])  # slots bound for rank 0 come first
    R = r0 + c.T
    recv = torch.empty((R, sent.shape[1]), dtype=torch.uint8, device=sent.device)
    recv[:r0] = sent[:r0]
    gops.pack_rows(g["x"], El, recv[r0:R])
    ids = gops.ids(recv, R, H)
    tb_g = gops.tables(ids, El + SH, 128)
    tb_o = oops.tables(ids.cpu(), El + SH, 128)
    assert np.array_equal(_np(tb_g.exp2perm), _np(tb_o.exp2perm))
    qp_g, sfp_g = gops.unpack(recv, R, H, tb_g)
    qp_o, sfp_o = oops.unpack(recv.cpu(), R, H, tb_o)
    rows = np.unique(_np(tb_g.exp2perm).reshape(-1))
    assert np.array_equal(oracle.t128_rows(_np(qp_g), rows, H), oracle.t128_rows(qp_o, rows, H))
    r = rows[:, None].astype(np.int64)
    kb = np.arange(H // 32)[None, :]
    off = ((r // 128) * (H // 128) + kb // 4) * 512 + (r % 32) * 16 + ((r % 128) // 32) * 4 + kb % 4
    assert np.array_equal(_np(sfp_g)[off], sfp_o[off])
    # FFN with rows stored in receive order, rank 0's experts [0, El) and the shared expert
    t = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(sent.device)
    w = k3moe_ep.slice_weights(t(c.w13), t(c.w13_sf), t(c.w2), t(c.w2_sf), E, SH, 0, W, H, I)
    y_g = gops.ffn(w, qp_g, sfp_g, tb_g, H, I, El + SH, R)
    y_o = oops.ffn({k: v.cpu() for k, v in w.items()}, qp_o, sfp_o, tb_o, H, I, El + SH, R)
    ok, rel, ratio = cases.within_contract(y_g.float().cpu().numpy(), y_o.float().numpy())
    assert ok, f"ffn rel-L2 {rel:.3e} worst {ratio:.2f}"
    # combine: the oracle's arithmetic over the same returned rows
    back = torch.zeros((n, H), dtype=torch.bfloat16, device=sent.device)
    back[:r0] = y_g[:r0]
    out_g = gops.combine(back, send_pos, wts, y_g[r0:R], c.T, K, H)
    out_o = oops.combine(back.cpu(), send_pos.cpu(), wts.cpu(), y_g[r0:R].cpu(), c.T, K, H)
    assert torch.equal(out_g.cpu().view(torch.int16), out_o.view(torch.int16))


def test_pair_rows_plan_pack_unpack_return(setup):
    """The per-destination dispatch on one GPU against the oracle ops: the (token, rank) pairs and their plan,
    the packed rows with their id headers, the received ids (K a row), the unpacked operand at every expert
    of a row, and the return-row map FC2 stores by."""
    c, g, gops, oops = setup
    idx, _ = gops.topk(g["S"], g["bias"], g["rs"], K)
    dest = (idx // El).to(torch.int32).contiguous()
    lid = (idx - dest * El).to(torch.int32).contiguous()
    pairs_g = gops.pairs(dest, W)
    pairs_o = oops.pairs(dest.cpu(), W)
    assert np.array_equal(_np(pairs_g), _np(pairs_o))
    rplan = gops.tables(pairs_g, W, 1)
    n_pairs = int(rplan.counts[:W].sum())
    assert n_pairs < c.T * K  # several picks of a token share a rank
    pp = rplan.exp2perm.reshape(c.T, W)
    sg = gops.pack_pairs(g["x"], dest, lid, pp, W, c.T * min(W, K))
    so = oops.pack_pairs(g["x"].cpu(), dest.cpu(), lid.cpu(), pp.cpu(), W, c.T * min(W, K))
    used = H + H // 32 + 2 * K
    assert np.array_equal(_np(sg)[:n_pairs, :used], _np(so)[:n_pairs, :used])
    # received: rank 0's rows, then the shared expert's local rows
    r0 = int(rplan.counts[0])
    R = r0 + c.T
    recv = torch.empty((R, sg.shape[1]), dtype=torch.uint8, device=sg.device)
    recv[:r0] = sg[:r0]
    gops.pack_pair_rows(g["x"], K, El, recv[r0:R])
    recv_o = recv.cpu().clone()
    oops.pack_pair_rows(g["x"].cpu(), K, El, recv_o[r0:R])
    assert np.array_equal(_np(recv)[:, :used], _np(recv_o)[:, :used])
    ids = gops.ids_k(recv, R, H, K)
    assert np.array_equal(_np(ids), _np(oops.ids_k(recv_o, R, H, K)))
    assert int((ids >= 0).sum()) == int((dest == 0).sum()) + c.T  # every pick bound for rank 0, and the shared
    tb_g = gops.tables(ids, El + SH, 128)
    tb_o = oops.tables(ids.cpu(), El + SH, 128)
    assert np.array_equal(_np(tb_g.exp2perm), _np(tb_o.exp2perm))
    qp_g, sfp_g = gops.unpack_k(recv, R, H, K, tb_g)
    qp_o, sfp_o = oops.unpack_k(recv_o, R, H, K, tb_o)
    rows = np.unique(_np(tb_g.exp2perm).reshape(-1))
    rows = rows[rows >= 0]
    assert np.array_equal(oracle.t128_rows(_np(qp_g), rows, H), oracle.t128_rows(qp_o, rows, H))
    r = rows[:, None].astype(np.int64)
    kb = np.arange(H // 32)[None, :]
    off = ((r // 128) * (H // 128) + kb // 4) * 512 + (r % 32) * 16 + ((r % 128) // 32) * 4 + kb % 4
    assert np.array_equal(_np(sfp_g)[off], sfp_o[off])
    ret_g = _np(gops.return_rows(tb_g, R, K))
    ret_o = _np(oops.return_rows(tb_o, R, K))
    assert np.array_equal(ret_g[rows], ret_o[rows])
    assert np.array_equal(np.sort(ret_g[rows]), np.arange(rows.size))
