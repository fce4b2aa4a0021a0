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


# ------------------------------------------------------------------ the peer-memory transport's kernels, one GPU
def test_pack_pairs_to_lands_rows_where_the_all_to_all_would(setup):
    """k3moe_ep_pack_pairs_to with every rank's receive buffer local (three ranks' buffers on this GPU, this
    rank = 1): the rows for rank d land at peer_offsets' shift, the same bytes as the contiguous pack."""
    c, g, gops, oops = setup
    Wn, me = 3, 1
    idx, wts = gops.topk(g["S"], g["bias"], g["rs"], K)
    dest = (idx % Wn).to(torch.int32).contiguous()
    lid = (idx // Wn).to(torch.int32).contiguous()
    pairs = gops.pairs(dest, Wn)
    rplan = gops.tables(pairs, Wn, 1)
    rows_to = rplan.counts[:Wn].tolist()
    n = sum(rows_to)
    flat = gops.pack_pairs(g["x"], dest, lid, rplan.exp2perm.reshape(c.T, Wn), Wn, n)
    st = flat.shape[1]
    # counts of the other two (made-up) ranks, so this rank's rows land after theirs at some destinations
    C = [[(5, 9), (0, 0), (3, 4)], [(r, r) for r in rows_to], [(2, 2), (7, 8), (0, 0)]]
    lay = k3moe_ep.peer_offsets(C, me)
    bufs = [torch.full((lay["recv_rows"][d] + 4, st), 0xA5, dtype=torch.uint8, device=flat.device) for d in range(Wn)]
    base = [bufs[d].data_ptr() + lay["shift"][d] * st for d in range(Wn)]
    gops.pack_pairs_to(g["x"], dest, lid, rplan.exp2perm.reshape(c.T, Wn), Wn, base, st)
    torch.cuda.synchronize()
    used = H + H // 32 + 2 * K
    slot0 = 0
    for d in range(Wn):
        land = sum(C[s][d][0] for s in range(me))
        got = bufs[d][land:land + rows_to[d], :used]
        assert torch.equal(got, flat[slot0:slot0 + rows_to[d], :used]), f"destination {d}"
        assert bool((bufs[d][:land] == 0xA5).all()) and bool((bufs[d][land + rows_to[d]:] == 0xA5).all())
        slot0 += rows_to[d]


def test_fc2_to_row_pointers_equals_fc2_to_rows(setup):
    """FC2 storing each permuted row through a pointer table (k3moe_ep_row_ptrs over four blocks, the last empty)
    equals FC2 storing row out_rows[r] of one buffer.  The tables number every permuted row through exp2perm (no
    shared expert folded in, as on the receiving rank of the expert-parallel layer, where the shared rows arrive
    as ordinary rows): k3moe_ep_return_rows then gives every real row its number."""
    c, g, gops, oops = setup
    idx, _ = gops.topk(g["S"], g["bias"], g["rs"], K)
    tb = k3moe.route_tables(idx, E, 0, 0)
    qp, sfp = k3moe.quant_permute(g["x"], tb)
    f1q, f1sf = k3moe.fc1(g["w13"], g["w13_sf"], qp, sfp, tb, H, I, E + SH, gops.err)
    out_rows = gops.return_rows(tb, c.T, K)
    P = c.T * K
    P_all = P
    ref = torch.zeros((P_all, H), dtype=torch.bfloat16, device=qp.device)
    k3moe._check(k3moe.lib().k3moe_fc2_to_rows(
        g["w2"].data_ptr(), g["w2_sf"].data_ptr(), f1q.data_ptr(), f1sf.data_ptr(), tb.cta_batch.data_ptr(),
        tb.cta_limit.data_ptr(), tb.meta.data_ptr(), out_rows.data_ptr(), ref.data_ptr(), H, I, E + SH, tb.cap_rows,
        tb.max_ctas, gops.err.data_ptr(), k3moe._stream()), "fc2_to_rows")
    # the same rows split over four buffers: [0, a), [a, b), [b, P) and an empty block [P, P)
    cuts = [0, P // 3, (2 * P) // 3, P, P_all]
    bufs = [torch.zeros((cuts[i + 1] - cuts[i] + 3, H), dtype=torch.bfloat16, device=qp.device) for i in range(4)]
    sink = torch.zeros(H, dtype=torch.bfloat16, device=qp.device)
    ptrs = gops.row_ptrs(tb, c.T, K, out_rows, [b.data_ptr() + 3 * H * 2 for b in bufs], cuts, H * 2, sink)
    gops.fc2_to_ptrs(g, f1q, f1sf, tb, H, I, E + SH, ptrs)
    torch.cuda.synchronize()
    assert gops.err[:2].tolist() == [0, 0]
    for i in range(4):
        assert torch.equal(bufs[i][3:].view(torch.int16), ref[cuts[i]:cuts[i + 1]].view(torch.int16)), f"block {i}"
        assert bool((bufs[i][:3] == 0).all())
    assert bool((sink == 0).all())


def test_signal_writes_the_peers_slots(dev):
    Wn, me, epoch = 4, 2, 7
    flags = [torch.zeros(2 * Wn, dtype=torch.int32, device=dev) for _ in range(Wn)]
    ops = k3moe_ep.GpuOps(dev)
    ops.signal([f.data_ptr() for f in flags], Wn, me, Wn, epoch)
    torch.cuda.synchronize()
    for s in range(Wn):
        want = [0] * (2 * Wn)
        if s != me:
            want[Wn + me] = epoch
        assert flags[s].tolist() == want


def test_wait_returns_an_error_when_a_flag_is_never_set(dev):
    """Failure detection on the device: a wait whose flags nothing sets gives up after its 1 ms budget, records
    the late source in the error words and returns; the context stays usable and the host reads the status."""
    import time

    Wn, skip = 4, 0
    flags = torch.zeros(Wn, dtype=torch.int32, device=dev)
    flags[1] = 3  # source 1 arrived; 2 and 3 never do
    ops = k3moe_ep.GpuOps(dev)
    t0 = time.perf_counter()
    ops.wait(flags, Wn, skip, 3, 1_000_000)
    rc, words = k3moe.read_error(ops.err)
    dt = time.perf_counter() - t0
    assert rc == -6 and words[0] & 1 and words[1] in (0xA02, 0xA03), (rc, [hex(w) for w in words])
    assert dt < 2.0
    # the context still works, and a wait whose flags are all set records nothing
    flags.fill_(3)
    ops.wait(flags, Wn, skip, 3, 1_000_000)
    rc, words = k3moe.read_error(ops.err)
    assert rc == 0 and words == (0, 0)
    x = torch.ones(1024, device=dev)
    assert float(x.sum().item()) == 1024.0
