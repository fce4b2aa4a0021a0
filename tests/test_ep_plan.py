"""CPU tests of the expert-parallel plans (no GPU, no process group): the expert placement and the
(token, rank) pair plan that decides how many rows cross the links."""
import numpy as np
import pytest
import torch

import ep_oracle_ops
import k3moe_ep
import oracle


@pytest.mark.parametrize("world", [2, 4, 8])
def test_balanced_owner_evens_the_modelled_load(world):
    """Every rank gets E / world experts, and the load modelled from the router bias (an expert's pick rate
    growing with its bias) is within 0.5% of even, better than contiguous blocks."""
    E = 896
    rng = np.random.default_rng(world)
    bias = rng.uniform(-0.1, 0.1, E).astype(np.float32)
    owner = k3moe_ep.balanced_owner(bias, world).numpy()
    assert np.bincount(owner, minlength=world).tolist() == [E // world] * world
    load = np.exp(10.0 * bias)                     # pick rate rising with the bias (0.37x .. 2.7x)
    per = np.bincount(owner, weights=load, minlength=world)
    assert per.max() / per.mean() < 1.005
    contiguous = np.bincount(np.arange(E) // (E // world), weights=load, minlength=world)
    assert per.max() / per.mean() < contiguous.max() / contiguous.mean()


@pytest.mark.parametrize("world,K", [(2, 8), (4, 8), (8, 8), (8, 16)])
def test_pair_plan_rows_per_token(world, K):
    """One row a (token, rank) pair: with uniform routing a token's K picks land on about
    world * (1 - (1 - 1/world)^K) ranks, and the plan's slots are dense and grouped by rank in token order."""
    T, E = 512, 896
    rng = np.random.default_rng(world * 100 + K)
    idx = np.stack([rng.choice(E, K, replace=False) for _ in range(T)]).astype(np.int32)
    dest = torch.from_numpy((idx // (E // world)).astype(np.int32))
    ops = ep_oracle_ops.OracleOps()
    pairs = ops.pairs(dest, world).numpy()
    rows = int((pairs >= 0).sum())
    expect = T * world * (1 - (1 - 1 / world) ** K)
    assert abs(rows - expect) < 0.05 * expect
    assert rows < T * K
    plan = oracle.tables(pairs, world, 0, 0, 1)
    slots = plan["exp2perm"][pairs >= 0]
    assert np.array_equal(np.sort(slots), np.arange(rows))
    for r in range(world):  # rank r's slots: one block, tokens in order
        s = plan["exp2perm"][:, r][pairs[:, r] >= 0]
        assert (np.diff(s) == 1).all()


@pytest.mark.parametrize("world", [1, 2, 3, 8, 16])
def test_peer_offsets_reproduce_the_all_to_all_layouts(world):
    """The peer transport's store addresses (k3moe_ep.peer_offsets) put every dispatched row and every returned
    result where the two all-to-alls would: received rows grouped by source rank, results grouped by the rank
    that computed them, each block in its sender's order.  Checked against a simulation of the all-to-alls for
    random count matrices, empty blocks included."""
    rng = np.random.default_rng(world)
    for trial in range(20):
        C = rng.integers(0, 5, (world, world, 2))
        C[:, :, 1] += C[:, :, 0]          # picks >= rows (a row carries one or more picks)
        if trial % 4 == 0:
            C[rng.integers(0, world), :, :] = 0   # a rank that sends nothing
        lay = [k3moe_ep.peer_offsets(C.tolist(), r) for r in range(world)]
        # dispatch: source s's slot p for rank d (slots grouped by destination) -> row p + shift[d] at d
        for d in range(world):
            want = [(s, j) for s in range(world) for j in range(C[s, d, 0])]   # the all-to-all's receive order
            got = {}
            for s in range(world):
                slot0 = int(C[s, :d, 0].sum())
                for j in range(C[s, d, 0]):
                    got[slot0 + j + lay[s]["shift"][d]] = (s, j)
            assert [got[i] for i in range(len(want))] == want and len(got) == len(want)
            assert lay[d]["R_recv"] == len(want) == lay[0]["recv_rows"][d]
        # combine: at computing rank d, result q of source s (q in [pstart[s], pstart[s+1])) -> row
        # back_row0[s] + q - pstart[s] of s's return buffer, which the all-to-all fills grouped by computing rank
        for s in range(world):
            want = [(d, j) for d in range(world) for j in range(C[s, d, 1])]
            got = {}
            for d in range(world):
                L = lay[d]
                for q in range(L["pstart"][s], L["pstart"][s + 1]):
                    got[L["back_row0"][s] + q - L["pstart"][s]] = (d, q - L["pstart"][s])
            assert [got[i] for i in range(len(want))] == want and len(got) == len(want)
            assert lay[0]["back_rows"][s] == len(want)
