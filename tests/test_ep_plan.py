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
