"""Host-side check of the device-resident expert-parallel step's addressing (k3moe_ep_forward; the kernels
ep_plan_kernel, ep_pack_pairs_kernel with return indices, ep_ids_k_kernel over regions and
ep_step_ptrs_kernel): the step's plans restated with numpy, then W ranks emulated on the host with every row
stored at the address the kernels compute.  Each FC2 result is replaced by a tag naming its (token, expert);
the owner's combine must find, at send_pos of every pick, the tag of exactly that pick.  Runs on the CPU."""
import numpy as np
import pytest


def plan(idx, W, El, owner=None):
    """ep_plan_kernel: (dest, lid, pair_pos, pair_back, send_pos, rows_to) of one rank's tokens."""
    T, K = idx.shape
    if owner is None:
        dest = idx // El
        lid = idx - dest * El
    else:
        owner = np.asarray(owner)
        local = np.zeros_like(owner)
        for r in range(W):
            mine = np.nonzero(owner == r)[0]
            local[mine] = np.arange(len(mine))
        dest, lid = owner[idx], local[idx]
    c = np.zeros((T, W), np.int64)  # picks of token t on rank d
    for k in range(K):
        np.add.at(c, (np.arange(T), dest[:, k]), 1)
    on = c > 0
    rows_to = on.sum(0)
    first = np.concatenate([[0], np.cumsum(c.sum(0))[:-1]])  # return indices grouped by destination
    before = np.cumsum(c, 0) - c                                # picks on d of the tokens before t
    pair_pos = np.where(on, np.cumsum(on, 0) - 1, -1)
    pair_back = np.where(on, first[None, :] + before, -1)
    send_pos = np.empty((T, K), np.int64)
    for t in range(T):
        seen = np.zeros(W, np.int64)
        for k in range(K):
            d = dest[t, k]
            send_pos[t, k] = first[d] + before[t, d] + seen[d]
            seen[d] += 1
    return dest, lid, pair_pos, pair_back, send_pos, rows_to


def emulate(idx_by_rank, W, El, K, T_max, owner=None):
    """Every rank's step; returns, per rank, back[send_pos] as (token, global expert) tags."""
    glob = []  # global expert of (rank, local id)
    for r in range(W):
        if owner is None:
            glob.append(np.arange(r * El, (r + 1) * El))
        else:
            glob.append(np.nonzero(np.asarray(owner) == r)[0])
    plans = [plan(idx, W, El, owner) for idx in idx_by_rank]
    # dispatch: rank s's row for rank d at region s, row pair_pos (ids of its picks there in k order, back index)
    recv = [[[None] * T_max for _ in range(W)] for _ in range(W)]
    counts = np.zeros((W, W), np.int64)
    for s in range(W):
        dest, lid, pair_pos, pair_back, _, rows_to = plans[s]
        T = dest.shape[0]
        for t in range(T):
            for d in range(W):
                if pair_pos[t, d] < 0:
                    continue
                assert 0 <= pair_pos[t, d] < rows_to[d] <= T_max
                ids = [int(lid[t, k]) for k in range(K) if dest[t, k] == d]
                recv[d][s][pair_pos[t, d]] = (t, ids, int(pair_back[t, d]))
        counts[:, s] = rows_to  # rank d's count of source s
    # compute: receiver d stores result j of row (s, i) at rank s's back[return index + j]
    back = [np.full((T_max * K, 2), -1, np.int64) for _ in range(W)]
    for d in range(W):
        for s in range(W):
            for i in range(counts[d, s]):
                t, ids, b0 = recv[d][s][i]
                for j, l in enumerate(ids):
                    assert 0 <= b0 + j < T_max * K
                    assert back[s][b0 + j, 0] == -1, "two results at one return row"
                    back[s][b0 + j] = (t, glob[d][l])
    return [back[r][plans[r][4]] for r in range(W)]


@pytest.mark.parametrize("W,El,K,T,owner_seed", [(2, 8, 4, 37, None), (4, 4, 8, 50, None), (4, 8, 8, 64, 3),
                                                 (8, 2, 16, 19, 5), (1, 16, 8, 11, None)])
def test_every_pick_finds_its_own_result(W, El, K, T, owner_seed):
    rng = np.random.default_rng(W * 100 + K)
    E = W * El
    owner = None
    if owner_seed is not None:
        owner = np.repeat(np.arange(W), El)
        np.random.default_rng(owner_seed).shuffle(owner)
    idx_by_rank = [np.stack([rng.choice(E, K, replace=False) for _ in range(T)]) for _ in range(W)]
    got = emulate(idx_by_rank, W, El, K, T, owner)
    for r in range(W):
        want_t = np.repeat(np.arange(T)[:, None], K, 1)
        assert np.array_equal(got[r][..., 0], want_t)
        assert np.array_equal(got[r][..., 1], idx_by_rank[r])


def test_send_pos_is_the_destination_grouped_plan():
    """The picks' return indices are the routing-table builder's positions with one column a destination
    (tile 1): grouped by destination rank, (token, pick) order within one, which the counts-exchange path
    uses, so both transports combine the same rows in the same order."""
    rng = np.random.default_rng(7)
    W, El, K, T = 4, 8, 8, 200
    idx = np.stack([rng.choice(W * El, K, replace=False) for _ in range(T)])
    dest, _, _, _, send_pos, _ = plan(idx, W, El)
    order = np.argsort(dest.reshape(-1), kind="stable")
    pos = np.empty(T * K, np.int64)
    pos[order] = np.arange(T * K)
    assert np.array_equal(send_pos.reshape(-1), pos)
