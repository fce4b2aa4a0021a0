"""The expert-parallel layer's host logic on CPU: world_size 2 gloo ranks run
k3moe_ep.EPMoELayer with oracle-built steps (tests/ep_oracle_ops.py) and the
two halves of the output must equal, bit for bit, the single-device layer over
all the tokens (every rank holds half the experts and its own tokens)."""
import multiprocessing as mp
import os
import socket
import tempfile

import numpy as np
import pytest

import cases


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


CFG = dict(T=96, H=256, I=256, E=8, K=2, shared=1, rs=2.5, seed=11)
# several picks of a token on one rank (4 of 8 experts a rank, top-4): one dispatched row carries them all
CFG_DENSE = dict(T=64, H=256, I=256, E=8, K=4, shared=1, rs=2.5, seed=12)


# FC2 in two 256-column slices
CFG_OVERLAP = dict(T=64, H=512, I=256, E=8, K=2, shared=1, rs=2.5, seed=13)


def _cfg(mode):
    return {"dense": CFG_DENSE, "overlap": CFG_OVERLAP}.get(mode, CFG)


def _worker(rank, world, port, outdir, mode):
    import sys

    here = os.path.dirname(os.path.abspath(__file__))
    root = os.path.dirname(here)
    sys.path[:0] = [here, os.path.join(root, "oracle"), os.path.join(root, "kern-k3-pp-prefill_b200")]
    import torch
    import torch.distributed as dist

    import cases as C
    import ep_oracle_ops
    import k3moe_ep

    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            timeout=__import__("datetime").timedelta(seconds=60))
    c = C.make_case(**_cfg(mode))
    T_l = c.T // world
    rows = slice(rank * T_l, (rank + 1) * T_l)
    t = lambda a: torch.from_numpy(np.ascontiguousarray(a))
    owner = k3moe_ep.balanced_owner(c.bias, world) if mode == "placed" else None
    w = k3moe_ep.slice_weights(t(c.w13), t(c.w13_sf), t(c.w2), t(c.w2_sf), c.E, c.shared, rank, world, c.H, c.I,
                               owner=owner)
    rs = t(np.array([c.rs_bits], np.uint16)).view(torch.bfloat16)
    layer = k3moe_ep.EPMoELayer(c.H, c.I, c.E, c.K, c.shared, w, t(c.bias), rs, ops=ep_oracle_ops.OracleOps(),
                                fixed_tokens=T_l if mode == "fixed" else None, owner=owner,
                                overlap_chunks=2 if mode == "overlap" else 1)
    out = layer.forward(t(c.S[rows]), t(c.x_bits[rows]).view(torch.bfloat16))
    np.save(os.path.join(outdir, f"out{rank}.npy"), out.view(torch.int16).numpy().view(np.uint16))
    dist.barrier()
    dist.destroy_process_group()


def _run(world, mode):
    ctx = mp.get_context("spawn")
    port = _free_port()
    with tempfile.TemporaryDirectory() as d:
        procs = [ctx.Process(target=_worker, args=(r, world, port, d, mode)) for r in range(world)]
        for p in procs:
            p.start()
        for p in procs:
            p.join(180)
            if p.is_alive():
                p.kill()
        assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
        return np.concatenate([np.load(os.path.join(d, f"out{r}.npy")) for r in range(world)])


@pytest.mark.parametrize("mode", ["counts", "placed"])
def test_ep4_gloo_matches_single_device(mode):
    """Four ranks (two experts each): the pair plan and the counts exchange over more than two ranks."""
    got = _run(4, mode)
    c = cases.make_case(**_cfg(mode))
    ref, _ = cases.oracle_forward(c)
    assert np.array_equal(got, ref)


@pytest.mark.parametrize("mode", ["counts", "dense", "fixed", "placed", "overlap"])
def test_ep2_gloo_matches_single_device(mode):
    # counts / dense: one dispatched row a (token, rank) pair, headed by the token's picks there (dense: top-4
    # of 8 experts, so most rows carry several); fixed: the fixed-block all-to-all (no counts exchange, empty
    # slots marked -1) of decode-sized batches; placed: experts dealt to the ranks by router bias
    # (balanced_owner) instead of in contiguous blocks; overlap: FC2 in two column slices, each returned by
    # its own all-to-all
    got = _run(2, mode)
    c = cases.make_case(**_cfg(mode))
    ref, _ = cases.oracle_forward(c)
    assert np.array_equal(got, ref)


def _late_worker(rank, world, port, outdir, mode):
    """Rank 1 fails on the host before its step (mode "dead": exits; "silent": stays up but never posts its
    sends); rank 0 runs the step and must come back with an error from the collective, within its timeout."""
    import sys
    import time

    here = os.path.dirname(os.path.abspath(__file__))
    root = os.path.dirname(here)
    sys.path[:0] = [here, os.path.join(root, "oracle"), os.path.join(root, "kern-k3-pp-prefill_b200")]
    import datetime

    import torch
    import torch.distributed as dist

    import cases as C
    import ep_oracle_ops
    import k3moe_ep

    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=3))
    c = C.make_case(**CFG)
    T_l = c.T // world
    rows = slice(rank * T_l, (rank + 1) * T_l)
    t = lambda a: torch.from_numpy(np.ascontiguousarray(a))
    w = k3moe_ep.slice_weights(t(c.w13), t(c.w13_sf), t(c.w2), t(c.w2_sf), c.E, c.shared, rank, world, c.H, c.I)
    rs = t(np.array([c.rs_bits], np.uint16)).view(torch.bfloat16)
    layer = k3moe_ep.EPMoELayer(c.H, c.I, c.E, c.K, c.shared, w, t(c.bias), rs, ops=ep_oracle_ops.OracleOps())
    if rank == 1:
        if mode == "silent":
            time.sleep(12)
        os._exit(0)
    t0 = time.time()
    try:
        layer.forward(t(c.S[rows]), t(c.x_bits[rows]).view(torch.bfloat16))
        msg = "no error"
    except Exception as ex:  # the collective's failure, seen on the host
        msg = f"raised {type(ex).__name__}"
    open(os.path.join(outdir, "rank0"), "w").write(f"{msg} after {time.time() - t0:.1f} s")
    os._exit(0)


@pytest.mark.parametrize("mode", ["dead", "silent"])
def test_ep_rank_that_never_sends_fails_on_the_host(mode):
    """Failure detection on the host: a rank that exits, or never posts its sends, makes the other rank's step
    end in an exception from the collective (process-group timeout 3 s), not a hang."""
    ctx = mp.get_context("spawn")
    port = _free_port()
    with tempfile.TemporaryDirectory() as d:
        procs = [ctx.Process(target=_late_worker, args=(r, 2, port, d, mode)) for r in range(2)]
        for p in procs:
            p.start()
        for p in procs:
            p.join(60)
            if p.is_alive():
                p.kill()
        assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
        got = open(os.path.join(d, "rank0")).read()
        assert got.startswith("raised"), got
        assert float(got.split(" after ")[1].split()[0]) < 30.0, got
