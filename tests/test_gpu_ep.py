"""Expert parallelism on 2 GPUs over NCCL: every rank holds half the experts
and its own tokens; the layer's output must equal, bit for bit, the single-GPU
layer (all experts on one GPU) over all the tokens.  Needs 2 GPUs.  Modes: the
counts-exchange all-to-all, the fixed-block all-to-all, the fixed-block step
captured in a CUDA graph (NCCL calls inside) and replayed, experts dealt to
the ranks by router bias instead of contiguous blocks, FC2 in column slices
returned beside the next slice, the peer-memory transport (rows and
results stored into the peers' buffers over NVLink, flags, bounded waits),
and the device-resident step (k3moe_ep_forward: fixed receive regions, no host
synchronisation) eagerly, with experts placed by bias, and captured whole in a
CUDA graph."""
import multiprocessing as mp
import os
import socket
import tempfile

import pytest
import torch

pytestmark = pytest.mark.gpu

CFG = dict(T_local=160, H=1024, I=512, E=16, K=4, shared=1, rs=2.5)


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, outdir, mode):
    import datetime
    import sys

    here = os.path.dirname(os.path.abspath(__file__))
    root = os.path.dirname(here)
    sys.path[:0] = [here, os.path.join(root, "kern-k3-pp-prefill_b200")]
    import torch
    import torch.distributed as dist

    import k3moe
    import k3moe_ep

    dev = torch.device("cuda", rank)
    torch.cuda.set_device(dev)
    dist.init_process_group("nccl", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60), device_id=dev)
    c = CFG
    H, I, E, K, sh = c["H"], c["I"], c["E"], c["K"], c["shared"]
    T = c["T_local"] * world
    w13, w13_sf = k3moe.synth_mxfp4(21, (E + sh) * 2 * I, H, 0.02, device=dev)
    w2, w2_sf = k3moe.synth_mxfp4(22, (E + sh) * H, I, 0.02, device=dev)
    # inputs made on the host, so every rank and the one-GPU reference see the same bytes
    import numpy as np

    rng = np.random.default_rng(5)
    xf = rng.standard_normal((T, H)).astype(np.float32)
    x = torch.from_numpy(xf).to(torch.bfloat16).to(dev)
    S = torch.from_numpy((x.float().cpu().numpy().astype(np.float64) @ (rng.standard_normal((H, E)) / H ** 0.5))
                         .astype(np.float32)).to(dev)
    bias = torch.from_numpy(rng.uniform(-0.1, 0.1, E).astype(np.float32)).to(dev)
    rs = torch.tensor([c["rs"]], dtype=torch.bfloat16, device=dev)
    rows = slice(rank * c["T_local"], (rank + 1) * c["T_local"])
    owner = k3moe_ep.balanced_owner(bias, world) if mode in ("placed", "device_placed") else None
    w = k3moe_ep.slice_weights(w13, w13_sf, w2, w2_sf, E, sh, rank, world, H, I, owner=owner)
    if mode.startswith("device"):
        layer = k3moe_ep.DeviceEPMoELayer(H, I, E, K, sh, w, bias, rs, max_tokens=c["T_local"], owner=owner,
                                          device=dev)
    else:
        layer = k3moe_ep.EPMoELayer(H, I, E, K, sh, w, bias, rs, device=dev,
                                    fixed_tokens=c["T_local"] if mode in ("fixed", "graph") else None, owner=owner,
                                    overlap_chunks=2 if mode == "overlap" else 1,
                                    fc2_grid_cap=100 if mode == "overlap" else 0,
                                    transport="peer" if mode == "peer" else "nccl",
                                    max_tokens=c["T_local"] if mode == "peer" else None)
    xs, Ss = x[rows].contiguous(), S[rows].contiguous()
    graph = None
    if mode in ("graph", "device_graph"):
        side = torch.cuda.Stream()
        side.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(side):
            for _ in range(2):
                layer.forward(Ss, xs)
        torch.cuda.current_stream().wait_stream(side)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            static_out = layer.forward(Ss, xs)
        outs = []
        for _ in range(2):
            graph.replay()
            outs.append(static_out.clone())
    else:
        outs = [layer.forward(Ss, xs) for _ in range(2)]  # twice: reused buffers
    full = [torch.empty_like(outs[1]) for _ in range(world)]
    dist.all_gather(full, outs[1])
    torch.cuda.synchronize()
    ok = torch.equal(outs[0].view(torch.int16), outs[1].view(torch.int16))
    if rank == 0:
        ref = k3moe.MoELayer(H, I, E, K, sh, w13, w13_sf, w2, w2_sf, bias, rs, max_tokens=T, device=dev)
        want = ref.forward(S, x)
        got = torch.cat(full)
        torch.cuda.synchronize()
        same = got.view(torch.int16) == want.view(torch.int16)
        bad_rows = (~same.all(1)).nonzero().flatten().tolist()
        diff = (got.float() - want.float()).abs().max().item()
        ok = ok and not bad_rows
        open(os.path.join(outdir, "result"), "w").write(
            "ok" if ok else f"mismatch: repeat-equal={ok} rows={bad_rows[:20]} n={len(bad_rows)} maxdiff={diff}")
    if mode == "peer" or mode.startswith("device"):
        # the waits recorded nothing, and the peers' buffers are unmapped before the group goes
        words = layer.ops.err[:2].tolist() if mode == "peer" else list(layer.error_words()[1])
        if rank == 0 and words != [0, 0]:
            open(os.path.join(outdir, "result"), "w").write(f"device error words {words}")
        dist.barrier()
        layer.close()
    if graph is not None:  # a graph holding NCCL calls is released before the process group goes
        graph.reset()
    del graph
    torch.cuda.synchronize()
    dist.barrier()
    dist.destroy_process_group()


@pytest.mark.parametrize("mode", ["counts", "fixed", "graph", "placed", "overlap", "peer", "device",
                                  "device_placed", "device_graph"])
def test_ep2_nccl_bit_identical_to_one_gpu(mode):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    ctx = mp.get_context("spawn")
    port = _free_port()
    with tempfile.TemporaryDirectory() as d:
        procs = [ctx.Process(target=_worker, args=(r, 2, port, d, mode)) for r in range(2)]
        for p in procs:
            p.start()
        for p in procs:
            p.join(300)
            if p.is_alive():
                p.kill()
        assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
        assert open(os.path.join(d, "result")).read() == "ok"
