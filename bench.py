"""Benchmark of the Kimi-K3 routed-MoE layer on B200 (config 1: an 8192-row prefill chunk on one GPU).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl k3moe|reference]

A step is one MoE layer over an 8192-row prefill chunk: router top-k ->
routing tables -> MXFP8 permute -> FC1 (MXFP8 x MXFP4, SwiGLU, MXFP8 out) ->
FC2 (bf16) -> routing-weighted combine, plus the always-on shared expert.
Shapes: T=8192 (16 packed sequences, Dirichlet lengths), H=7168, I=2048,
E=896 routed experts, top-8, routed scale 2.5, shared expert width 2048; all
expert weights MXFP4 (20.96 GB), synthetic and seeded (no checkpoint, no
dataset).  The router logits S = x.W_router are computed once before timing
(the router GEMM is the layer before this path).

`value` is device-resident throughput (tokens/s over all ranks); `e2e` is the
same layer through the public API with x and S copied from pinned host memory
and the output copied back inside every timed step.  With N > 1 the layer is
expert parallel (config 4's layout): every rank owns an 8192-row chunk and
896/N experts (+ the shared expert), tokens travel to their experts' ranks and
back by NCCL all-to-all (timed separately), weak scaling.  `--impl reference` times the
CPU restatement of the same path (oracle/, the reference's algorithm) on a
bounded sample on the host cores.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import sys
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
for _p in (os.path.join(ROOT, "kern-k3-pp-prefill_b200"), os.path.join(ROOT, "oracle"), os.path.join(ROOT, "tests")):
    if _p not in sys.path:
        sys.path.insert(0, _p)

METRIC = "MoE layer tokens/s @8192-row prefill"
T_DEF, H, I, E, K, SHARED, RS = 8192, 7168, 2048, 896, 8, 1, 2.5
W_SEED13, W_SEED2, WSD = 11, 12, 0.02
FP8_PEAK_TFLOPS = 4500.0  # dense FP8 / MXF8F6F4 nominal (no measured figure for this kind exists here)


def peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            m = json.load(f)
        return float(m["hbm_gbs"]), "measured"
    except Exception:
        return 6650.0, "fallback"


def cu_seqlens(T, n=16, seed=0):
    rng = np.random.default_rng(seed)
    w = rng.dirichlet(np.ones(n))
    lens = np.maximum(1, np.floor(w * T).astype(np.int64))
    lens[-1] = T - lens[:-1].sum()
    return np.concatenate([[0], np.cumsum(lens)]).astype(np.int32)


def prefill_config(T, E, zipf):
    """The `config` of the 1-GPU prefill line, the same for the GPU arm and the reference arm."""
    return {"workload": ("K3-shape prefill MoE layer, Zipf(1.1) expert popularity (config 3)" if zipf else
                         "K3-shape prefill MoE layer (config 1)"), "zipf": zipf,
            "T": T, "H": H, "I": I, "E": E, "K": K, "shared_expert_width": I, "rs": RS, "global_batch": T,
            "seq_len": T, "sequences": 16, "cu_seqlens": cu_seqlens(T).tolist(), "parallelism": "ep1",
            "l2": "inputs larger than L2: 20.96 GB of expert weights streamed every step"}


def layer_flops(T):
    return 6.0 * H * I * (T * K + SHARED * T)


# ------------------------------------------------------------------ clocks
class ClockSampler:
    """NVML samples of SM clock and throttle reasons while the timed region runs."""

    REASONS = {0x8: "hw_slowdown", 0x40: "hw_thermal_slowdown", 0x20: "sw_thermal_slowdown", 0x4: "sw_power_cap",
               0x80: "hw_power_brake_slowdown"}

    def __init__(self, uuid):
        self.samples, self.reasons, self.ok = [], set(), False
        try:
            import pynvml

            pynvml.nvmlInit()
            self.nv = pynvml
            self.h = pynvml.nvmlDeviceGetHandleByUUID(uuid)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self.h, pynvml.NVML_CLOCK_SM)
            self.ok = True
        except Exception as ex:  # no NVML: the line says so
            self.err = str(ex)
        self._stop = threading.Event()

    def _run(self):
        while not self._stop.is_set():
            try:
                self.samples.append(self.nv.nvmlDeviceGetClockInfo(self.h, self.nv.NVML_CLOCK_SM))
                get = getattr(self.nv, "nvmlDeviceGetCurrentClocksEventReasons", None) or \
                    self.nv.nvmlDeviceGetCurrentClocksThrottleReasons
                r = get(self.h)
                for bit, name in self.REASONS.items():
                    if r & bit:
                        self.reasons.add(name)
            except Exception:
                pass
            time.sleep(0.01)

    def __enter__(self):
        if self.ok:
            self.t = threading.Thread(target=self._run, daemon=True)
            self.t.start()
        return self

    def __exit__(self, *a):
        if self.ok:
            self._stop.set()
            self.t.join()

    def summary(self):
        if not self.ok:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "note": f"NVML unavailable: {self.err}"}
        return {"sm_mhz": statistics.median(self.samples) if self.samples else None, "sm_max_mhz": self.max_mhz,
                "reasons": sorted(self.reasons), "samples": len(self.samples)}


# ------------------------------------------------------------------ CPU baseline (oracle port)
def cpu_sample(sample_tiles, tb, wsrc, qsrc, threads=0):
    """Time the oracle's FC1 + FC2 over `sample_tiles` token tiles (compact copies).

    tb: host tables (cta_batch, cta_limit); wsrc(e) -> (w13, w13_sf, w2, w2_sf) of expert e;
    qsrc(c) -> (q rows [128, H], tiled sf of the tile).  Returns seconds."""
    import oracle

    oracle.set_threads(threads)
    ns = len(sample_tiles)
    kg4 = H // 128
    qp = np.zeros((ns * 128, H), np.uint8)
    sfp = np.zeros(ns * kg4 * 512, np.uint8)
    w13 = np.zeros((ns * 2 * I, H // 2), np.uint8)
    w13sf = np.zeros(ns * 2 * I // 128 * kg4 * 512, np.uint8)
    w2 = np.zeros((ns * H, I // 2), np.uint8)
    w2sf = np.zeros(ns * H // 128 * (I // 128) * 512, np.uint8)
    cb = np.arange(ns, dtype=np.int32)
    cl = np.zeros(ns, np.int32)
    for i, c in enumerate(sample_tiles):
        e = int(tb["cta_batch"][c])
        n = int(tb["cta_limit"][c]) - c * 128
        cl[i] = i * 128 + n
        q, sf = qsrc(c)
        qp[i * 128:(i + 1) * 128] = q
        sfp[i * kg4 * 512:(i + 1) * kg4 * 512] = sf
        a, asf, b, bsf = wsrc(e)
        w13[i * 2 * I:(i + 1) * 2 * I] = a
        w13sf[i * len(asf):(i + 1) * len(asf)] = asf
        w2[i * H:(i + 1) * H] = b
        w2sf[i * len(bsf):(i + 1) * len(bsf)] = bsf
    t0 = time.perf_counter()
    f1q, f1sf = oracle.fc1(w13, w13sf, qp, sfp, cb, cl, 0, ns, H, I)
    oracle.fc2(w2, w2sf, f1q, f1sf, cb, cl, 0, ns, H, I)
    return time.perf_counter() - t0


def cpu_topk_time(S, bias, rs_bits):
    import oracle

    t0 = time.perf_counter()
    oracle.topk(S, bias, rs_bits, K)
    return time.perf_counter() - t0


def sample_tiles_of(nne, n=16):
    return sorted(set(np.linspace(0, nne - 1, n).astype(int).tolist()))


# ------------------------------------------------------------------ the reference arm (CPU)
def run_reference(args):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    import oracle

    threads = oracle.set_threads(0)
    T = args.tokens
    rng = np.random.default_rng(0)
    x_bits = oracle.bf16_bits(rng.standard_normal((T, H), dtype=np.float32))
    wr = (rng.standard_normal((H, E), dtype=np.float32) / np.sqrt(H)).astype(np.float32)
    S = (oracle.bf16_to_f32(x_bits) @ wr).astype(np.float32)
    bias = rng.uniform(-0.1, 0.1, E).astype(np.float32)
    rs_bits = int(oracle.bf16_bits(np.array([RS], np.float32))[0])
    idx, wts = oracle.topk(S, bias, rs_bits, K)
    tb = oracle.tables(idx, E, 0, SHARED)
    nne = int(tb["meta"][0])
    tiles = sample_tiles_of(nne, args.cpu_tiles)
    wcache = {}

    def wsrc(e):
        if e not in wcache:
            a = oracle.synth_f32(W_SEED13, 2 * I, H, WSD, row0=e * 2 * I)
            b = oracle.synth_f32(W_SEED2, H, I, WSD, row0=e * H)
            wcache[e] = oracle.quant_mxfp4(a) + oracle.quant_mxfp4(b)
        return wcache[e]

    def qsrc(c):
        rows = tb["route_map"][c * 128:(c + 1) * 128]
        q, sf = oracle.quant_mxfp8(x_bits[rows], tiled=True)
        return q, sf

    for e in {int(tb["cta_batch"][c]) for c in tiles}:
        wsrc(e)
    times = []
    for step in range(args.warmup + args.steps):
        t = cpu_topk_time(S, bias, rs_bits) + cpu_sample(tiles, tb, wsrc, qsrc, threads) * nne / len(tiles)
        if step >= args.warmup:
            times.append(t)
    sec = statistics.mean(times)
    value = T / sec
    sample = (f"router top-k over all {T} rows + oracle FC1+FC2 over {len(tiles)} of {nne} token tiles (spread "
              f"evenly), scaled by {nne}/{len(tiles)}")
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": sec * 1e3, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "mxfp8 x mxfp4 (f32 accumulate)", "data": "synthetic",
        "config": prefill_config(T, E, None),
        "cpu_baseline": {"value": value, "unit": "tokens/s", "cores": threads, "kind": "port", "sample": sample},
        "e2e": {"value": value, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def e2e_overlapped(fwd, S_h, x_h, out_shape, steps, stream, dev):
    """ms a step of the layer end to end: every step copies its inputs (S, x) from pinned host memory to the
    device and its whole output back to pinned host memory.  The copies run on two side streams with double
    buffers, so step i's input copy and step i-1's output copy overlap step i's compute, as a serving loop
    would run them; every byte of every step still crosses PCIe inside the timed region.
    fwd(S_dev, x_dev, out_dev) -> the output tensor."""
    import torch

    cin, cout = torch.cuda.Stream(device=dev), torch.cuda.Stream(device=dev)
    xd = [torch.empty(x_h.shape, dtype=x_h.dtype, device=dev) for _ in range(2)]
    Sd = [torch.empty(S_h.shape, dtype=S_h.dtype, device=dev) for _ in range(2)]
    od = [torch.empty(out_shape, dtype=torch.bfloat16, device=dev) for _ in range(2)]
    out_h = [torch.empty(out_shape, dtype=torch.bfloat16).pin_memory() for _ in range(2)]
    ev_in, ev_comp, ev_out = ([torch.cuda.Event() for _ in range(2)] for _ in range(3))
    keep = []

    def loop(n):
        for i in range(n):
            b = i & 1
            if i >= 2:
                cin.wait_event(ev_comp[b])  # step i-2 has consumed these input buffers
            with torch.cuda.stream(cin):
                xd[b].copy_(x_h, non_blocking=True)
                Sd[b].copy_(S_h, non_blocking=True)
                ev_in[b].record(cin)
            stream.wait_event(ev_in[b])
            if i >= 2:
                stream.wait_event(ev_out[b])  # step i-2's output has reached the host
            o = fwd(Sd[b], xd[b], od[b])
            ev_comp[b].record(stream)
            cout.wait_event(ev_comp[b])
            with torch.cuda.stream(cout):
                out_h[b].copy_(o, non_blocking=True)
                ev_out[b].record(cout)
            if o is not od[b]:  # an output the layer allocated: alive until its copy has run
                o.record_stream(cout)
                keep.append(o)

    loop(2)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    cin.wait_event(e0)
    loop(steps)
    stream.wait_stream(cout)
    e1.record(stream)
    torch.cuda.synchronize()
    keep.clear()
    return e0.elapsed_time(e1) / steps


def rank_weights(E, experts, dev):
    """The listed routed experts (in order) then the shared expert, from the same synthetic stream as the full
    set (every expert's rows are synthesised from their global row index)."""
    import torch

    import k3moe

    El = len(experts)
    w = {}
    for name, rows_per, K_, seed in (("w13", 2 * I, H, W_SEED13), ("w2", H, I, W_SEED2)):
        packed = torch.empty(((El + SHARED) * rows_per, K_ // 2), dtype=torch.uint8, device=dev)
        sf = torch.zeros((El + SHARED) * rows_per // 128 * (K_ // 128) * 512, dtype=torch.uint8, device=dev)
        per_sf = rows_per // 128 * (K_ // 128) * 512
        # runs of consecutive experts in one synthesis call each
        runs, i = [], 0
        while i < El:
            j = i + 1
            while j < El and experts[j] == experts[j - 1] + 1:
                j += 1
            runs.append((i, experts[i], j - i))
            i = j
        for at, e0, n in runs + ([(El, E, 1)] if SHARED else []):
            k3moe.synth_mxfp4(seed, n * rows_per, K_, WSD, row0=e0 * rows_per,
                              packed=packed[at * rows_per:(at + n) * rows_per], sf=sf[at * per_sf:(at + n) * per_sf])
        w[name], w[name + "_sf"] = packed, sf
    return w


def rank_experts(E, world, rank, bias, placement):
    """(owner [E] or None, this rank's experts in id order) for the placement policy."""
    import k3moe_ep

    if placement == "contiguous":
        El = E // world
        return None, list(range(rank * El, (rank + 1) * El))
    owner = k3moe_ep.balanced_owner(bias, world)
    return owner, (owner == rank).nonzero().flatten().tolist()


def rank_inputs(T, E, rank, dev):
    """bf16 x [T, H] ~ N(0, 1) of this rank, router logits S = x.W_router (W_router ~ N(0, 1/H), the same on
    every rank), bias ~ U(-0.1, 0.1), rs."""
    import torch

    g = torch.Generator(device=dev)
    g.manual_seed(1000 + rank)
    x = torch.randn((T, H), generator=g, device=dev, dtype=torch.float32).to(torch.bfloat16)
    g.manual_seed(7)
    wr = torch.randn((H, E), generator=g, device=dev, dtype=torch.float32) / H ** 0.5
    S = (x.float() @ wr).contiguous()
    bias = (torch.rand(E, generator=g, device=dev) * 0.2 - 0.1).float()
    rs = torch.tensor([RS], dtype=torch.bfloat16, device=dev)
    return x, S, bias, rs


# ------------------------------------------------------------------ the GPU arm, N > 1: expert parallel
def run_ep(args, world, rank, dev):
    """Config 4's layout at N GPUs: every rank owns an 8192-row chunk (16 packed sequences) and E/N experts
    (+ the shared expert); dispatch and combine are NCCL all-to-all; weak scaling (N x 8192 rows a step)."""
    import torch
    import torch.distributed as dist

    import k3moe
    import k3moe_ep

    E, T = args.experts, args.tokens
    El = E // world
    x, S, bias, rs = rank_inputs(T, E, rank, dev)
    owner, mine = rank_experts(E, world, rank, bias, args.ep_placement)
    w = rank_weights(E, mine, dev)
    layer = k3moe_ep.EPMoELayer(H, I, E, K, SHARED, w, bias, rs, device=dev, owner=owner,
                                overlap_chunks=args.ep_overlap, fc2_grid_cap=args.ep_fc2_cap)
    for _ in range(args.warmup):
        layer.forward(S, x)
    torch.cuda.synchronize()
    names = ("dispatch", "fc1", "combine")
    evs = [{n: (torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for n in names}
           for _ in range(args.steps)]
    start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    dist.barrier()
    torch.cuda.synchronize()
    uuid = "GPU-" + str(torch.cuda.get_device_properties(dev).uuid)
    with ClockSampler(uuid) as clk:
        start.record()
        for s in range(args.steps):
            layer.forward(S, x, evs[s])
        stop.record()
        torch.cuda.synchronize()
    dist.barrier()
    ms = start.elapsed_time(stop) / args.steps
    part = {n: float(np.mean([e[n][0].elapsed_time(e[n][1]) for e in evs])) for n in names}
    t = torch.tensor([ms, part["dispatch"], part["combine"], part["fc1"]], device=dev)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms, disp_ms, comb_ms, fc1_ms = [float(v) for v in t.tolist()]
    # e2e: x and S from pinned host memory in, the output back, every step (copies overlapped)
    x_h, S_h = x.cpu().pin_memory(), S.cpu().pin_memory()
    dist.barrier()
    n_e2e = args.e2e_steps or args.steps
    e2e_ms = e2e_overlapped(lambda Sd, xd, od: layer.forward(Sd, xd), S_h, x_h, (T, H), n_e2e,
                            torch.cuda.current_stream(), dev)
    t = torch.tensor([e2e_ms], device=dev)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    e2e_ms = float(t.item())
    tb = layer.last["tables"]
    counts = tb.counts.cpu().numpy()
    routed_rows, touched = int(counts.sum()), int((counts > 0).sum())
    fc1_bytes = touched * (2 * I * H // 2 + 2 * I * H // 32) + routed_rows * (H + H // 32 + I + I // 32)
    hbm_peak, peak_kind = peaks()
    if rank == 0:
        flops = layer_flops(T) * world
        achieved = fc1_bytes / (fc1_ms / 1e3) / 1e9
        line = {
            "metric": METRIC, "value": T * world / (ms / 1e3), "unit": "tokens/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "mxfp8 x mxfp4 (f32 accumulate)", "data": "synthetic",
            "config": {"workload": f"K3-shape prefill MoE layer, expert parallel over {world} GPUs (config 4 layout)",
                       "T_per_gpu": T, "H": H, "I": I, "E": E, "E_per_gpu": El, "K": K, "shared_expert_width": I,
                       "rs": RS, "global_batch": T * world, "seq_len": T, "parallelism": f"ep{world}",
                       "expert_placement": args.ep_placement, "fc2_slices": args.ep_overlap,
                       "fc2_grid_cap": args.ep_fc2_cap,
                       "l2": "inputs larger than L2: each GPU streams its experts' weights every step"},
            "tflops": flops / (ms / 1e3) / 1e12,
            "a2a_ms": {"dispatch": disp_ms, "combine": comb_ms},
            "roofline": {"kernel": "FC1 grouped GEMM (grouped_gemm_kernel<0>), rank 0", "bound": "hbm",
                         "achieved": achieved, "peak": hbm_peak, "unit": "GB/s", "frac": achieved / hbm_peak,
                         "peak_kind": peak_kind, "algorithmic_bytes_per_launch": fc1_bytes, "traffic": None},
            "e2e": {"value": T * world / (e2e_ms / 1e3), "unit": "tokens/s", "ms_per_step": e2e_ms,
                    "h2d_bytes_per_step": int(x.numel() * 2 + S.numel() * 4) * world,
                    "d2h_bytes_per_step": int(x.numel() * 2) * world,
                    "copies": "every step's x, S in and output back over PCIe, on side streams overlapping the "
                              "neighbouring steps' compute (double buffers)"},
            # topk, 2 x 3 plan launches, pairs, pack, shared pack, ids, 3 table launches, unpack, return rows,
            # FC1, FC2 (a launch a slice), combine
            "gpu_launches": (18 + args.ep_overlap) * args.steps,
            "clocks": clk.summary(),
            "cpu_baseline": None,
        }
        print(json.dumps(line), flush=True)
    dist.barrier()
    dist.destroy_process_group()


# ------------------------------------------------------------------ decode (config 2): --decode
DECODE_METRIC = "EP decode us/layer (64 tokens x top-8)"


def run_decode(args, world, rank, dev):
    """Config 2: one MoE decode step of 64 tokens x top-8 over E = 896 experts, expert parallel over the N GPUs
    (E/N contiguous experts each, 64/N tokens each); the figure is microseconds a layer, max over ranks."""
    import torch
    import torch.distributed as dist

    import k3moe
    import k3moe_ep

    E, Tall = args.experts, args.decode_tokens
    if Tall % world or E % world:
        raise SystemExit(f"--decode needs tokens ({Tall}) and experts ({E}) divisible by {world}")
    T, El = Tall // world, E // world
    # the same 64 tokens whatever N: rank r owns rows [r T, r T + T) of one global batch
    x_all, S_all, bias, rs = rank_inputs(Tall, E, 0, dev)
    x, S = x_all[rank * T:(rank + 1) * T].contiguous(), S_all[rank * T:(rank + 1) * T].contiguous()
    if world == 1:
        w13, w13_sf = k3moe.synth_mxfp4(W_SEED13, (E + SHARED) * 2 * I, H, WSD, device=dev)
        w2, w2_sf = k3moe.synth_mxfp4(W_SEED2, (E + SHARED) * H, I, WSD, device=dev)
        layer = k3moe.MoELayer(H, I, E, K, SHARED, w13, w13_sf, w2, w2_sf, bias, rs, max_tokens=T, device=dev)
        out = torch.empty((T, H), dtype=torch.bfloat16, device=dev)
        run = lambda: layer.forward(S, x, out)  # noqa: E731
    else:
        # fixed-size all-to-all blocks: no host synchronisation in the step, so it can be graph-captured
        owner, mine = rank_experts(E, world, rank, bias, args.ep_placement)
        w = rank_weights(E, mine, dev)
        layer = k3moe_ep.EPMoELayer(H, I, E, K, SHARED, w, bias, rs, device=dev, fixed_tokens=T, owner=owner)
        run = lambda: layer.forward(S, x)  # noqa: E731
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        for _ in range(args.warmup):
            run()
    torch.cuda.current_stream().wait_stream(side)
    torch.cuda.synchronize()

    def max_over_ranks(v):
        if world == 1:
            return v
        t = torch.tensor([v], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    def timed(step):
        start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()
        start.record()
        for _ in range(args.steps):
            step()
        stop.record()
        torch.cuda.synchronize()
        return max_over_ranks(start.elapsed_time(stop) / args.steps * 1e3)

    eager_us = timed(run)
    # the whole step (its NCCL calls included) as one CUDA graph, replayed
    graph, graph_note = None, None
    try:
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            static_out = run()
        graph.replay()
        torch.cuda.synchronize()
    except Exception as ex:  # capture unsupported here: the eager step is the figure
        graph, graph_note = None, f"graph capture failed: {type(ex).__name__}: {str(ex)[:120]}"
    ok = torch.tensor([1.0 if graph is not None else 0.0], device=dev)
    if world > 1:
        dist.all_reduce(ok, op=dist.ReduceOp.MIN)
    if ok.item() < 1.0:
        graph = None
    step = graph.replay if graph is not None else run
    uuid = "GPU-" + str(torch.cuda.get_device_properties(dev).uuid)
    with ClockSampler(uuid) as clk:
        us = timed(step)
    # end to end: this rank's x and S from pinned host memory into the step's inputs, its output back
    x_h, S_h = x.cpu().pin_memory(), S.cpu().pin_memory()
    out_h = torch.empty((T, H), dtype=torch.bfloat16).pin_memory()
    if world > 1:
        dist.barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    n_e2e = args.e2e_steps or args.steps
    e0.record()
    for _ in range(n_e2e):
        x.copy_(x_h, non_blocking=True)
        S.copy_(S_h, non_blocking=True)
        if graph is not None:
            graph.replay()
            o = static_out
        else:
            o = run()
        out_h.copy_(o, non_blocking=True)
    e1.record()
    torch.cuda.synchronize()
    e2e_us = max_over_ranks(e0.elapsed_time(e1) / n_e2e * 1e3)
    # bytes a layer must stream on the slowest rank: its touched experts' weights (+ the shared expert's)
    if world == 1:
        off = layer.offsets(T)
        counts = layer.ws[off["counts"]:off["counts"] + 4 * (E + SHARED)].view(torch.int32).cpu().numpy()
    else:
        counts = layer.last["tables"].counts.cpu().numpy()
    touched = int((counts > 0).sum())
    per_expert = 2 * I * H // 2 + 2 * I * H // 32 + H * I // 2 + H * I // 32
    wbytes = max_over_ranks(float(touched * per_expert))
    hbm_peak, peak_kind = peaks()
    achieved = wbytes / (us / 1e6) / 1e9
    if rank == 0:
        line = {
            "metric": DECODE_METRIC, "value": us, "unit": "us/layer", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": us / 1e3, "higher_is_better": False, "scaling": "strong",
            "vs_baseline": None, "dtype": "mxfp8 x mxfp4 (f32 accumulate)", "data": "synthetic",
            "config": {"workload": "K3-shape decode MoE step (config 2)", "tokens": Tall, "tokens_per_gpu": T,
                       "H": H, "I": I, "E": E, "E_per_gpu": El, "K": K, "shared_expert_width": I, "rs": RS,
                       "parallelism": f"ep{world}", "expert_placement": args.ep_placement if world > 1 else None,
                       "l2": "inputs larger than L2: each step streams the touched experts' weights"},
            "roofline": {"kernel": "whole decode layer (weights of the touched experts, slowest rank)",
                         "bound": "hbm", "achieved": achieved, "peak": hbm_peak, "unit": "GB/s",
                         "frac": achieved / hbm_peak, "peak_kind": peak_kind, "algorithmic_bytes_per_launch": wbytes,
                         "traffic": None},
            "routing": {"touched_experts_max_rank": int(wbytes // per_expert)},
            "e2e": {"value": e2e_us, "unit": "us/layer", "h2d_bytes_per_step": int(x.numel() * 2 + S.numel() * 4),
                    "d2h_bytes_per_step": int(x.numel() * 2)},
            "gpu_launches": (8 if world == 1 else 14) * args.steps,
            "cuda_graph": graph is not None, "eager_us": eager_us,
            "clocks": clk.summary(),
            "cpu_baseline": None,
        }
        if graph_note:
            line["note"] = graph_note
        print(json.dumps(line), flush=True)
    # a graph holding NCCL calls is released before the process group goes (step holds a reference too)
    step = None
    if graph is not None:
        graph.reset()
    del graph
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


# ------------------------------------------------------------------ the GPU arm
def run_native(args, dev):
    """The layer at the reference's own shapes (K3: latent 3584, I 3072, top-16, SiTU gate, 896 experts, the
    shared expert outside the MoE kernels as in the reference's P step), 8192 rows on one GPU: the workload of
    the reference's published P MoE layer time (route + FC1 + FC2 + finalize, roofline/prefill.md:101, measured
    on GB300).  One JSON line; ms a layer, lower is better."""
    import torch

    import k3moe

    Hn, In, En, Kn, T = 3584, 3072, 896, 16, args.tokens
    k3moe.lib()
    w13, w13_sf = k3moe.synth_mxfp4(W_SEED13, En * 2 * In, Hn, WSD, device=dev)
    w2, w2_sf = k3moe.synth_mxfp4(W_SEED2, En * Hn, In, WSD, device=dev)
    g = torch.Generator(device=dev)
    g.manual_seed(1000)
    x = torch.randn((T, Hn), generator=g, device=dev, dtype=torch.float32).to(torch.bfloat16)
    g.manual_seed(7)
    wr = torch.randn((Hn, En), generator=g, device=dev, dtype=torch.float32) / Hn ** 0.5
    S = (x.float() @ wr).contiguous()
    bias = (torch.rand(En, generator=g, device=dev) * 0.2 - 0.1).float()
    rs = torch.tensor([RS], dtype=torch.bfloat16, device=dev)
    del wr
    layer = k3moe.MoELayer(Hn, In, En, Kn, 0, w13, w13_sf, w2, w2_sf, bias, rs, max_tokens=T, device=dev,
                           activation=k3moe.ACT_SITU)
    out = torch.empty((T, Hn), dtype=torch.bfloat16, device=dev)
    for _ in range(args.warmup):
        layer.forward(S, x, out)
    torch.cuda.synchronize()
    layer.check_device_error(T)
    stream = torch.cuda.current_stream()
    ev = [[torch.cuda.Event(enable_timing=True) for _ in range(7)] for _ in range(args.steps)]
    for row in ev:
        for e in row:
            e.record(stream)
    start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    uuid = "GPU-" + str(torch.cuda.get_device_properties(dev).uuid)
    torch.cuda.synchronize()
    with ClockSampler(uuid) as clk:
        start.record(stream)
        for s in range(args.steps):
            layer.forward_events(S, x, out, ev[s])
        stop.record(stream)
        torch.cuda.synchronize()
    layer.check_device_error(T)
    ms = start.elapsed_time(stop) / args.steps
    stage_ms = np.array([[ev[s][i].elapsed_time(ev[s][i + 1]) for i in range(6)] for s in range(args.steps)]).mean(0)
    flops = 2.0 * T * Kn * (Hn * 2 * In + In * Hn)
    line = {"metric": "MoE layer ms @8192-row prefill, K3 native shape", "value": ms, "unit": "ms/layer",
            "n_gpus": 1, "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": False,
            "tokens_per_s": T / (ms / 1e3), "tflops": flops / (ms / 1e3) / 1e12, "dtype": "mxfp8 x mxfp4 (f32 accumulate)",
            "data": "synthetic", "stage_ms": dict(zip(["topk", "tables", "permute", "fc1", "fc2", "combine"],
                                                      [round(float(v), 4) for v in stage_ms])),
            "config": {"workload": "K3 native-shape prefill MoE layer (latent 3584, I 3072, top-16, SiTU, no shared)",
                       "T": T, "H": Hn, "I": In, "E": En, "K": Kn, "shared_expert_width": 0, "rs": RS,
                       "parallelism": "ep1", "l2": "inputs larger than L2: 15.7 GB of expert weights"},
            "reference_published": {"value": 4.76, "unit": "ms/layer", "hardware": "GB300 (sm_103a, 1400 W)",
                                    "source": "roofline/prefill.md:101 (52.37 ms per 11 layers)"},
            "clocks": clk.summary()}
    print(json.dumps(line), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="k3moe", choices=["k3moe", "reference"])
    ap.add_argument("--tokens", type=int, default=T_DEF)
    ap.add_argument("--experts", type=int, default=896, help="routed experts (smaller only for profiling captures)")
    ap.add_argument("--e2e-steps", type=int, default=0, help="e2e steps (default: --steps)")
    ap.add_argument("--cpu-tiles", type=int, default=8)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--decode", action="store_true", help="config 2: one 64-token decode step, us/layer")
    ap.add_argument("--decode-tokens", type=int, default=64)
    ap.add_argument("--ep-placement", default="balanced", choices=["balanced", "contiguous"],
                    help="N > 1: experts dealt to ranks by router bias (balanced) or in contiguous blocks")
    ap.add_argument("--zipf", action="store_true",
                    help="config 3: the routing bias makes expert popularity Zipf(1.1) (N = 1 prefill)")
    ap.add_argument("--ep-overlap", type=int, default=1,
                    help="N > 1: FC2 in this many column slices, each returned by its own all-to-all beside the next")
    ap.add_argument("--ep-fc2-cap", type=int, default=0,
                    help="N > 1 with --ep-overlap > 1: FC2's persistent blocks (0: one an SM), SMs left to NCCL")
    ap.add_argument("--native", action="store_true",
                    help="the layer at the reference's own K3 shapes (latent 3584, I 3072, top-16, SiTU), N = 1")
    args = ap.parse_args()
    if args.impl == "reference":
        return run_reference(args)

    import torch
    import torch.distributed as dist

    import k3moe

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        import datetime

        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300), device_id=dev)
        return run_decode(args, world, rank, dev) if args.decode else run_ep(args, world, rank, dev)
    if args.decode:
        return run_decode(args, world, rank, dev)
    if args.native:
        return run_native(args, dev)
    E = args.experts  # noqa: N806  (the routed experts of this run; smaller only for profiling captures)
    T = args.tokens
    k3moe.lib()

    # weights: [gate; up] rows of every routed expert then the shared expert (expert E)
    ne = E + SHARED
    w13, w13_sf = k3moe.synth_mxfp4(W_SEED13, ne * 2 * I, H, WSD, device=dev)
    w2, w2_sf = k3moe.synth_mxfp4(W_SEED2, ne * H, I, WSD, device=dev)
    g = torch.Generator(device=dev)
    g.manual_seed(1000 + rank)
    x = torch.randn((T, H), generator=g, device=dev, dtype=torch.float32).to(torch.bfloat16)
    g.manual_seed(7)
    wr = torch.randn((H, E), generator=g, device=dev, dtype=torch.float32) / H ** 0.5
    S = (x.float() @ wr).contiguous()
    bias = (torch.rand(E, generator=g, device=dev) * 0.2 - 0.1).float()
    rs = torch.tensor([RS], dtype=torch.bfloat16, device=dev)
    del wr
    zipf = None
    if args.zipf:  # config 3: bias fitted (on the host) so the realised top-8 histogram follows Zipf(1.1)
        import cases

        zb, beta, kl = cases.zipf_bias(S.cpu().numpy(), K)
        bias = torch.from_numpy(zb).to(dev)
        zipf = {"s": 1.1, "seed": 3, "beta": beta, "kl": round(kl, 4)}
    layer = k3moe.MoELayer(H, I, E, K, SHARED, w13, w13_sf, w2, w2_sf, bias, rs, max_tokens=T, device=dev)
    out = torch.empty((T, H), dtype=torch.bfloat16, device=dev)

    for _ in range(args.warmup):
        layer.forward(S, x, out)
    torch.cuda.synchronize()
    layer.check_device_error(T)

    # ---------------- device-resident timing, per-stage events on the launching stream
    stream = torch.cuda.current_stream()
    ev = [[torch.cuda.Event(enable_timing=True) for _ in range(7)] for _ in range(args.steps)]
    for row in ev:
        for e in row:
            e.record(stream)
    start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    uuid = "GPU-" + str(torch.cuda.get_device_properties(dev).uuid)
    with ClockSampler(uuid) as clk:
        start.record(stream)
        for s in range(args.steps):
            layer.forward_events(S, x, out, ev[s])
        stop.record(stream)
        torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    layer.check_device_error(T)
    ms = start.elapsed_time(stop) / args.steps
    # GEMM role counters over 2 extra (untimed) steps: where each role of FC1 / FC2 spends its cycles
    trace = torch.zeros(32, dtype=torch.int64, device=dev)
    k3moe.set_trace(trace)
    for _ in range(2):
        layer.forward(S, x, out)
    torch.cuda.synchronize()
    k3moe.set_trace(None)
    tr = trace.cpu().tolist()
    gemm_trace = {}
    stage_ms = np.array([[ev[s][i].elapsed_time(ev[s][i + 1]) for i in range(6)] for s in range(args.steps)]).mean(0)
    for mode, name in ((0, "fc1"), (1, "fc2")):
        c = dict(zip(k3moe.TRACE_FIELDS, tr[16 * mode:16 * mode + 8]))
        # the MMA role's clock64 cycles a block over the kernel's event time: the SM clock the GEMM ran at
        # (NVML's samples miss the power-capped dips inside the GEMMs)
        blocks = min(torch.cuda.get_device_properties(dev).multi_processor_count, max(int(c["units"]), 1))
        sm_mhz = c["mma"] / 2 / blocks / (float(stage_ms[3 + mode]) * 1e3)
        gemm_trace[name] = {
            "sm_mhz_in_kernel": round(sm_mhz),
            "mma_busy": round(1 - (c["mma_wait_loaded"] + c["mma_wait_drained"]) / max(c["mma"], 1), 3),
            "mma_wait_loaded": round(c["mma_wait_loaded"] / max(c["mma"], 1), 3),
            "mma_wait_drained": round(c["mma_wait_drained"] / max(c["mma"], 1), 3),
            "producer_wait_stage": round(c["producer_wait_stage"] / max(c["producer"], 1), 3),
            "epilogue_busy": round(1 - c["epilogue_wait_acc"] / max(c["epilogue"], 1), 3),
        }
    if world > 1:
        t = torch.tensor([ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    value = T * world / (ms / 1e3)

    # ---------------- tables of the run: algorithmic bytes of FC1 (the dominant kernel)
    off = layer.offsets(T)
    ws = layer.ws
    meta = ws[off["meta"]:off["meta"] + 16].view(torch.int32).cpu().numpy()
    nne = int(meta[0])
    counts = ws[off["counts"]:off["counts"] + 4 * (E + SHARED)].view(torch.int32).cpu().numpy()
    routed_rows = int(counts.sum())
    touched = int((counts > 0).sum())
    w13_bytes_expert = 2 * I * H // 2 + 2 * I * H // 32
    fc1_bytes = touched * w13_bytes_expert + routed_rows * (H + H // 32) + routed_rows * (I + I // 32)
    fc1_ms = float(stage_ms[3])
    hbm_peak, peak_kind = peaks()
    achieved = fc1_bytes / (fc1_ms / 1e3) / 1e9
    # DRAM bytes (read + write) of one FC1 launch of this workload, from the ncu capture summarised in
    # profiles/grouped_gemm_fc1_config1_traffic.md (line "bytes_per_launch: N")
    traffic = None
    tf = os.path.join(ROOT, "profiles", "grouped_gemm_fc1_config1_traffic.md")
    if os.path.exists(tf) and T == T_DEF and E == 896 and not args.zipf:
        for ln in open(tf):
            if ln.startswith("bytes_per_launch:"):
                traffic = int(ln.split(":")[1].strip())

    # ---------------- end to end through the public API: host x/S in, host out back
    e2e_steps = args.e2e_steps or args.steps
    x_h = x.cpu().pin_memory()
    S_h = S.cpu().pin_memory()

    def fwd(Sd, xd, od):
        layer.forward(Sd, xd, od)
        return od

    e2e_ms = e2e_overlapped(fwd, S_h, x_h, (T, H), e2e_steps, stream, dev)
    if world > 1:
        t = torch.tensor([e2e_ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        e2e_ms = float(t.item())
    layer.check_device_error(T)

    # ---------------- CPU baseline (rank 0, N = 1): the oracle on a bounded sample
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        import oracle

        threads = oracle.set_threads(0)
        cb = ws[off["cta_batch"]:off["cta_batch"] + 4 * nne].view(torch.int32).cpu().numpy()
        cl = ws[off["cta_limit"]:off["cta_limit"] + 4 * nne].view(torch.int32).cpu().numpy()
        tb = {"cta_batch": cb, "cta_limit": cl}
        tiles = sample_tiles_of(nne, args.cpu_tiles)
        kg4 = H // 128
        a13 = 2 * I * (H // 2)
        s13 = 2 * I // 128 * kg4 * 512
        a2 = H * (I // 2)
        s2 = H // 128 * (I // 128) * 512

        def wsrc(e):
            return (w13[e * 2 * I:(e + 1) * 2 * I].cpu().numpy(), w13_sf[e * s13:(e + 1) * s13].cpu().numpy(),
                    w2[e * H:(e + 1) * H].cpu().numpy(), w2_sf[e * s2:(e + 1) * s2].cpu().numpy())

        qp = ws[off["q_perm"]:]
        sfp = ws[off["sf_perm"]:]

        def qsrc(c):
            q = qp[c * 128 * H:(c + 1) * 128 * H].view(128, H).cpu().numpy()
            sf = sfp[c * kg4 * 512:(c + 1) * kg4 * 512].cpu().numpy()
            return q, sf

        rs_bits = int(rs.view(torch.int16).item()) & 0xFFFF
        t_topk = cpu_topk_time(S.cpu().numpy(), bias.cpu().numpy(), rs_bits)
        t_fc = cpu_sample(tiles, tb, wsrc, qsrc, threads)
        sec = t_topk + t_fc * nne / len(tiles)
        cpu = {"value": T / sec, "unit": "tokens/s", "cores": threads, "kind": "port",
               "sample": (f"router top-k over all {T} rows ({t_topk:.2f} s) + oracle FC1+FC2 over {len(tiles)} of "
                          f"{nne} token tiles ({t_fc:.2f} s), scaled by {nne}/{len(tiles)}")}

    if rank == 0:
        flops = layer_flops(T) * world
        line = {
            "metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "mxfp8 x mxfp4 (f32 accumulate)", "data": "synthetic",
            "config": prefill_config(T, E, zipf),
            "tflops": flops / (ms / 1e3) / 1e12,
            "pct_fp8_peak": flops / (ms / 1e3) / 1e12 / (FP8_PEAK_TFLOPS * world) * 100,
            "stage_ms": dict(zip(k3moe.MoELayer.STAGES, [round(float(v), 4) for v in stage_ms])),
            "routing": {"num_non_exiting": nne, "routed_rows": routed_rows, "touched_experts": touched,
                        "empty_experts": int((counts[:E] == 0).sum()), "max_expert_rows": int(counts[:E].max())},
            "roofline": {"kernel": "FC1 grouped GEMM (grouped_gemm_kernel<0>)", "bound": "hbm",
                         "achieved": achieved, "peak": hbm_peak, "unit": "GB/s", "frac": achieved / hbm_peak,
                         "peak_kind": peak_kind, "algorithmic_bytes_per_launch": fc1_bytes,
                         "traffic": traffic},
            "e2e": {"value": T * world / (e2e_ms / 1e3), "unit": "tokens/s", "ms_per_step": e2e_ms,
                    "h2d_bytes_per_step": int(x.numel() * 2 + S.numel() * 4),
                    "d2h_bytes_per_step": int(out.numel() * 2),
                    "copies": "every step's x, S in and output back over PCIe, on side streams overlapping the "
                              "neighbouring steps' compute (double buffers)"},
            "gpu_launches": 8 * args.steps,
            "gemm_trace": gemm_trace,
            "clocks": clk.summary(),
            "cpu_baseline": cpu,
        }
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
