"""Benchmark of the Kimi-K3 routed-MoE layer on B200 (config 1: an 8192-row prefill chunk on one GPU).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl k3moe|reference]

A step is one MoE layer over an 8192-row prefill chunk: router top-k ->
routing tables -> MXFP8 permute -> FC1 (MXFP8 x MXFP4, SwiGLU, MXFP8 out) ->
FC2 (bf16) -> routing-weighted combine, plus the always-on shared expert.
Shapes: T=8192 (16 packed sequences, Dirichlet lengths), H=7168, I=2048,
E=896 routed experts, top-8, routed scale 2.5, shared expert width 2048; all
expert weights MXFP4 (20.96 GB), synthetic and seeded (no checkpoint, no
dataset).  The inputs (x, router weight, bias) are made on the host with
numpy from fixed seeds, the same in both arms, and the router logits
S = x.W_router are computed once before timing (the router GEMM is the layer
before this path).

`value` is device-resident throughput (tokens/s over all ranks); `e2e` is the
same layer through the public API with x and S copied from pinned host memory
and the output copied back inside every timed step.  After timing, the CPU leg
checks the run's own intermediates against the CPU restatement (`parity`:
routing and quantisation bit for bit, FC1 / FC2 on sampled token tiles within
tolerance, the combine of sampled tokens bit for bit) and times that
restatement's FC1 + FC2 on the sample (`cpu_baseline`).  With N > 1 the layer is
expert parallel (config 4's layout): every rank owns an 8192-row chunk and
896/N experts (+ the shared expert), tokens travel to their experts' ranks and
back by NCCL all-to-all (timed separately), weak scaling; every rank then
checks its output bytes against the 1-GPU layer over all experts
(`ep_bit_identical`) and a config-2 decode step is timed at the same N
(`decode`).  `--impl reference` times the CPU restatement of the same path
(oracle/, the reference's algorithm) on a bounded sample on the host cores.
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


# ------------------------------------------------------------------ inputs (both arms)
def gpu_local_cpus(dev):
    """The host CPUs NVML reports as local to `dev` (its NUMA node), or None when NVML cannot say."""
    try:
        import pynvml
        import torch

        pynvml.nvmlInit()
        h = pynvml.nvmlDeviceGetHandleByUUID("GPU-" + str(torch.cuda.get_device_properties(dev).uuid))
        words = (os.cpu_count() + 63) // 64
        masks = pynvml.nvmlDeviceGetCpuAffinity(h, words)
        cpus = {64 * i + b for i, m in enumerate(masks) for b in range(64) if (int(m) >> b) & 1}
        cpus &= os.sched_getaffinity(0)
        return cpus or None
    except Exception:
        return None


class LocalHost:
    """Runs the block with this process on the host CPUs local to `dev`: pinned buffers allocated inside are
    first touched there, so they sit in the GPU's own NUMA node and N ranks' host copies spread over the
    sockets' memory instead of all crossing into one node.  The previous affinity comes back on exit."""

    def __init__(self, dev):
        self.dev, self.prev = dev, None

    def __enter__(self):
        cpus = gpu_local_cpus(self.dev)
        if cpus:
            self.prev = os.sched_getaffinity(0)
            os.sched_setaffinity(0, cpus)
        self.cpus = len(cpus) if cpus else None
        return self

    def __exit__(self, *a):
        if self.prev:
            os.sched_setaffinity(0, self.prev)


def bf16_round(a):
    """f32 -> bf16 bit patterns, round to nearest even (numpy)."""
    u = np.ascontiguousarray(a, dtype=np.float32).view(np.uint32).astype(np.uint64)
    return ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)


def host_inputs(T, E, seed_x, seed_router=7):
    """The layer's inputs, made on the host with numpy so both arms (the GPU arm and the CPU reference arm) route
    the same rows: x bf16 [T, H] ~ N(0, 1) (bit patterns), router weight [H, E] ~ N(0, 1/H) and S = x.W_router
    in f32, bias ~ U(-0.1, 0.1), rs = 2.5 (bf16 bits).  The router weight and bias are the same on every rank."""
    rng = np.random.default_rng(seed_x)
    x_bits = bf16_round(rng.standard_normal((T, H), dtype=np.float32))
    rr = np.random.default_rng(seed_router)
    wr = rr.standard_normal((H, E), dtype=np.float32) / np.float32(np.sqrt(H))
    bias = rr.uniform(-0.1, 0.1, E).astype(np.float32)
    xf = (x_bits.astype(np.uint32) << 16).view(np.float32)
    S = np.ascontiguousarray(xf @ wr, dtype=np.float32)
    return {"x_bits": x_bits, "S": S, "bias": bias, "rs_bits": int(bf16_round(np.array([RS], np.float32))[0]),
            "w_router": wr}


def device_inputs(h, dev):
    import torch

    x = torch.from_numpy(h["x_bits"].view(np.int16)).to(dev).view(torch.bfloat16)
    S = torch.from_numpy(h["S"]).to(dev)
    bias = torch.from_numpy(h["bias"]).to(dev)
    rs = torch.from_numpy(np.array([h["rs_bits"]], np.uint16).view(np.int16)).to(dev).view(torch.bfloat16)
    return x, S, bias, rs


def host_threads():
    """The host threads this process may run on (its CPU affinity), used explicitly by the CPU legs (torchrun
    sets OMP_NUM_THREADS=1, which the CPU restatement would otherwise inherit)."""
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:
        return os.cpu_count() or 1


def sample_tiles_of(nne, n):
    return sorted(set(np.linspace(0, nne - 1, n).astype(int).tolist()))


def tm_rows(block, K):
    """A 128-row block of a tile-major operand (K/128 tiles of 128 x 128 bytes) -> row-major [128, K]."""
    return np.ascontiguousarray(block.reshape(K // 128, 128, 128).transpose(1, 0, 2).reshape(128, K))


def rows_tm(rows128, K):
    """Row-major [128, K] -> one 128-row block of a tile-major operand (bytes)."""
    return np.ascontiguousarray(rows128.reshape(128, K // 128, 128).transpose(1, 0, 2).reshape(128, K))


# ------------------------------------------------------------------ the CPU leg: oracle as checker and as CPU baseline
def oracle_ffn(tiles, cta_batch, cta_limit, wsrc, qsrc, f1src=None, H=H, I=I):
    """The CPU restatement's FC1 + FC2 over token tiles `tiles` of a layer, on compact copies (tile i of the
    sample at rows [128 i, 128 i + 128)).  wsrc(e) -> (w13, w13_sf, w2, w2_sf) of expert e (tile-major bytes);
    qsrc(c) -> (q block [128, H] tile-major, its tiled scales).  FC2 reads FC1's output bytes from f1src(c) ->
    (block [128, I] tile-major, scales) when given (the device's own, for a check of FC2 alone), else the
    oracle's FC1 output.  Returns (FC1 q, FC1 sf, FC2 bf16 bits [ns*128, H], real rows a tile, seconds of the
    FC1 + FC2 calls)."""
    import oracle

    ns = len(tiles)
    kg4, ig4 = H // 128, I // 128
    qp = np.zeros((ns * 128, H), np.uint8)
    sfp = np.zeros(ns * kg4 * 512, np.uint8)
    w13 = np.zeros((ns * 2 * I, H // 2), np.uint8)
    w13sf = np.zeros(ns * 2 * I // 128 * kg4 * 512, np.uint8)
    w2 = np.zeros((ns * H, I // 2), np.uint8)
    w2sf = np.zeros(ns * H // 128 * ig4 * 512, np.uint8)
    cb = np.arange(ns, dtype=np.int32)
    cl = np.zeros(ns, np.int32)
    n_real = []
    for i, c in enumerate(tiles):
        e = int(cta_batch[c])
        n = int(cta_limit[c]) - c * 128
        n_real.append(n)
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
    t1 = time.perf_counter()
    if f1src is not None:
        dq = np.zeros_like(f1q)
        dsf = np.zeros_like(f1sf)
        for i, c in enumerate(tiles):
            a, s = f1src(c)
            dq[i * 128:(i + 1) * 128] = a
            dsf[i * ig4 * 512:(i + 1) * ig4 * 512] = s
        src_q, src_sf = dq, dsf
    else:
        src_q, src_sf = f1q, f1sf
    t2 = time.perf_counter()
    y = oracle.fc2(w2, w2sf, src_q, src_sf, cb, cl, 0, ns, H, I)
    t3 = time.perf_counter()
    return f1q, f1sf, y, n_real, (t1 - t0) + (t3 - t2)


def inrun_parity(layer, host, w, out, T, E, tiles, n_tokens=64):
    """The 1-GPU arm's check of its own timed run (after timing, outside the timed region): the run's
    intermediates, read back from the layer's workspace, against the CPU restatement on the same inputs.
    Bit-exact: router ids and weights (all rows), routing tables, the MXFP8 rows and scales of the sampled
    token tiles, the combine of `n_tokens` tokens (from the device's own FC2 rows).  Tolerance (rel-L2 <= 1e-2,
    max-abs <= 2e-2 widened per element to 3 bf16 ulp + 1e-3 as cases.within_contract): FC1 (dequantised
    MXFP8 out) and FC2 (bf16, from the device's own FC1 bytes) over the sampled tiles.  Also returns the CPU
    seconds of top-k (all rows) and of FC1 + FC2 over the tiles: the CPU baseline's sample.  FC1's output is
    MXFP8, so one requantised element may sit one E4M3 step from the oracle's where the two f32 accumulations
    straddle a rounding boundary: its check is rel-L2 <= 1e-2 of the dequantised rows, with the share of
    differing bytes reported."""
    import torch

    import cases
    import oracle

    off = layer.offsets(T)
    ws = layer.ws
    K_, H, I, SHARED = layer.K, layer.H, layer.I, layer.shared

    def get(name, nbytes, dtype=np.uint8, at=0):
        return ws[off[name] + at:off[name] + at + nbytes].cpu().numpy().view(dtype)

    meta = get("meta", 16, np.int32)
    nne, total_padded = int(meta[0]), int(meta[1])
    d_idx = get("idx", T * K_ * 4, np.int32).reshape(T, K_)
    d_wts = get("wts", T * K_ * 4, np.int32).reshape(T, K_)
    t0 = time.perf_counter()
    o_idx, o_wts = oracle.topk(host["S"], host["bias"], host["rs_bits"], K_)
    t_topk = time.perf_counter() - t0
    # ids bit for bit; the weights to an ulp or two (the CPU restatement's expf is the C library's, the device's
    # CUDA's: sigmoid may differ in its last bit)
    wd = np.abs(d_wts.astype(np.int64) - o_wts.view(np.int32).astype(np.int64))
    res = {"topk_ids_equal": bool(np.array_equal(d_idx, o_idx)), "topk_wts_max_ulp": int(wd.max()),
           "topk_wts_bits_equal_share": float(np.mean(wd == 0))}
    res["topk_equal"] = res["topk_ids_equal"] and res["topk_wts_max_ulp"] <= 4
    tb = oracle.tables(o_idx, E, 0, SHARED)
    cb = get("cta_batch", nne * 4, np.int32)
    cl = get("cta_limit", nne * 4, np.int32)
    e2p = get("exp2perm", T * K_ * 4, np.int32).reshape(T, K_)
    res["tables_equal"] = bool(
        np.array_equal(get("counts", (E + SHARED) * 4, np.int32), tb["counts"]) and
        np.array_equal(meta[:3], tb["meta"][:3]) and np.array_equal(cb, tb["cta_batch"][:nne]) and
        np.array_equal(cl, tb["cta_limit"][:nne]) and
        np.array_equal(get("route_map", total_padded * 4, np.int32), tb["route_map"][:total_padded]) and
        np.array_equal(e2p, tb["exp2perm"]))
    kg4, ig4 = H // 128, I // 128
    route_map = tb["route_map"]
    quant_ok = True

    def qsrc(c):
        nonlocal quant_ok
        q = get("q_perm", 128 * H, at=c * 128 * H).reshape(128, H)
        sf = get("sf_perm", kg4 * 512, at=c * kg4 * 512)
        n = int(cl[c]) - c * 128
        oq, osf = oracle.quant_mxfp8(host["x_bits"][route_map[c * 128:c * 128 + n]], tiled=True)
        real = np.zeros(kg4 * 512, bool)  # the scale bytes of the real rows
        r = np.arange(n)[:, None]
        kb = np.arange(H // 32)[None, :]
        real[((r // 128) * kg4 + kb // 4) * 512 + (r % 32) * 16 + ((r % 128) // 32) * 4 + kb % 4] = True
        quant_ok &= bool(np.array_equal(tm_rows(q, H)[:n], oq) and np.array_equal(sf[real], osf[real]))
        return q, sf

    per13 = 2 * I // 128 * kg4 * 512
    per2 = H // 128 * ig4 * 512

    def wsrc(e):
        return (w["w13"][e * 2 * I:(e + 1) * 2 * I].cpu().numpy(), w["w13_sf"][e * per13:(e + 1) * per13].cpu().numpy(),
                w["w2"][e * H:(e + 1) * H].cpu().numpy(), w["w2_sf"][e * per2:(e + 1) * per2].cpu().numpy())

    def f1src(c):
        return get("fc1_q", 128 * I, at=c * 128 * I).reshape(128, I), get("fc1_sf", ig4 * 512, at=c * ig4 * 512)

    f1q, f1sf, y, n_real, t_ffn = oracle_ffn(tiles, cb, cl, wsrc, qsrc, f1src, H, I)
    res["quant_tiles_equal"] = quant_ok
    rows = np.concatenate([np.arange(i * 128, i * 128 + n) for i, n in enumerate(n_real)])
    dq = np.concatenate([f1src(c)[0] for c in tiles])
    dsf = np.concatenate([f1src(c)[1] for c in tiles])
    got1 = oracle.dequant_rows(dq, dsf, rows)
    ref1 = oracle.dequant_rows(f1q, f1sf, rows)
    rel1 = cases.rel_l2(got1, ref1)
    ok1 = rel1 <= 1e-2
    res["fc1"] = {"rel_l2": rel1, "max_abs": float(np.abs(got1 - ref1).max()),
                  "e4m3_bytes_differing": float(np.mean(tm_rows_all(dq, I, rows) != tm_rows_all(f1q, I, rows))),
                  "ok": bool(ok1)}
    dfc2 = np.concatenate([get("fc2", 128 * H * 2, np.uint16, at=c * 128 * H * 2).reshape(128, H) for c in tiles])
    got2, ref2 = oracle.bf16_to_f32(dfc2[rows]), oracle.bf16_to_f32(y[rows])
    ok2, rel2, ratio2 = cases.within_contract(got2, ref2)
    res["fc2"] = {"rel_l2": rel2, "max_abs": float(np.abs(got2 - ref2).max()), "worst_vs_bound": ratio2,
                  "ok": bool(ok2)}
    # the combine of n_tokens tokens from the device's own FC2 rows: bit-exact
    toks = sample_tiles_of(T, n_tokens)
    nt = len(toks)
    prow = e2p[toks]                                   # [nt, K] permuted rows
    srow = int(meta[2]) + np.asarray(toks) if SHARED else None
    gather = np.concatenate([prow.reshape(-1)] + ([srow] if SHARED else [])).astype(np.int64)
    fc2_all = ws[off["fc2"]:off["fc2"] + total_padded * H * 2].view(torch.int16).view(-1, H)
    fc2rows = torch.index_select(fc2_all, 0, torch.from_numpy(gather).to(ws.device)).cpu().numpy().view(np.uint16)
    ce2p = np.where(prow >= 0, np.arange(nt * K_).reshape(nt, K_), -1).astype(np.int32)
    cmeta = np.array([0, 0, nt * K_ if SHARED else -1, 0], np.int32)
    ocomb = oracle.combine(fc2rows, ce2p, d_wts[toks].view(np.float32), cmeta, nt, K_)
    dout = out[toks].view(torch.int16).cpu().numpy().view(np.uint16)
    res["combine_tokens_equal"] = bool(np.array_equal(ocomb, dout))
    res["tiles"] = len(tiles)
    res["combine_tokens"] = nt
    res["ok"] = bool(res["topk_equal"] and res["tables_equal"] and quant_ok and ok1 and ok2 and
                     res["combine_tokens_equal"])
    return res, t_topk, t_ffn


def tm_rows_all(buf, K, rows):
    """Rows `rows` of a compact tile-major operand [n*128, K] as row-major bytes."""
    import oracle

    return oracle.t128_rows(buf, rows, K)


# ------------------------------------------------------------------ the reference arm (CPU)
def ep_config(T, E, world, args):
    return {"workload": f"K3-shape prefill MoE layer, expert parallel over {world} GPUs (config 4 layout)",
            "T_per_gpu": T, "H": H, "I": I, "E": E, "E_per_gpu": E // world, "K": K, "shared_expert_width": I,
            "rs": RS, "global_batch": T * world, "seq_len": T, "parallelism": f"ep{world}",
            "expert_placement": args.ep_placement, "fc2_slices": args.ep_overlap, "fc2_grid_cap": args.ep_fc2_cap,
            "transport": args.ep_transport,
            "l2": "inputs larger than L2: each GPU streams its experts' weights every step"}


def run_reference(args):
    """The reference's algorithm on the host cores: the CPU restatement (oracle/, kind "port") on the GPU arm's
    own inputs (the same host generator and seeds, so the same routing and tiles).  A step times the router top-k
    over every row plus FC1 + FC2 over `--cpu-tiles` token tiles spread over the layer (a bounded sample); the
    value projects it to the whole layer (all its tiles).  With N > 1 rank 0 runs its own chunk of the
    expert-parallel job (the host cores would run the N chunks one after another: the same tokens/s)."""
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    if rank != 0:
        return
    import oracle

    threads = oracle.set_threads(host_threads())
    T, E = args.tokens, args.experts
    hin = host_inputs(T, E, 1000)
    bias, zipf = hin["bias"], None
    if args.zipf and world == 1:  # the GPU arm's config-3 bias, fitted on the same logits
        import cases

        bias, beta, kl = cases.zipf_bias(hin["S"], K)
        zipf = {"s": 1.1, "seed": 3, "beta": beta, "kl": round(kl, 4)}
    idx, wts = oracle.topk(hin["S"], bias, hin["rs_bits"], K)
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
        n = int(tb["cta_limit"][c]) - c * 128
        rows = np.zeros(128, np.int64)
        rows[:n] = tb["route_map"][c * 128:c * 128 + n]
        q, sf = oracle.quant_mxfp8(hin["x_bits"][rows], tiled=True)
        return rows_tm(q, H), sf

    for c in tiles:
        wsrc(int(tb["cta_batch"][c]))
    step_s, layer_s = [], []
    for step in range(args.warmup + args.steps):
        t0 = time.perf_counter()
        t1 = time.perf_counter()
        oracle.topk(hin["S"], bias, hin["rs_bits"], K)
        t_topk = time.perf_counter() - t1
        t_ffn = oracle_ffn(tiles, tb["cta_batch"], tb["cta_limit"], wsrc, qsrc)[4]
        if step >= args.warmup:
            step_s.append(time.perf_counter() - t0)
            layer_s.append(t_topk + t_ffn * nne / len(tiles))
    sec = statistics.mean(layer_s)
    value = T / sec
    sample = (f"router top-k over all {T} rows + oracle FC1+FC2 over {len(tiles)} of {nne} token tiles (spread "
              f"evenly), timed each step and projected to all {nne} tiles (whole layer {sec * 1e3:.0f} ms)")
    config = prefill_config(T, E, zipf) if world == 1 else ep_config(T, E, world, args)
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": statistics.mean(step_s) * 1e3,
        "layer_ms_projected": sec * 1e3, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "mxfp8 x mxfp4 (f32 accumulate)", "data": "synthetic",
        "config": config, "routing": {"num_non_exiting": nne},
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


def full_layer(E, bias, rs, T, dev):
    """The 1-GPU layer over every expert (the same synthetic weight streams as the ranks' slices): the
    expert-parallel arm's check that its output is the same bytes."""
    import k3moe

    w13, w13_sf = k3moe.synth_mxfp4(W_SEED13, (E + SHARED) * 2 * I, H, WSD, device=dev)
    w2, w2_sf = k3moe.synth_mxfp4(W_SEED2, (E + SHARED) * H, I, WSD, device=dev)
    return k3moe.MoELayer(H, I, E, K, SHARED, w13, w13_sf, w2, w2_sf, bias, rs, max_tokens=T, device=dev)


# ------------------------------------------------------------------ the GPU arm, N > 1: expert parallel
def run_ep(args, world, rank, dev):
    """Config 4's layout at N GPUs: every rank owns an 8192-row chunk (16 packed sequences) and E/N experts
    (+ the shared expert); dispatch and combine by the chosen transport (default: the device-resident step, one
    C-ABI call with peer-memory stores and no host synchronisation); weak scaling (N x 8192 rows a step).
    After timing, every rank checks its output against the 1-GPU layer over all experts on its own rows
    (`ep_bit_identical`, all ranks), and a config-2 decode step (64 tokens over the N ranks) is timed as a
    CUDA graph and checked the same way (`decode`)."""
    import torch
    import torch.distributed as dist

    import k3moe_ep

    E, T = args.experts, args.tokens
    El = E // world
    x, S, bias, rs = device_inputs(host_inputs(T, E, 1000 + rank), dev)
    owner, mine = rank_experts(E, world, rank, bias, args.ep_placement)
    w = rank_weights(E, mine, dev)
    device_step = args.ep_transport == "device"
    if device_step:
        layer = k3moe_ep.DeviceEPMoELayer(H, I, E, K, SHARED, w, bias, rs, max_tokens=T, owner=owner, device=dev)
    else:
        layer = k3moe_ep.EPMoELayer(H, I, E, K, SHARED, w, bias, rs, device=dev, owner=owner,
                                    overlap_chunks=args.ep_overlap, fc2_grid_cap=args.ep_fc2_cap,
                                    transport=args.ep_transport,
                                    max_tokens=T if args.ep_transport == "peer" else None)
    for _ in range(args.warmup):
        layer.forward(S, x)
    torch.cuda.synchronize()
    names = ("dispatch", "fc1", "combine")
    if device_step:  # the step's 8 stage events, read as the same three intervals
        evs = [[torch.cuda.Event(enable_timing=True) for _ in range(8)] for _ in range(args.steps)]
    else:
        evs = [{n: (torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for n in names}
               for _ in range(args.steps)]
    start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    dist.barrier()
    torch.cuda.synchronize()
    uuid = "GPU-" + str(torch.cuda.get_device_properties(dev).uuid)
    with ClockSampler(uuid) as clk:
        start.record()
        for s in range(args.steps):
            layer.forward(S, x, events=evs[s])
        stop.record()
        torch.cuda.synchronize()
    dist.barrier()
    ms = start.elapsed_time(stop) / args.steps
    if device_step:  # dispatch: pack + exchange; fc1; combine: FC2's end to every peer's results in
        spans = {"dispatch": (1, 2), "fc1": (3, 4), "combine": (5, 6)}
        part = {n: float(np.mean([e[a].elapsed_time(e[b]) for e in evs])) for n, (a, b) in spans.items()}
    else:
        part = {n: float(np.mean([e[n][0].elapsed_time(e[n][1]) for e in evs])) for n in names}
    t = torch.tensor([ms, part["dispatch"], part["combine"], part["fc1"]], device=dev)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms, disp_ms, comb_ms, fc1_ms = [float(v) for v in t.tolist()]
    # e2e: x and S from pinned host memory in, the output back, every step (copies overlapped)
    with LocalHost(dev) as local:
        x_h, S_h = x.cpu().pin_memory(), S.cpu().pin_memory()
        dist.barrier()
        n_e2e = args.e2e_steps or args.steps
        e2e_ms = e2e_overlapped(lambda Sd, xd, od: layer.forward(Sd, xd), S_h, x_h, (T, H), n_e2e,
                                torch.cuda.current_stream(), dev)
    t = torch.tensor([e2e_ms], device=dev)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    e2e_ms = float(t.item())
    counts = (layer.expert_rows() if device_step else layer.last["tables"].counts).cpu().numpy()
    routed_rows, touched = int(counts.sum()), int((counts > 0).sum())
    fc1_bytes = touched * (2 * I * H // 2 + 2 * I * H // 32) + routed_rows * (H + H // 32 + I + I // 32)
    # ---------------- the check (untimed): this rank's rows through the 1-GPU layer over all 896 experts
    out_ep = layer.forward(S, x)
    torch.cuda.synchronize()
    full = full_layer(E, bias, rs, T, dev)
    out_1 = full.forward(S, x)
    torch.cuda.synchronize()
    full.check_device_error(T)
    # the transport's bounded waits and table checks
    words = list(layer.error_words()[1]) if device_step else layer.ops.err[:2].tolist()
    same = torch.tensor([1 if torch.equal(out_ep.view(torch.int16), out_1.view(torch.int16)) and words == [0, 0]
                         else 0], device=dev)
    dist.all_reduce(same, op=dist.ReduceOp.MIN)
    ep_identical = bool(same.item() == 1)
    del out_1
    # ---------------- config 2 at this N: a 64-token decode step, CUDA graph, checked against the full layer
    dec = decode_pass(args, world, rank, dev, w, owner, full) if args.decode_tokens % world == 0 else None
    del full
    hbm_peak, peak_kind = peaks()
    if rank == 0:
        flops = layer_flops(T) * world
        achieved = fc1_bytes / (fc1_ms / 1e3) / 1e9
        line = {
            "metric": METRIC, "value": T * world / (ms / 1e3), "unit": "tokens/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "mxfp8 x mxfp4 (f32 accumulate)", "data": "synthetic",
            "config": ep_config(T, E, world, args),
            "tflops": flops / (ms / 1e3) / 1e12,
            "a2a_ms": {"dispatch": disp_ms, "combine": comb_ms},
            "ep_bit_identical": ep_identical,
            "parity": {"ep_bit_identical": ep_identical, "ranks_checked": world,
                       "against": "the 1-GPU layer over all experts on each rank's own 8192 rows", "ok": ep_identical},
            "roofline": {"kernel": "FC1 grouped GEMM (grouped_gemm_kernel<0>), rank 0", "bound": "hbm",
                         "achieved": achieved, "peak": hbm_peak, "unit": "GB/s", "frac": achieved / hbm_peak,
                         "peak_kind": peak_kind, "algorithmic_bytes_per_launch": fc1_bytes,
                         "traffic": fc1_traffic(fc1_bytes), "traffic_source": TRAFFIC_SOURCE},
            "e2e": {"value": T * world / (e2e_ms / 1e3), "unit": "tokens/s", "ms_per_step": e2e_ms,
                    "h2d_bytes_per_step": int(x.numel() * 2 + S.numel() * 4) * world,
                    "d2h_bytes_per_step": int(x.numel() * 2) * world,
                    "copies": "every step's x, S in and output back over PCIe, on side streams overlapping the "
                              "neighbouring steps' compute (double buffers)",
                    "host_buffers": "pinned on each GPU's local NUMA node" if local.cpus else "NUMA placement unknown"},
            # nccl / peer: topk, 2 x 3 plan launches, pairs, pack, shared pack, ids, 3 table launches, unpack,
            # return rows, FC1, FC2 (a launch a slice), combine (+ peer: row pointers, 2 signals, 2 waits);
            # device: topk, plan, pack, exchange, ids, 3 table launches, unpack, FC1, row pointers, FC2,
            # exchange, combine
            "gpu_launches": (14 if device_step else
                             18 + args.ep_overlap + (4 if args.ep_transport == "peer" else 0)) * args.steps,
            "decode": dec,
            "clocks": clk.summary(),
            "cpu_baseline": None,
        }
        print(json.dumps(line), flush=True)
    dist.barrier()
    layer.close()
    dist.barrier()
    dist.destroy_process_group()


# ------------------------------------------------------------------ decode (config 2)
DECODE_METRIC = "EP decode us/layer (64 tokens x top-8)"


def decode_pass(args, world, rank, dev, w, owner, full):
    """Config 2 inside the expert-parallel run: 64 tokens (rank r owns rows [r T, r T + T) of one global batch)
    through this rank's experts `w` by the device-resident step (transport "device"), or with fixed-size
    all-to-all blocks over NCCL (the other transports); neither synchronises with the host, and the whole step is
    captured as one CUDA graph and replayed.  Returns us a layer (max over ranks), an eager breakdown, and
    whether every rank's output equals the 1-GPU layer `full` on the same rows."""
    import torch
    import torch.distributed as dist

    import k3moe_ep

    E, Tall = args.experts, args.decode_tokens
    T = Tall // world
    x_all, S_all, bias, rs = device_inputs(host_inputs(Tall, E, 2000), dev)
    x, S = x_all[rank * T:(rank + 1) * T].contiguous(), S_all[rank * T:(rank + 1) * T].contiguous()
    device_step = args.ep_transport == "device"
    if device_step:
        layer = k3moe_ep.DeviceEPMoELayer(H, I, E, K, SHARED, w, bias, rs, max_tokens=T, owner=owner, device=dev)
    else:
        layer = k3moe_ep.EPMoELayer(H, I, E, K, SHARED, w, bias, rs, device=dev, fixed_tokens=T, owner=owner)
    run = lambda: layer.forward(S, x)  # noqa: E731
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        for _ in range(max(args.warmup, 3)):
            run()
    torch.cuda.current_stream().wait_stream(side)
    torch.cuda.synchronize()
    steps = max(args.steps, 20)

    def mx(v):
        t = torch.tensor([v], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    def timed(step):
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        dist.barrier()
        torch.cuda.synchronize()
        a.record()
        for _ in range(steps):
            step()
        b.record()
        torch.cuda.synchronize()
        return mx(a.elapsed_time(b) / steps * 1e3)

    eager_us = timed(run)
    # eager breakdown: the dispatch all-to-all, the expert GEMMs (tables .. FC2), the combine all-to-all
    names = ("dispatch", "ffn", "combine")
    dist.barrier()
    if device_step:  # dispatch: plans + pack + exchange; ffn: tables .. FC2; combine: exchange + combine
        ev8 = [torch.cuda.Event(enable_timing=True) for _ in range(8)]
        layer.forward(S, x, events=ev8)
        torch.cuda.synchronize()
        spans = {"dispatch": (0, 2), "ffn": (2, 5), "combine": (5, 7)}
        stage_us = {n: round(mx(ev8[a].elapsed_time(ev8[b]) * 1e3), 1) for n, (a, b) in spans.items()}
    else:
        ev = {n: (torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for n in names}
        layer.forward(S, x, ev)
        torch.cuda.synchronize()
        stage_us = {n: round(mx(ev[n][0].elapsed_time(ev[n][1]) * 1e3), 1) for n in names}
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        static_out = run()
    graph.replay()
    torch.cuda.synchronize()
    us = timed(graph.replay)
    graph.replay()
    torch.cuda.synchronize()
    ref = full.forward(S, x)
    torch.cuda.synchronize()
    same = torch.tensor([1 if torch.equal(static_out.view(torch.int16), ref.view(torch.int16)) else 0], device=dev)
    dist.all_reduce(same, op=dist.ReduceOp.MIN)
    counts = (layer.expert_rows() if device_step else layer.last["tables"].counts).cpu().numpy()
    per_expert = 2 * I * H // 2 + 2 * I * H // 32 + H * I // 2 + H * I // 32
    wbytes = mx(float(int((counts > 0).sum()) * per_expert))
    hbm_peak, _ = peaks()
    graph.reset()
    del graph
    torch.cuda.synchronize()
    if device_step:
        dist.barrier()  # every rank's last step done before the peers' buffers are unmapped
        layer.close()
    return {"us": us, "eager_us": eager_us, "graph": True, "tokens": Tall, "tokens_per_gpu": T,
            "transport": args.ep_transport,
            "stage_us_eager": stage_us, "bit_identical_to_1gpu": bool(same.item() == 1),
            "roofline": {"bound": "hbm", "bytes_slowest_rank": wbytes,
                         "frac": wbytes / (us / 1e6) / 1e9 / hbm_peak}}


def run_decode(args, world, rank, dev):
    """Config 2 alone (`--decode`): one MoE decode step of 64 tokens x top-8 over E = 896 experts, expert
    parallel over the N GPUs (64/N tokens each); the figure is microseconds a layer, max over ranks."""
    import torch
    import torch.distributed as dist

    import k3moe
    import k3moe_ep

    E, Tall = args.experts, args.decode_tokens
    if Tall % world or E % world:
        raise SystemExit(f"--decode needs tokens ({Tall}) and experts ({E}) divisible by {world}")
    T, El = Tall // world, E // world
    x_all, S_all, bias, rs = device_inputs(host_inputs(Tall, E, 2000), dev)
    x, S = x_all[rank * T:(rank + 1) * T].contiguous(), S_all[rank * T:(rank + 1) * T].contiguous()
    if world == 1:
        layer = full_layer(E, bias, rs, T, dev)
        out = torch.empty((T, H), dtype=torch.bfloat16, device=dev)
        run = lambda: layer.forward(S, x, out)  # noqa: E731
    else:
        owner, mine = rank_experts(E, world, rank, bias, args.ep_placement)
        w = rank_weights(E, mine, dev)
        if args.ep_transport == "device":
            layer = k3moe_ep.DeviceEPMoELayer(H, I, E, K, SHARED, w, bias, rs, max_tokens=T, owner=owner,
                                              device=dev)
        else:
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
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        static_out = run()
    graph.replay()
    torch.cuda.synchronize()
    uuid = "GPU-" + str(torch.cuda.get_device_properties(dev).uuid)
    with ClockSampler(uuid) as clk:
        us = timed(graph.replay)
    # end to end: this rank's x and S from pinned host memory into the step's inputs, its output back
    local = LocalHost(dev).__enter__()  # pinned buffers on this GPU's NUMA node (restored below)
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
        graph.replay()
        out_h.copy_(static_out, non_blocking=True)
    e1.record()
    torch.cuda.synchronize()
    e2e_us = max_over_ranks(e0.elapsed_time(e1) / n_e2e * 1e3)
    local.__exit__()
    # bytes a layer must stream on the slowest rank: its touched experts' weights (+ the shared expert's)
    if world == 1:
        off = layer.offsets(T)
        counts = layer.ws[off["counts"]:off["counts"] + 4 * (E + SHARED)].view(torch.int32).cpu().numpy()
    elif args.ep_transport == "device":
        counts = layer.expert_rows().cpu().numpy()
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
                       "transport": args.ep_transport if world > 1 else None,
                       "l2": "inputs larger than L2: each step streams the touched experts' weights"},
            "roofline": {"kernel": "whole decode layer (weights of the touched experts, slowest rank)",
                         "bound": "hbm", "achieved": achieved, "peak": hbm_peak, "unit": "GB/s",
                         "frac": achieved / hbm_peak, "peak_kind": peak_kind, "algorithmic_bytes_per_launch": wbytes,
                         "traffic": None},
            "routing": {"touched_experts_max_rank": int(wbytes // per_expert)},
            "e2e": {"value": e2e_us, "unit": "us/layer", "h2d_bytes_per_step": int(x.numel() * 2 + S.numel() * 4),
                    "d2h_bytes_per_step": int(x.numel() * 2)},
            "gpu_launches": (8 if world == 1 else 14) * args.steps,
            "cuda_graph": True, "eager_us": eager_us,
            "clocks": clk.summary(),
            "cpu_baseline": None,
        }
        print(json.dumps(line), flush=True)
    # a graph holding NCCL calls is released before the process group goes
    graph.reset()
    del graph
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
        if args.ep_transport == "device":
            layer.close()
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


def router_gemm_timing(x, wr, dev, n=20):
    """The router GEMM S = x . W_router^T (bf16 in, f32 out, k3moe_router_gemm) timed with CUDA events, against
    cuBLAS's bf16 GEMM of the same operands (torch.mm, bf16 out), and checked against an f32 matmul."""
    import torch

    import k3moe

    w = torch.from_numpy(bf16_round(np.ascontiguousarray(wr.T)).view(np.int16)).to(dev).view(torch.bfloat16)
    T, Hh = x.shape
    E_ = w.shape[0]
    err = torch.zeros(4, dtype=torch.int32, device=dev)
    S = k3moe.router_gemm(x, w, err)
    ref = x.float() @ w.float().t()
    rel = float((S - ref).norm() / ref.norm())

    def timed(fn):
        for _ in range(3):
            fn()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        torch.cuda.synchronize()
        a.record()
        for _ in range(n):
            fn()
        b.record()
        torch.cuda.synchronize()
        return a.elapsed_time(b) / n

    ms = timed(lambda: k3moe.router_gemm(x, w, err))
    ms_cublas = timed(lambda: torch.mm(x, w.t()))
    flop = 2.0 * T * Hh * E_
    try:
        peak = float(json.load(open(os.path.join(ROOT, "MEASURED_PEAKS.json")))["bf16_tflops"])
        kind = "measured"
    except Exception:
        peak, kind = 1590.0, "fallback"
    return {"ms": ms, "tflops": flop / ms / 1e9, "cublas_bf16_out_ms": ms_cublas, "vs_cublas": ms_cublas / ms,
            "frac_of_bf16_peak": flop / ms / 1e9 / peak, "peak_kind": kind, "rel_l2_vs_f32": rel,
            "device_error_words": err[:2].tolist(), "shape": [T, Hh, E_]}


def reference_kernels_leg(x, S, w, bias, rs, E, dev, n=20):
    """The reference's own GEMM family on this GPU (a baseline, like the CPU leg): FlashInfer's TRT-LLM-gen MoE
    (oracle/flashinfer_ref.py) on the same quantised operands, routed experts only (it has no shared expert),
    tuned on this token count; beside it this build's layer without the shared expert on the same rows.  Both
    timed with CUDA events after warm-up; their outputs compared (rel-L2)."""
    import torch

    import flashinfer_ref
    import k3moe

    if not flashinfer_ref.available():
        return {"unavailable": "FlashInfer's TRT-LLM-gen launcher is not prebuilt (make -C oracle flashinfer)"}
    T = x.shape[0]
    ne = E * 2 * I
    mine = k3moe.MoELayer(H, I, E, K, 0, w["w13"], w["w13_sf"], w["w2"], w["w2_sf"], bias, rs, max_tokens=T,
                          device=dev)
    out = torch.empty((T, H), dtype=torch.bfloat16, device=dev)

    def timed(fn):
        for _ in range(3):
            fn()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        torch.cuda.synchronize()
        a.record()
        for _ in range(n):
            fn()
        b.record()
        torch.cuda.synchronize()
        return a.elapsed_time(b) / n

    ms_mine = timed(lambda: mine.forward(S, x, out))
    off = mine.offsets(T)
    idx = mine.ws[off["idx"]:off["idx"] + T * K * 4].view(torch.int32).view(T, K).clone()
    wts = mine.ws[off["wts"]:off["wts"] + T * K * 4].view(torch.float32).view(T, K).clone()
    kg4 = H // 128
    ref = flashinfer_ref.ReferenceMoE(w["w13"][:ne], w["w13_sf"][:ne // 128 * kg4 * 512], w["w2"][:E * H],
                                      w["w2_sf"][:E * H // 128 * (I // 128) * 512], E, H, I, K)
    q, sf = k3moe.quant_mxfp8(x, tiled_sf=False)
    qf = q.view(torch.float8_e4m3fn)
    tk = flashinfer_ref.pack_topk(idx, wts)
    ref.tune(qf, sf, tk)
    ms_ref = timed(lambda: ref.forward(qf, sf, tk, finalize=True, tune_max=T))
    ms_quant = timed(lambda: k3moe.quant_mxfp8(x, tiled_sf=False))
    y = ref.forward(qf, sf, tk, finalize=True, tune_max=T)
    torch.cuda.synchronize()
    rel = float((out.float() - y.float()).norm() / y.float().norm())
    del ref, mine
    torch.cuda.empty_cache()
    return {"flashinfer_trtllm_gen_ms": ms_ref, "flashinfer_input_quant_ms": ms_quant,
            "k3moe_routed_layer_ms": ms_mine, "vs_reference_kernels": (ms_ref + ms_quant) / ms_mine,
            "output_rel_l2": rel,
            "what": "routed experts only (no shared expert), the same rows, routing and quantised operands; "
                    "FlashInfer 0.6.11 trtllm_fp4_block_scale_routed_moe (routing from the given top-k, FC1, FC2, "
                    "finalize), tuned on this token count, plus its input MXFP8 quantisation; k3moe: the whole "
                    "layer (top-k, tables, permute, FC1, FC2, combine)"}


TRAFFIC_SOURCE = ("ncu DRAM bytes (read + write) per algorithmic byte of FC1 on the small-case capture "
                  "(profiles/grouped_gemm_fc1_fc2_small_case.md), times this launch's algorithmic bytes")


def fc1_traffic(fc1_bytes):
    """DRAM bytes (read + write) of one FC1 launch of this workload: the ratio of DRAM traffic to algorithmic
    bytes measured by ncu on the small-case capture of the same kernel
    (profiles/grouped_gemm_fc1_fc2_small_case.md, line "fc1_dram_per_algorithmic_byte: R"), scaled by this
    launch's algorithmic bytes (traffic grows with the touched experts' weights and the rows, as the bytes do).
    Returns the bytes, or None when the summary is absent."""
    tf = os.path.join(ROOT, "profiles", "grouped_gemm_fc1_fc2_small_case.md")
    if not os.path.exists(tf):
        return None
    for ln in open(tf):
        if ln.startswith("fc1_dram_per_algorithmic_byte:"):
            r = float(ln.split(":")[1].strip())
            return r * fc1_bytes
    return None


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="k3moe", choices=["k3moe", "reference"])
    ap.add_argument("--tokens", type=int, default=T_DEF)
    ap.add_argument("--experts", type=int, default=896, help="routed experts (smaller only for profiling captures)")
    ap.add_argument("--e2e-steps", type=int, default=0, help="e2e steps (default: --steps)")
    ap.add_argument("--cpu-tiles", type=int, default=16, help="token tiles in the CPU leg's sample")
    ap.add_argument("--no-cpu-baseline", action="store_true", help="skip the CPU leg (parity check and baseline)")
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
    ap.add_argument("--no-reference-kernels", action="store_true",
                    help="skip the leg that times the reference's GEMM family (FlashInfer TRT-LLM-gen) on this GPU")
    ap.add_argument("--ep-transport", default="device", choices=["nccl", "peer", "device"],
                    help="N > 1: the two all-to-alls over NCCL; stores into the peers' buffers over NVLink after "
                         "a counts exchange (peer); or the device-resident step, one C-ABI call with fixed peer "
                         "regions and no host synchronisation (device)")
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
    hin = host_inputs(T, E, 1000)
    zipf = None
    if args.zipf:  # config 3: bias fitted (on the host) so the realised top-8 histogram follows Zipf(1.1)
        import cases

        zb, beta, kl = cases.zipf_bias(hin["S"], K)
        hin["bias"] = zb
        zipf = {"s": 1.1, "seed": 3, "beta": beta, "kl": round(kl, 4)}
    x, S, bias, rs = device_inputs(hin, dev)
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
    uuid = "GPU-" + str(torch.cuda.get_device_properties(dev).uuid)
    with ClockSampler(uuid) as clk:
        start.record(stream)
        for s in range(args.steps):
            layer.forward_events(S, x, out, ev[s])
        stop.record(stream)
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
    value = T / (ms / 1e3)

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

    # ---------------- end to end through the public API: host x/S in, host out back
    e2e_steps = args.e2e_steps or args.steps

    def fwd(Sd, xd, od):
        layer.forward(Sd, xd, od)
        return od

    with LocalHost(dev):
        x_h = x.cpu().pin_memory()
        S_h = S.cpu().pin_memory()
        e2e_ms = e2e_overlapped(fwd, S_h, x_h, (T, H), e2e_steps, stream, dev)
    layer.check_device_error(T)

    # ---------------- the router GEMM (the step before the path, outside the layer's time): this build's
    # tcgen05 kernel against cuBLAS (torch.mm, bf16 out) on the same x and W_router (bf16)
    router = router_gemm_timing(x, hin["w_router"], dev)
    refk = None
    if not args.no_reference_kernels:
        try:
            refk = reference_kernels_leg(x, S, {"w13": w13, "w13_sf": w13_sf, "w2": w2, "w2_sf": w2_sf}, bias, rs,
                                         E, dev)
        except Exception as ex:  # the baseline may not load here: the line says why
            refk = {"unavailable": f"{type(ex).__name__}: {str(ex)[:200]}"}

    # ---------------- the CPU leg (after timing): the oracle checks this run's own intermediates on sampled
    # token tiles and every row's routing, and its FC1 + FC2 time over the sample is the CPU baseline
    cpu, parity = None, None
    if not args.no_cpu_baseline:
        import oracle

        threads = oracle.set_threads(host_threads())
        layer.forward(S, x, out)  # the workspace holds this call's intermediates
        torch.cuda.synchronize()
        tiles = sample_tiles_of(nne, args.cpu_tiles)
        wd = {"w13": w13, "w13_sf": w13_sf, "w2": w2, "w2_sf": w2_sf}
        parity, t_topk, t_fc = inrun_parity(layer, hin, wd, out, T, E, tiles)
        sec = t_topk + t_fc * nne / len(tiles)
        cpu = {"value": T / sec, "unit": "tokens/s", "cores": threads, "kind": "port",
               "sample": (f"router top-k over all {T} rows ({t_topk:.2f} s) + oracle FC1+FC2 over {len(tiles)} of "
                          f"{nne} token tiles ({t_fc:.2f} s, spread evenly), projected to all {nne} tiles")}

    flops = layer_flops(T)
    line = {
        "metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": 1, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "mxfp8 x mxfp4 (f32 accumulate)", "data": "synthetic",
        "config": prefill_config(T, E, zipf),
        "tflops": flops / (ms / 1e3) / 1e12,
        "pct_fp8_peak": flops / (ms / 1e3) / 1e12 / FP8_PEAK_TFLOPS * 100,
        "stage_ms": dict(zip(k3moe.MoELayer.STAGES, [round(float(v), 4) for v in stage_ms])),
        "routing": {"num_non_exiting": nne, "routed_rows": routed_rows, "touched_experts": touched,
                    "empty_experts": int((counts[:E] == 0).sum()), "max_expert_rows": int(counts[:E].max())},
        "roofline": {"kernel": "FC1 grouped GEMM (grouped_gemm_kernel<0>)", "bound": "hbm",
                     "achieved": achieved, "peak": hbm_peak, "unit": "GB/s", "frac": achieved / hbm_peak,
                     "peak_kind": peak_kind, "algorithmic_bytes_per_launch": fc1_bytes,
                     "traffic": fc1_traffic(fc1_bytes), "traffic_source": TRAFFIC_SOURCE},
        "parity": parity,
        "e2e": {"value": T / (e2e_ms / 1e3), "unit": "tokens/s", "ms_per_step": e2e_ms,
                "h2d_bytes_per_step": int(x.numel() * 2 + S.numel() * 4),
                "d2h_bytes_per_step": int(out.numel() * 2),
                "copies": "every step's x, S in and output back over PCIe, on side streams overlapping the "
                          "neighbouring steps' compute (double buffers)"},
        "gpu_launches": 8 * args.steps,
        "router_gemm": router,
        "reference_kernels": refk,
        "gemm_trace": gemm_trace,
        "clocks": clk.summary(),
        "cpu_baseline": cpu,
    }
    print(json.dumps(line), flush=True)


if __name__ == "__main__":
    main()
