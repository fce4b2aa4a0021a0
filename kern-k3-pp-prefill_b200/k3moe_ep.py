"""Expert-parallel routed-MoE layer: one process a GPU, experts split in
contiguous blocks, tokens owned by their rank, dispatch and combine as NCCL
all-to-all (torch.distributed for the plumbing; the only collective of the path).

Per rank (world W, E_local = E / W experts, T local tokens):

1. router top-k on the local tokens (global expert ids);
2. two plans from the routing-table builder with tile 1 (deterministic): over
   the expanded (token, k) picks by destination rank, each pick's row among the
   results that come back (grouped by rank, (token, k) order within one); and
   over the (token, rank) pairs, each token's slot in the send buffer of every
   rank holding any of its picks;
3. pack: each token quantised to MXFP8 once and written once a destination
   rank, headed by the local expert ids of its picks there (E4M3 | UE8M0 |
   int16 ids): a token with several experts on one rank crosses the link once;
4. counts all-to-all (rows and picks a rank; the one host synchronisation),
   then the dispatch all-to-all of the rows; the local tokens are appended for
   the shared expert, which every rank holds (local expert E_local);
5. routing tables over the received rows' ids (K a row), unpack each row into
   the GEMM operand at all its experts, FC1, FC2 storing each (row, pick)
   result at its number in (row, pick) order;
6. the combine all-to-all sends the results back, one row a pick, to the
   owner, which sums its K rows in k order with f32 FMAs plus the shared row:
   the single-GPU combine's arithmetic, so the layer's output is bit-identical
   to one GPU holding every expert.

The fixed-block mode (decode) sends one row a pick in fixed-size blocks.

DeviceEPMoELayer is the same layer as one C-ABI call a step (k3moe_ep_forward): fixed receive regions in
peer memory, no host synchronisation, capturable whole in a CUDA graph; the output is the same bytes.

The reference has no MoE all-to-all (its decode EP replicates the batch and
all-reduces, roofline/decode.md:164-166); this is the token-sharded layout of
the benchmark configurations.
"""
from __future__ import annotations

import ctypes
import math

import torch
import torch.distributed as dist

import k3moe


class GpuOps:
    """The path's steps on the GPU (libk3moe.so through the C ABI)."""

    def __init__(self, device):
        self.device = device
        self.err = torch.zeros(4, dtype=torch.int32, device=device)

    def topk(self, S, bias, rs, K):
        return k3moe.route_topk(S, bias, rs, K)

    def tables(self, ids, E, tile):
        return k3moe.route_tables(ids, E, 0, 0, tile)

    def stride(self, H):
        return k3moe.lib().k3moe_ep_row_stride(H)

    def pack(self, x, idx, send_pos, E_local, n_slots, out=None):
        H = x.shape[1]
        st = self.stride(H)
        buf = torch.empty((n_slots, st), dtype=torch.uint8, device=x.device) if out is None else out
        k3moe._check(k3moe.lib().k3moe_ep_pack(x.data_ptr(), x.stride(0), x.shape[0], H, idx.shape[1], idx.data_ptr(),
                                               send_pos.data_ptr(), E_local, 0, buf.data_ptr(), st,
                                               k3moe._stream()), "ep_pack")
        return buf

    def pack_rows(self, x, eid, dst):
        H = x.shape[1]
        k3moe._check(k3moe.lib().k3moe_ep_pack(x.data_ptr(), x.stride(0), x.shape[0], H, 1, None, None, 1, eid,
                                               dst.data_ptr(), dst.shape[1], k3moe._stream()), "ep_pack_rows")

    def ids(self, rows, R, H):
        ids = torch.empty((R, 1), dtype=torch.int32, device=rows.device)
        k3moe._check(k3moe.lib().k3moe_ep_ids(rows.data_ptr(), rows.shape[1], R, H, ids.data_ptr(),
                                              k3moe._stream()), "ep_ids")
        return ids

    def unpack(self, rows, R, H, tb):
        # rows past a tile's real rows are never read into a result: no need to clear either buffer
        qp = torch.empty((tb.cap_rows, H), dtype=torch.uint8, device=rows.device)
        sfp = torch.empty(tb.cap_rows * H // 32, dtype=torch.uint8, device=rows.device)
        k3moe._check(k3moe.lib().k3moe_ep_unpack(rows.data_ptr(), rows.shape[1], R, H, tb.exp2perm.data_ptr(),
                                                 qp.data_ptr(), sfp.data_ptr(), k3moe._stream()), "ep_unpack")
        return qp, sfp

    def pair_stride(self, H, K):
        return k3moe.lib().k3moe_ep_pair_row_stride(H, K)

    def pairs(self, dest, W):
        T, K = dest.shape
        out = torch.empty((T, W), dtype=torch.int32, device=dest.device)
        k3moe._check(k3moe.lib().k3moe_ep_pairs(dest.data_ptr(), T, K, W, out.data_ptr(), k3moe._stream()),
                     "ep_pairs")
        return out

    def pack_pairs(self, x, dest, lid, pair_pos, W, n_slots):
        H, K = x.shape[1], dest.shape[1]
        st = self.pair_stride(H, K)
        buf = torch.empty((max(n_slots, 1), st), dtype=torch.uint8, device=x.device)
        k3moe._check(k3moe.lib().k3moe_ep_pack_pairs(x.data_ptr(), x.stride(0), x.shape[0], H, K, dest.data_ptr(),
                                                     lid.data_ptr(), pair_pos.data_ptr(), W, 0, buf.data_ptr(), st,
                                                     k3moe._stream()), "ep_pack_pairs")
        return buf

    def pack_pair_rows(self, x, K, eid, dst):
        H = x.shape[1]
        k3moe._check(k3moe.lib().k3moe_ep_pack_pairs(x.data_ptr(), x.stride(0), x.shape[0], H, K, None, None, None, 1,
                                                     eid, dst.data_ptr(), dst.shape[1], k3moe._stream()),
                     "ep_pack_pair_rows")

    def ids_k(self, rows, R, H, K):
        ids = torch.empty((R, K), dtype=torch.int32, device=rows.device)
        k3moe._check(k3moe.lib().k3moe_ep_ids_k(rows.data_ptr(), rows.shape[1], R, H, K, ids.data_ptr(),
                                                k3moe._stream()), "ep_ids_k")
        return ids

    def unpack_k(self, rows, R, H, K, tb):
        qp = torch.empty((tb.cap_rows, H), dtype=torch.uint8, device=rows.device)
        sfp = torch.empty(tb.cap_rows * H // 32, dtype=torch.uint8, device=rows.device)
        k3moe._check(k3moe.lib().k3moe_ep_unpack_k(rows.data_ptr(), rows.shape[1], R, H, K, tb.exp2perm.data_ptr(),
                                                   qp.data_ptr(), sfp.data_ptr(), k3moe._stream()), "ep_unpack_k")
        return qp, sfp

    def return_rows(self, tb, R, K):
        out = torch.empty(tb.cap_rows, dtype=torch.int32, device=tb.exp2perm.device)
        k3moe._check(k3moe.lib().k3moe_ep_return_rows(tb.exp2perm.data_ptr(), R, K, out.data_ptr(),
                                                      k3moe._stream()), "ep_return_rows")
        return out

    def fc1(self, w, qp, sfp, tb, H, I, n_experts):
        return k3moe.fc1(w["w13"], w["w13_sf"], qp, sfp, tb, H, I, n_experts, self.err)

    def fc2_cols(self, w, f1q, f1sf, tb, H, I, n_experts, out_rows, out, col0, ncols, grid_cap=0):
        """FC2's output columns [col0, col0 + ncols) into `out` (row stride out.stride(0)), row out_rows[r]."""
        k3moe._check(k3moe.lib().k3moe_fc2_cols(
            w["w2"].data_ptr(), w["w2_sf"].data_ptr(), f1q.data_ptr(), f1sf.data_ptr(), tb.cta_batch.data_ptr(),
            tb.cta_limit.data_ptr(), tb.meta.data_ptr(), out_rows.data_ptr(), out.data_ptr(), out.stride(0), col0,
            ncols, H, I, n_experts, tb.cap_rows, tb.max_ctas, grid_cap, self.err.data_ptr(), k3moe._stream()),
            "fc2_cols")

    def side_stream(self):
        return torch.cuda.Stream(device=self.device)

    def after(self, side):
        """`side` waits for the work queued on the current stream so far."""
        side.wait_stream(torch.cuda.current_stream())

    def on(self, side):
        return torch.cuda.stream(side)

    def join(self, side, *tensors):
        """The current stream waits for `side`; `tensors` were used on it."""
        torch.cuda.current_stream().wait_stream(side)
        for t in tensors:
            t.record_stream(side)

    def combine_chunked(self, back, send_pos, wts, shared_rows, T, K, H):
        """combine() over results that came back as column chunks: back [C, rows, H/C], shared_rows [C, T, H/C]
        (a view) or None."""
        C, cc = back.shape[0], back.shape[2]
        out = torch.empty((T, H), dtype=torch.bfloat16, device=back.device)
        sp = shared_rows.data_ptr() if shared_rows is not None else None
        scs = shared_rows.stride(0) if shared_rows is not None else 0
        sld = shared_rows.stride(1) if shared_rows is not None else 0
        k3moe._check(k3moe.lib().k3moe_combine_ep_chunked(back.data_ptr(), back.stride(0), back.stride(1),
                                                          send_pos.data_ptr(), wts.data_ptr(), sp, scs, sld,
                                                          out.data_ptr(), H, T, K, H, cc, k3moe._stream()),
                     "combine_ep_chunked")
        return out

    def ffn(self, w, qp, sfp, tb, H, I, n_experts, n_rows, events=None, out_rows=None):
        """FC1 and FC2; FC2 stores permuted row r at row out_rows[r] (default: tb.route_map, the received row)."""
        if events:
            events["fc1"][0].record()
        f1q, f1sf = k3moe.fc1(w["w13"], w["w13_sf"], qp, sfp, tb, H, I, n_experts, self.err)
        if events:
            events["fc1"][1].record()
        rows = tb.route_map if out_rows is None else out_rows
        y = torch.empty((max(n_rows, 1), H), dtype=torch.bfloat16, device=qp.device)
        k3moe._check(k3moe.lib().k3moe_fc2_to_rows(
            w["w2"].data_ptr(), w["w2_sf"].data_ptr(), f1q.data_ptr(), f1sf.data_ptr(), tb.cta_batch.data_ptr(),
            tb.cta_limit.data_ptr(), tb.meta.data_ptr(), rows.data_ptr(), y.data_ptr(), H, I, n_experts,
            tb.cap_rows, tb.max_ctas, self.err.data_ptr(), k3moe._stream()), "fc2_to_rows")
        return y

    # ---- the peer-memory transport (k3moe_ep_pack_pairs_to / _row_ptrs / fc2_to_ptrs / _signal / _wait)
    def pack_pairs_to(self, x, dest, lid, pair_pos, W, row_base, stride):
        H, K = x.shape[1], dest.shape[1]
        rb = (ctypes.c_uint64 * W)(*row_base)
        k3moe._check(k3moe.lib().k3moe_ep_pack_pairs_to(x.data_ptr(), x.stride(0), x.shape[0], H, K, dest.data_ptr(),
                                                        lid.data_ptr(), pair_pos.data_ptr(), W,
                                                        ctypes.cast(rb, ctypes.c_void_p), stride, k3moe._stream()),
                     "ep_pack_pairs_to")

    def row_ptrs(self, tb, R, K, out_rows, block_base, block_start, row_bytes, sink):
        ptrs = torch.empty(tb.cap_rows, dtype=torch.int64, device=out_rows.device)
        nb = len(block_base)
        bb = (ctypes.c_uint64 * nb)(*block_base)
        bs = (ctypes.c_int64 * (nb + 1))(*block_start)
        k3moe._check(k3moe.lib().k3moe_ep_row_ptrs(tb.exp2perm.data_ptr(), R, K, out_rows.data_ptr(), nb,
                                                   ctypes.cast(bb, ctypes.c_void_p), ctypes.cast(bs, ctypes.c_void_p),
                                                   row_bytes, sink.data_ptr(), ptrs.data_ptr(), self.err.data_ptr(),
                                                   k3moe._stream()), "ep_row_ptrs")
        return ptrs

    def fc1_only(self, w, qp, sfp, tb, H, I, n_experts):
        return k3moe.fc1(w["w13"], w["w13_sf"], qp, sfp, tb, H, I, n_experts, self.err)

    def fc2_to_ptrs(self, w, f1q, f1sf, tb, H, I, n_experts, ptrs):
        k3moe._check(k3moe.lib().k3moe_fc2_to_ptrs(
            w["w2"].data_ptr(), w["w2_sf"].data_ptr(), f1q.data_ptr(), f1sf.data_ptr(), tb.cta_batch.data_ptr(),
            tb.cta_limit.data_ptr(), tb.meta.data_ptr(), ptrs.data_ptr(), H, I, n_experts, tb.cap_rows, tb.max_ctas,
            self.err.data_ptr(), k3moe._stream()), "fc2_to_ptrs")

    def signal(self, flag_bases, W, me, slot0, epoch):
        fb = (ctypes.c_uint64 * W)(*flag_bases)
        k3moe._check(k3moe.lib().k3moe_ep_signal(ctypes.cast(fb, ctypes.c_void_p), W, me, slot0, epoch,
                                                 k3moe._stream()), "ep_signal")

    def wait(self, flags, W, skip, epoch, budget_ns):
        k3moe._check(k3moe.lib().k3moe_ep_wait(flags.data_ptr(), W, skip, epoch, budget_ns, self.err.data_ptr(),
                                               k3moe._stream()), "ep_wait")

    def combine(self, back, send_pos, wts, shared_rows, T, K, H):
        out = torch.empty((T, H), dtype=torch.bfloat16, device=back.device)
        sp = shared_rows.data_ptr() if shared_rows is not None else None
        ld = shared_rows.stride(0) if shared_rows is not None else 0
        k3moe._check(k3moe.lib().k3moe_combine_ep(back.data_ptr(), send_pos.data_ptr(), wts.data_ptr(), sp, ld,
                                                  out.data_ptr(), H, T, K, H, k3moe._stream()), "combine_ep")
        return out


# the packing kernel writes id mod E_local for each pick; handed local ids already, this modulus keeps them
LOCAL_IDS = 1 << 30


def balanced_owner(bias, world):
    """An expert placement that evens the expected load: experts in decreasing router bias (the bias is what
    makes an expert popular) dealt to the ranks in snake order, E / world each."""
    order = torch.argsort(torch.as_tensor(bias, dtype=torch.float32).cpu(), descending=True, stable=True)
    owner = torch.empty(order.numel(), dtype=torch.int64)
    for i, e in enumerate(order.tolist()):
        rnd, pos = divmod(i, world)
        owner[e] = pos if rnd % 2 == 0 else world - 1 - pos
    return owner


def peer_offsets(C, me):
    """Where the peer-memory transport stores rows, for rank `me`, from C [W, W, 2] (C[s, d] = rows and picks
    rank s sends to rank d; every rank holds the same C).  The stores reproduce the two all-to-alls' layouts:
    received rows grouped by source rank, results returned grouped by the rank that computed them.
    - dispatch: my pair-plan slots for rank d start at sum_{d' < d} C[me, d'].rows and land in rank d's receive
      buffer from row sum_{s < me} C[s, d].rows: shift[d] = landing row - slot (slot p goes to row p + shift[d]);
    - I receive R_recv = sum_s C[s, me].rows rows and P_recv = sum_s C[s, me].picks picks (source s's from
      row sum_{s' < s}); my FC2 result q of source s (q in [pstart[s], pstart[s + 1])) goes to row
      back_row0[s] + (q - pstart[s]) of s's return buffer, back_row0[s] = sum_{d < me} C[s, d].picks;
    - recv_rows[d] / back_rows[d]: the rows rank d receives / gets back in all (capacity checks)."""
    C = [[(int(C[s][d][0]), int(C[s][d][1])) for d in range(len(C))] for s in range(len(C))]
    W = len(C)
    shift = []
    slot0 = 0
    for d in range(W):
        land = sum(C[s][d][0] for s in range(me))
        shift.append(land - slot0)
        slot0 += C[me][d][0]
    pstart = [0]
    for s in range(W):
        pstart.append(pstart[-1] + C[s][me][1])
    back_row0 = [sum(C[s][d][1] for d in range(me)) for s in range(W)]
    return {"shift": shift, "R_recv": sum(C[s][me][0] for s in range(W)), "P_recv": pstart[-1], "pstart": pstart,
            "back_row0": back_row0, "recv_rows": [sum(C[s][d][0] for s in range(W)) for d in range(W)],
            "back_rows": [sum(C[s][d][1] for d in range(W)) for s in range(W)]}


class PeerBuffers:
    """One rank's memory that its peers store into, mapped into every rank (CUDA IPC): the receive buffer of
    dispatched rows, the return buffer of FC2 results for this rank's picks, and 2W flag words (dispatch,
    combine).  One allocation a rank, exported once; every rank imports its peers' at set-up."""

    def __init__(self, W, rank, cap_rows, stride, back_rows, H, device, group=None):
        self.W, self.rank, self.stride, self.H = W, rank, stride, H
        self.cap_rows, self.back_cap = cap_rows, back_rows
        recv_bytes = cap_rows * stride
        self.back_off = -(-recv_bytes // 256) * 256
        self.flag_off = self.back_off + -(-(back_rows * H * 2) // 256) * 256
        total = self.flag_off + 256
        self.mem = torch.zeros(total, dtype=torch.uint8, device=device)
        self.recv = self.mem[:recv_bytes].view(cap_rows, stride)
        self.back = self.mem[self.back_off:self.back_off + back_rows * H * 2].view(torch.bfloat16).view(back_rows, H)
        self.flags = self.mem[self.flag_off:self.flag_off + 8 * W].view(torch.int32)
        handle = (ctypes.c_uint8 * 64)()
        off = ctypes.c_uint64()
        k3moe._check(k3moe.lib().k3moe_ipc_export(self.mem.data_ptr(), ctypes.cast(handle, ctypes.c_void_p),
                                                  ctypes.byref(off)), "ipc_export")
        torch.cuda.synchronize(device)
        mine = (bytes(handle), int(off.value))
        every = [None] * W
        dist.all_gather_object(every, mine, group=group)
        self.base = []   # every rank's allocation in this process's address space
        self._opened = []
        for s, (h, o) in enumerate(every):
            if s == rank:
                self.base.append(self.mem.data_ptr())
                continue
            hb = (ctypes.c_uint8 * 64).from_buffer_copy(h)
            p = ctypes.c_void_p()
            k3moe._check(k3moe.lib().k3moe_ipc_import(ctypes.cast(hb, ctypes.c_void_p), o, ctypes.byref(p)),
                         "ipc_import")
            self.base.append(int(p.value))
            self._opened.append((int(p.value), o))
        self.recv_addr = self.base
        self.back_addr = [b + self.back_off for b in self.base]
        self.flag_addr = [b + self.flag_off for b in self.base]

    def close(self):
        for p, o in self._opened:
            k3moe.lib().k3moe_ipc_release(ctypes.c_void_p(p), o)
        self._opened = []


class EPMoELayer:
    """One rank's part of an expert-parallel MoE layer.

    w: this rank's weights {w13, w13_sf, w2, w2_sf} holding its E_local routed experts (global ids
    [rank*E_local, (rank+1)*E_local)) and, with `shared`, the shared expert as local expert E_local.
    """

    def __init__(self, H, I, E, K, shared, w, bias, rs, group=None, ops=None, device=None, fixed_tokens=None,
                 owner=None, overlap_chunks=1, fc2_grid_cap=0, transport="nccl", max_tokens=None,
                 wait_budget_ns=5_000_000_000):
        """fixed_tokens: when set (at most that many tokens a call), every rank sends fixed-size blocks of
        fixed_tokens*K slots to every rank, empty slots marked by local expert id -1: no host
        synchronisation, so a whole step can be captured in a CUDA graph (decode-sized batches).
        owner: int [E], the rank holding each expert (E / world each; a rank's experts in increasing id order
        are its local experts 0, 1, ...; `w` holds them in that order).  None: contiguous blocks.
        overlap_chunks: C > 1 splits FC2 into C column slices (H / C a multiple of 256) and returns each slice's
        results with its own all-to-all on a side stream while the next slice computes; fc2_grid_cap then
        bounds FC2's persistent blocks (0: one an SM) to leave SMs to the collective.
        transport: "nccl" (the two all-to-alls) or "peer": the pack kernel and FC2's epilogue store rows straight
        into the receiving ranks' buffers over NVLink (CUDA IPC), flags mark each source done, and the waits
        for them are bounded by wait_budget_ns (a late source is recorded in the error words, ops.err).  The
        output is the same bytes.  "peer" needs max_tokens (tokens a rank, a call) for its fixed buffers."""
        if transport not in ("nccl", "peer"):
            raise ValueError(f"transport {transport!r}")
        if transport == "peer" and (fixed_tokens is not None or overlap_chunks != 1 or not max_tokens):
            raise ValueError("the peer transport takes the counts-exchange path, one FC2 pass, and max_tokens")
        self.transport, self.max_tokens, self.wait_budget_ns = transport, max_tokens, int(wait_budget_ns)
        self.peer = None
        self.epoch = 0
        self.fixed_tokens = fixed_tokens
        self.group = group
        self.rank = dist.get_rank(group)
        self.world = dist.get_world_size(group)
        if E % self.world:
            raise ValueError(f"{E} experts do not split over {self.world} ranks")
        if self.world > 16 and fixed_tokens is None:
            raise ValueError("the (token, rank) pair plan is a routing table of one column a rank: at most 16 ranks")
        self.H, self.I, self.E, self.K, self.shared = H, I, E, K, int(shared)
        self.E_local = E // self.world
        self.w, self.bias, self.rs = w, bias, rs
        self.owner_map = None
        if owner is not None:
            owner = torch.as_tensor(owner, dtype=torch.int64).cpu()
            if owner.numel() != E or torch.bincount(owner, minlength=self.world).tolist() != [self.E_local] * self.world:
                raise ValueError(f"owner must give each of {self.world} ranks {self.E_local} experts")
            local = torch.empty(E, dtype=torch.int64)
            for r in range(self.world):
                mine = (owner == r).nonzero().flatten()
                local[mine] = torch.arange(mine.numel())
            dev = bias.device
            self.owner_map = (owner.to(torch.int32).to(dev), local.to(torch.int32).to(dev))
        if overlap_chunks < 1 or H % (256 * overlap_chunks):
            raise ValueError(f"overlap_chunks {overlap_chunks} must cut H = {H} into multiples of 256")
        self.overlap_chunks, self.fc2_grid_cap = overlap_chunks, fc2_grid_cap
        self.ops = ops or GpuOps(device)
        self._side = None
        self.timing = None  # (dispatch_ms, combine_ms) of the last forward when events are given

    def _forward_peer(self, S, x, events=None):
        return _peer_forward(self, S, x, events)

    def close(self):
        """Unmap the peers' buffers (peer transport)."""
        if self.peer is not None:
            self.peer.close()
            self.peer = None

    def _route(self, idx):
        """(destination rank, local expert id at the destination) of every pick, int32 [T, K] each."""
        if self.owner_map is None:
            dest = torch.div(idx, self.E_local, rounding_mode="floor").to(torch.int32)
            return dest, idx - dest * self.E_local
        owner, local = self.owner_map
        flat = idx.reshape(-1).to(torch.int64)
        return owner[flat].reshape(idx.shape), local[flat].reshape(idx.shape)

    def _a2a(self, out, inp, out_rows, in_rows):
        """All-to-all of whole rows as bytes (every backend moves uint8); splits in rows."""
        ob = out.reshape(-1).view(torch.uint8)
        ib = inp.reshape(-1).view(torch.uint8)
        row_bytes = math.prod(out.shape[1:]) * out.element_size()
        dist.all_to_all_single(ob, ib, [r * row_bytes for r in out_rows], [r * row_bytes for r in in_rows],
                               group=self.group)

    def _forward_fixed(self, S, x, events=None):
        """forward() with fixed-size all-to-all blocks: cap = fixed_tokens * K slots a destination.
        events: optional {"dispatch", "ffn", "combine": (start, end)} CUDA events to record."""
        ops, H, K, El, W = self.ops, self.H, self.K, self.E_local, self.world
        T = x.shape[0]
        if T > self.fixed_tokens:
            raise ValueError(f"{T} tokens exceed fixed_tokens={self.fixed_tokens}")
        cap = self.fixed_tokens * K
        idx, wts = ops.topk(S, self.bias, self.rs, K)
        dest, lid = self._route(idx)
        plan = ops.tables(dest.reshape(-1, 1).contiguous(), W, 1)
        counts = plan.counts[:W]
        first = (torch.cumsum(counts, 0, dtype=torch.int32) - counts).to(torch.int64)
        d = dest.reshape(-1).to(torch.int64)
        # slot of pick (t, k): its destination's block, then its rank among that destination's picks
        slot = (d * cap + plan.exp2perm.reshape(-1).to(torch.int64) - first[d]).to(torch.int32).reshape(T, K)
        stride = ops.stride(H)
        n_slots = W * cap
        send = torch.empty((n_slots, stride), dtype=torch.uint8, device=x.device)
        eid_col = H + H // 32
        send[:, eid_col:eid_col + 4].view(torch.int32).fill_(-1)  # empty slots: no expert
        ops.pack(x, lid.contiguous(), slot, LOCAL_IDS, n_slots, out=send)
        R = n_slots + (T if self.shared else 0)
        recv = torch.empty((R, stride), dtype=torch.uint8, device=x.device)
        if events:
            events["dispatch"][0].record()
        dist.all_to_all_single(recv[:n_slots].reshape(-1), send.reshape(-1), group=self.group)
        if events:
            events["dispatch"][1].record()
            events["ffn"][0].record()
        if self.shared:
            ops.pack_rows(x, El, recv[n_slots:R])
        ids = ops.ids(recv, R, H)
        tb = ops.tables(ids, El + self.shared, 128)
        qp, sfp = ops.unpack(recv, R, H, tb)
        y = ops.ffn(self.w, qp, sfp, tb, H, self.I, El + self.shared, R)
        back = torch.empty((n_slots, H), dtype=y.dtype, device=y.device)
        if events:
            events["ffn"][1].record()
            events["combine"][0].record()
        dist.all_to_all_single(back.reshape(-1).view(torch.uint8), y[:n_slots].reshape(-1).view(torch.uint8),
                               group=self.group)
        if events:
            events["combine"][1].record()
        self.last = {"received_rows": None, "sent_rows": T * K, "tables": tb}
        shared_rows = y[n_slots:R] if self.shared else None
        return ops.combine(back, slot, wts, shared_rows, T, K, H)

    def forward(self, S, x, events=None):
        """events: optional {"dispatch", "fc1", "combine": (start, end)} CUDA events to record (fixed-block
        mode: "dispatch", "ffn", "combine")."""
        if self.fixed_tokens is not None:
            return self._forward_fixed(S, x, events)
        if self.transport == "peer":
            return self._forward_peer(S, x, events)
        ops, H, K, El, W = self.ops, self.H, self.K, self.E_local, self.world
        T = x.shape[0]
        idx, wts = ops.topk(S, self.bias, self.rs, K)
        dest, lid = self._route(idx)
        # the picks' plan: every pick's row in the returned results (grouped by rank, (token, k) order within
        # one) for the combine, and the picks a rank gets
        plan = ops.tables(dest.reshape(-1, 1).contiguous(), W, 1)
        send_pos = plan.exp2perm.reshape(T, K)          # [T, K] return row of each pick
        pick_counts = plan.counts[:W].to(torch.int64)
        # the rows' plan: a token travels once to each rank holding any of its picks (token order within a rank)
        pairs = ops.pairs(dest.contiguous(), W)
        rplan = ops.tables(pairs, W, 1)
        row_counts = rplan.counts[:W].to(torch.int64)
        send = ops.pack_pairs(x, dest.contiguous(), lid.contiguous(), rplan.exp2perm.reshape(T, W), W,
                              T * min(W, K))
        counts = torch.stack([row_counts, pick_counts], 1).contiguous()  # [W, 2]: rows, picks to each rank
        recv_counts = torch.empty_like(counts)
        self._a2a(recv_counts, counts, [1] * W, [1] * W)
        sc_rows, sc_picks = (counts[:, 0].tolist(), counts[:, 1].tolist())
        rc = recv_counts.tolist()
        rc_rows, rc_picks = [r[0] for r in rc], [r[1] for r in rc]
        R_recv, P_recv = sum(rc_rows), sum(rc_picks)
        R_all, P_all = R_recv + (T if self.shared else 0), P_recv + (T if self.shared else 0)
        stride = send.shape[1]
        recv = torch.empty((max(R_all, 1), stride), dtype=torch.uint8, device=send.device)
        if events:
            events["dispatch"][0].record()
        self._a2a(recv[:R_recv], send[:sum(sc_rows)], rc_rows, sc_rows)
        if events:
            events["dispatch"][1].record()
        if self.shared:
            ops.pack_pair_rows(x, K, El, recv[R_recv:R_all])
        ids = ops.ids_k(recv, R_all, H, K)               # [R_all, K] local ids of each row's picks
        tb = ops.tables(ids, El + self.shared, 128)
        qp, sfp = ops.unpack_k(recv, R_all, H, K, tb)
        out_rows = ops.return_rows(tb, R_all, K)         # results in (row, pick) order: returned picks, shared
        self.last = {"received_rows": R_recv, "received_picks": P_recv, "sent_rows": sum(sc_rows),
                     "sent_picks": T * K, "tables": tb}
        C = self.overlap_chunks
        if C == 1:
            y = ops.ffn(self.w, qp, sfp, tb, H, self.I, El + self.shared, P_all, events, out_rows=out_rows)
            back = torch.empty((T * K, H), dtype=y.dtype, device=y.device)
            if events:
                events["combine"][0].record()
            self._a2a(back, y[:P_recv], sc_picks, rc_picks)
            if events:
                events["combine"][1].record()
            shared_rows = y[P_recv:P_all] if self.shared else None
            return ops.combine(back, send_pos, wts, shared_rows, T, K, H)
        # FC2 in C column slices; each slice's results go back on a side stream while the next one computes
        if events:
            events["fc1"][0].record()
        f1q, f1sf = ops.fc1(self.w, qp, sfp, tb, H, self.I, El + self.shared)
        if events:
            events["fc1"][1].record()
        cc = H // C
        y = torch.empty((C, max(P_all, 1), cc), dtype=torch.bfloat16, device=qp.device)
        back = torch.empty((C, T * K, cc), dtype=torch.bfloat16, device=qp.device)
        if self._side is None:
            self._side = ops.side_stream()
        side = self._side
        for j in range(C):
            ops.fc2_cols(self.w, f1q, f1sf, tb, H, self.I, El + self.shared, out_rows, y[j], j * cc, cc,
                         self.fc2_grid_cap)
            ops.after(side)
            with ops.on(side):
                if events and j == 0:
                    events["combine"][0].record()
                self._a2a(back[j], y[j, :P_recv], sc_picks, rc_picks)
                if events and j == C - 1:
                    events["combine"][1].record()
        ops.join(side, y, back)
        shared_rows = y[:, P_recv:P_all] if self.shared else None
        return ops.combine_chunked(back, send_pos, wts, shared_rows, T, K, H)


def _peer_forward(layer, S, x, events=None):
    """EPMoELayer.forward over peer memory (transport "peer"); see the class."""
    ops, H, K, El, W, me = layer.ops, layer.H, layer.K, layer.E_local, layer.world, layer.rank
    T = x.shape[0]
    if T > layer.max_tokens:
        raise ValueError(f"{T} tokens exceed max_tokens={layer.max_tokens}")
    stride = ops.pair_stride(H, K)
    if layer.peer is None:
        layer.peer = PeerBuffers(W, me, W * layer.max_tokens + layer.max_tokens, stride, layer.max_tokens * K, H,
                                 x.device, layer.group)
        layer.shared_out = torch.empty((layer.max_tokens + 1, H), dtype=torch.bfloat16, device=x.device)
    pb = layer.peer
    layer.epoch = (layer.epoch + 1) & 0x7FFFFFFF
    epoch = layer.epoch
    idx, wts = ops.topk(S, layer.bias, layer.rs, K)
    dest, lid = layer._route(idx)
    plan = ops.tables(dest.reshape(-1, 1).contiguous(), W, 1)
    send_pos = plan.exp2perm.reshape(T, K)
    pairs = ops.pairs(dest.contiguous(), W)
    rplan = ops.tables(pairs, W, 1)
    counts = torch.stack([rplan.counts[:W], plan.counts[:W]], 1).to(torch.int32).contiguous()  # [W, 2]
    every = torch.empty((W, W, 2), dtype=torch.int32, device=x.device)
    dist.all_gather_into_tensor(every, counts, group=layer.group)
    C = every.tolist()  # the one host synchronisation
    lay = peer_offsets(C, me)
    if max(lay["recv_rows"]) + layer.max_tokens > pb.cap_rows or max(lay["back_rows"]) > pb.back_cap:
        raise ValueError("peer buffers too small for this step's routing")
    R_recv, P_recv = lay["R_recv"], lay["P_recv"]
    R_all, P_all = R_recv + (T if layer.shared else 0), P_recv + (T if layer.shared else 0)
    row_base = [pb.recv_addr[d] + lay["shift"][d] * stride for d in range(W)]
    if events:
        events["dispatch"][0].record()
    ops.pack_pairs_to(x, dest.contiguous(), lid.contiguous(), rplan.exp2perm.reshape(T, W), W, row_base, stride)
    ops.signal(pb.flag_addr, W, me, 0, epoch)
    ops.wait(pb.flags[:W], W, me, epoch, layer.wait_budget_ns)
    if events:
        events["dispatch"][1].record()
    recv = pb.recv[:max(R_all, 1)]
    if layer.shared:
        ops.pack_pair_rows(x, K, El, recv[R_recv:R_all])
    ids = ops.ids_k(recv, R_all, H, K)
    tb = ops.tables(ids, El + layer.shared, 128)
    qp, sfp = ops.unpack_k(recv, R_all, H, K, tb)
    out_rows = ops.return_rows(tb, R_all, K)
    layer.last = {"received_rows": R_recv, "received_picks": P_recv, "sent_rows": sum(c[0] for c in C[me]),
                  "sent_picks": T * K, "tables": tb}
    if events:
        events["fc1"][0].record()
    f1q, f1sf = ops.fc1_only(layer.w, qp, sfp, tb, H, layer.I, El + layer.shared)
    if events:
        events["fc1"][1].record()
    row_bytes = H * 2
    block_base = [pb.back_addr[s] + lay["back_row0"][s] * row_bytes for s in range(W)]
    block_start = list(lay["pstart"])
    if layer.shared:
        block_base.append(layer.shared_out.data_ptr())
        block_start.append(P_all)
    sink = layer.shared_out[layer.max_tokens]
    ptrs = ops.row_ptrs(tb, R_all, K, out_rows, block_base, block_start, row_bytes, sink)
    ops.fc2_to_ptrs(layer.w, f1q, f1sf, tb, H, layer.I, El + layer.shared, ptrs)
    if events:
        events["combine"][0].record()
    ops.signal(pb.flag_addr, W, me, W, epoch)
    ops.wait(pb.flags[W:2 * W], W, me, epoch, layer.wait_budget_ns)
    if events:
        events["combine"][1].record()
    shared_rows = layer.shared_out[:T] if layer.shared else None
    return ops.combine(pb.back[:T * K], send_pos, wts, shared_rows, T, K, H)


class DeviceEPMoELayer:
    """One rank's part of the expert-parallel layer as one device-resident C-ABI step (k3moe_ep_forward).

    Every rank allocates one peer buffer (k3moe_ep_peer_bytes) that the others map through CUDA IPC: a fixed
    region of max_tokens rows a source rank, so no rank needs another's counts before it sends and the step
    never synchronises with the host; the pack kernel stores rows straight into the destinations' regions and
    FC2's epilogue stores each result into its owner's return buffer.  w: this rank's weights as for
    EPMoELayer (slice_weights); owner: as for EPMoELayer (None: contiguous blocks).  With world 1 no process
    group is needed.  forward() may be captured in a CUDA graph (the same T, buffers and stream)."""

    def __init__(self, H, I, E, K, shared, w, bias, rs, max_tokens, group=None, owner=None, activation=0,
                 wait_budget_ns=5_000_000_000, device=None):
        self.group = group
        distributed = dist.is_available() and dist.is_initialized()
        self.rank = dist.get_rank(group) if distributed else 0
        self.world = dist.get_world_size(group) if distributed else 1
        self.H, self.I, self.E, self.K, self.shared = H, I, E, K, int(shared)
        self.max_tokens = int(max_tokens)
        self.w, self.bias, self.rs = w, bias, rs
        dev = torch.device(device) if device is not None else w["w13"].device
        cfg = k3moe.k3moe_ep_config(self.world, self.rank, H, I, E, K, self.shared, self.max_tokens, int(activation),
                                    int(wait_budget_ns))
        self.cfg = cfg
        L = k3moe.lib()
        pbytes = L.k3moe_ep_peer_bytes(ctypes.byref(cfg))
        wbytes = L.k3moe_ep_workspace_bytes(ctypes.byref(cfg))
        if pbytes == 0 or wbytes == 0:
            raise ValueError(f"unsupported expert-parallel configuration {self.world} ranks, E={E}, K={K}, "
                             f"max_tokens={max_tokens}")
        self.peer = torch.zeros(pbytes, dtype=torch.uint8, device=dev)
        self.ws = torch.empty(wbytes, dtype=torch.uint8, device=dev)
        self._opened = []
        bases = [0] * self.world
        bases[self.rank] = self.peer.data_ptr()
        if self.world > 1:
            handle = (ctypes.c_uint8 * 64)()
            off = ctypes.c_uint64()
            k3moe._check(L.k3moe_ipc_export(self.peer.data_ptr(), ctypes.cast(handle, ctypes.c_void_p),
                                            ctypes.byref(off)), "ipc_export")
            torch.cuda.synchronize(dev)
            every = [None] * self.world
            dist.all_gather_object(every, (bytes(handle), int(off.value)), group=group)
            for s, (h, o) in enumerate(every):
                if s == self.rank:
                    continue
                hb = (ctypes.c_uint8 * 64).from_buffer_copy(h)
                p = ctypes.c_void_p()
                k3moe._check(L.k3moe_ipc_import(ctypes.cast(hb, ctypes.c_void_p), o, ctypes.byref(p)), "ipc_import")
                bases[s] = int(p.value)
                self._opened.append((int(p.value), o))
        base_arr = (ctypes.c_uint64 * self.world)(*bases)
        own = None
        if owner is not None:
            own = (ctypes.c_int32 * E)(*[int(v) for v in torch.as_tensor(owner).cpu().tolist()])
        handle = ctypes.c_void_p()
        k3moe._check(L.k3moe_ep_create(ctypes.byref(cfg), own, k3moe._p(w["w13"]), k3moe._p(w["w13_sf"]),
                                       k3moe._p(w["w2"]), k3moe._p(w["w2_sf"]), self.peer.data_ptr(),
                                       ctypes.cast(base_arr, ctypes.c_void_p), self.ws.data_ptr(), wbytes,
                                       k3moe._stream(), ctypes.byref(handle)), "ep_create")
        self.handle = handle
        torch.cuda.synchronize(dev)
        if self.world > 1:
            dist.barrier(group=group)  # every rank's flags cleared before any rank's first step
        self.timing = None

    def forward(self, S, x, out=None, events=None):
        """out bf16 [T, H] (allocated when None).  events: optional list of up to 8 CUDA events recorded at the
        step's stage boundaries (k3moe_ep_forward_events)."""
        T = x.shape[0]
        if out is None:
            out = torch.empty((T, self.H), dtype=torch.bfloat16, device=x.device)
        L = k3moe.lib()
        if events:
            for e in events:  # torch creates events lazily: record once so each has a CUDA event
                e.record()
            arr = (ctypes.c_void_p * len(events))(*[e.cuda_event for e in events])
            rc = L.k3moe_ep_forward_events(self.handle, k3moe._p(S), S.stride(0), k3moe._p(self.bias),
                                           k3moe._p(self.rs), k3moe._p(x), x.stride(0), T, k3moe._p(out),
                                           out.stride(0), k3moe._stream(), ctypes.cast(arr, ctypes.c_void_p),
                                           len(events))
        else:
            rc = L.k3moe_ep_forward(self.handle, k3moe._p(S), S.stride(0), k3moe._p(self.bias), k3moe._p(self.rs),
                                    k3moe._p(x), x.stride(0), T, k3moe._p(out), out.stride(0), k3moe._stream())
        k3moe._check(rc, "ep_forward")
        return out

    def error_words(self):
        """The step's two device error words (synchronises; clears them)."""
        L = k3moe.lib()
        words = (ctypes.c_uint32 * 2)()
        rc = L.k3moe_read_error(L.k3moe_ep_errors(self.handle), ctypes.cast(words, ctypes.c_void_p), 1,
                                k3moe._stream())
        return rc, (int(words[0]), int(words[1]))

    def received_counts(self):
        """Rows each source sent this rank in the last step, then this rank's shared rows (host list)."""
        n = self.world + 1
        ptr = k3moe.lib().k3moe_ep_counts(self.handle)
        off = ptr - self.peer.data_ptr()
        return self.peer[off:off + 4 * n].view(torch.int32).tolist()

    def expert_rows(self):
        """Rows the last step routed to each local expert (the routed experts, then the shared one): a tensor."""
        n = self.E // self.world + self.shared
        off = k3moe.lib().k3moe_ep_expert_rows(self.handle) - self.ws.data_ptr()
        return self.ws[off:off + 4 * n].view(torch.int32).clone()

    def close(self):
        """Unmap the peers' buffers and free the host object (after every rank's last step)."""
        L = k3moe.lib()
        for p, o in self._opened:
            L.k3moe_ipc_release(ctypes.c_void_p(p), o)
        self._opened = []
        if self.handle:
            L.k3moe_ep_destroy(self.handle)
            self.handle = None


def slice_weights(w13, w13_sf, w2, w2_sf, E, shared, rank, world, H, I, owner=None):
    """This rank's experts (and the shared expert, stored last) out of full tile-major weight tensors
    laid out as k3moe_layer_forward expects (experts back to back, the shared expert after the routed):
    experts [rank E/world, (rank+1) E/world), or with `owner` the experts it gives this rank, in id order."""
    El = E // world
    mine = (list(range(rank * El, (rank + 1) * El)) if owner is None else
            (torch.as_tensor(owner) == rank).nonzero().flatten().tolist())

    def rows(t):  # the bytes of this rank's experts, then the shared expert's
        per_b = t.numel() // (E + shared)
        flat = t.reshape(-1)
        parts = [flat[e * per_b:(e + 1) * per_b] for e in mine]
        if shared:
            parts.append(flat[E * per_b:(E + 1) * per_b])
        return torch.cat(parts)

    return {"w13": rows(w13), "w13_sf": rows(w13_sf), "w2": rows(w2), "w2_sf": rows(w2_sf)}
