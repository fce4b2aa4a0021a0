"""The expert-parallel layer's steps on the CPU, made of the oracle — test
infrastructure: with these, k3moe_ep.EPMoELayer's host logic (send plan,
counts exchange, dispatch / combine all-to-all, receive layout) runs under
gloo ranks on a machine without a GPU."""
from __future__ import annotations

from types import SimpleNamespace

import numpy as np
import torch

import oracle


def _np(t):
    return t.detach().cpu().numpy()


def _bits(t):  # bf16 tensor -> uint16 bit array
    return _np(t.view(torch.int16)).view(np.uint16)


def _bf16(bits):
    return torch.from_numpy(np.ascontiguousarray(bits).view(np.int16)).view(torch.bfloat16)


class OracleOps:
    def topk(self, S, bias, rs, K):
        idx, wts = oracle.topk(_np(S), _np(bias), int(_bits(rs)[0]), K)
        return torch.from_numpy(idx), torch.from_numpy(wts)

    def tables(self, ids, E, tile):
        tb = oracle.tables(_np(ids), E, 0, 0, tile)
        return SimpleNamespace(counts=torch.from_numpy(tb["counts"]), exp2perm=torch.from_numpy(tb["exp2perm"]),
                               route_map=torch.from_numpy(tb["route_map"]), cta_batch=tb["cta_batch"],
                               cta_limit=tb["cta_limit"], meta=tb["meta"], cap_rows=tb["cap_rows"],
                               max_ctas=tb["max_ctas"])

    @staticmethod
    def stride(H):
        return (H + H // 32 + 4 + 15) // 16 * 16

    def _rows(self, x):
        q, sf = oracle.quant_mxfp8(_bits(x), tiled=False)
        return q, sf

    def pack(self, x, idx, send_pos, E_local, n_slots, out=None):
        H = x.shape[1]
        q, sf = self._rows(x)
        buf = np.zeros((n_slots, self.stride(H)), np.uint8) if out is None else _np(out)
        idx, pos = _np(idx), _np(send_pos)
        for t in range(idx.shape[0]):
            for k in range(idx.shape[1]):
                p = pos[t, k]
                buf[p, :H] = q[t]
                buf[p, H:H + H // 32] = sf[t]
                buf[p, H + H // 32:H + H // 32 + 4] = np.array([idx[t, k] % E_local], np.int32).view(np.uint8)
        return torch.from_numpy(buf) if out is None else out

    def pack_rows(self, x, eid, dst):
        H = x.shape[1]
        q, sf = self._rows(x)
        d = _np(dst)
        d[:, :H] = q
        d[:, H:H + H // 32] = sf
        d[:, H + H // 32:H + H // 32 + 4] = np.full((q.shape[0], 1), eid, np.int32).view(np.uint8)

    def ids(self, rows, R, H):
        r = _np(rows)[:R, H + H // 32:H + H // 32 + 4].copy()
        return torch.from_numpy(r.view(np.int32).reshape(R, 1))

    def unpack(self, rows, R, H, tb):
        r = _np(rows)
        perm = _np(tb.exp2perm).reshape(-1)
        qp = np.zeros(tb.cap_rows * H, np.uint8)
        sfp = np.zeros(tb.cap_rows * H // 32, np.uint8)
        kg4 = H // 128
        k = np.arange(H)
        kb = np.arange(H // 32)
        for i in range(R):
            p = int(perm[i])
            if p < 0:
                continue
            qp[((p // 128) * (H // 128) + k // 128) * 16384 + (p % 128) * 128 + k % 128] = r[i, :H]
            sfp[((p // 128) * kg4 + kb // 4) * 512 + (p % 32) * 16 + ((p % 128) // 32) * 4 + kb % 4] = r[i, H:H + H // 32]
        return qp.reshape(tb.cap_rows, H), sfp

    @staticmethod
    def pair_stride(H, K):
        return (H + H // 32 + 2 * K + 15) // 16 * 16

    def pairs(self, dest, W):
        d = _np(dest)
        out = np.full((d.shape[0], W), -1, np.int32)
        for t in range(d.shape[0]):
            for r in set(d[t].tolist()):
                out[t, r] = r
        return torch.from_numpy(out)

    def _pair_row(self, buf, p, q, sf, ids, K):
        H = q.shape[0]
        buf[p, :H] = q
        buf[p, H:H + H // 32] = sf
        hdr = np.full(K, -1, np.int16)
        hdr[:len(ids)] = ids
        buf[p, H + H // 32:H + H // 32 + 2 * K] = hdr.view(np.uint8)

    def pack_pairs(self, x, dest, lid, pair_pos, W, n_slots):
        H, K = x.shape[1], dest.shape[1]
        q, sf = self._rows(x)
        buf = np.zeros((max(n_slots, 1), self.pair_stride(H, K)), np.uint8)
        d, l, pp = _np(dest), _np(lid), _np(pair_pos)
        for t in range(d.shape[0]):
            for r in range(W):
                if pp[t, r] >= 0:
                    self._pair_row(buf, pp[t, r], q[t], sf[t], [l[t, k] for k in range(K) if d[t, k] == r], K)
        return torch.from_numpy(buf)

    def pack_pair_rows(self, x, K, eid, dst):
        q, sf = self._rows(x)
        d = _np(dst)
        for t in range(q.shape[0]):
            self._pair_row(d, t, q[t], sf[t], [eid], K)

    def ids_k(self, rows, R, H, K):
        r = _np(rows)[:R, H + H // 32:H + H // 32 + 2 * K].copy()
        return torch.from_numpy(r.view(np.int16).astype(np.int32).reshape(R, K))

    def unpack_k(self, rows, R, H, K, tb):
        r = _np(rows)
        perm = _np(tb.exp2perm).reshape(R, K)
        qp = np.zeros(tb.cap_rows * H, np.uint8)
        sfp = np.zeros(tb.cap_rows * H // 32, np.uint8)
        kg4 = H // 128
        k = np.arange(H)
        kb = np.arange(H // 32)
        for i in range(R):
            for j in range(K):
                p = int(perm[i, j])
                if p < 0:
                    continue
                qp[((p // 128) * (H // 128) + k // 128) * 16384 + (p % 128) * 128 + k % 128] = r[i, :H]
                sfp[((p // 128) * kg4 + kb // 4) * 512 + (p % 32) * 16 + ((p % 128) // 32) * 4 + kb % 4] = \
                    r[i, H:H + H // 32]
        return qp.reshape(tb.cap_rows, H), sfp

    def return_rows(self, tb, R, K):
        perm = _np(tb.exp2perm).reshape(R, K)
        out = np.full(tb.cap_rows, -1, np.int32)
        n = 0
        for i in range(R):
            for j in range(K):
                if perm[i, j] >= 0:
                    out[perm[i, j]] = n
                    n += 1
        return torch.from_numpy(out)

    def ffn(self, w, qp, sfp, tb, H, I, n_experts, n_rows, events=None, out_rows=None):
        nne = int(tb.meta[0])
        wn = {k: _np(v) for k, v in w.items()}
        f1q, f1sf = oracle.fc1(wn["w13"], wn["w13_sf"], qp, sfp, tb.cta_batch, tb.cta_limit, 0, nne, H, I)
        yp = oracle.fc2(wn["w2"], wn["w2_sf"], f1q, f1sf, tb.cta_batch, tb.cta_limit, 0, nne, H, I)
        y = np.zeros((max(n_rows, 1), H), np.uint16)
        rmap = _np(tb.route_map if out_rows is None else out_rows)
        for c in range(nne):
            for r in range(c * 128, int(tb.cta_limit[c])):
                y[rmap[r]] = yp[r]
        return _bf16(y)

    def fc1(self, w, qp, sfp, tb, H, I, n_experts):
        nne = int(tb.meta[0])
        wn = {k: _np(v) for k, v in w.items()}
        return oracle.fc1(wn["w13"], wn["w13_sf"], qp, sfp, tb.cta_batch, tb.cta_limit, 0, nne, H, I)

    def fc2_cols(self, w, f1q, f1sf, tb, H, I, n_experts, out_rows, out, col0, ncols, grid_cap=0):
        nne = int(tb.meta[0])
        wn = {k: _np(v) for k, v in w.items()}
        yp = oracle.fc2(wn["w2"], wn["w2_sf"], f1q, f1sf, tb.cta_batch, tb.cta_limit, 0, nne, H, I)
        o = _bits(out)  # a view: writes land in `out`
        rmap = _np(out_rows)
        for c in range(nne):
            for r in range(c * 128, int(tb.cta_limit[c])):
                o[rmap[r]] = yp[r, col0:col0 + ncols]

    # no streams on the CPU: the side stream is the main one
    def side_stream(self):
        return None

    def after(self, side):
        pass

    def on(self, side):
        import contextlib

        return contextlib.nullcontext()

    def join(self, side, *tensors):
        pass

    def combine_chunked(self, back, send_pos, wts, shared_rows, T, K, H):
        whole = torch.cat(list(back), dim=1)  # [rows, H]: the chunks side by side again
        sh = torch.cat(list(shared_rows), dim=1) if shared_rows is not None else None
        return self.combine(whole, send_pos, wts, sh, T, K, H)

    def combine(self, back, send_pos, wts, shared_rows, T, K, H):
        fc2 = _bits(back)
        meta = None
        if shared_rows is not None:
            fc2 = np.concatenate([fc2, _bits(shared_rows)])
            meta = np.array([0, 0, back.shape[0], 0], np.int32)  # the shared rows follow every returned row
        out = oracle.combine(fc2, _np(send_pos), _np(wts), meta, T, K)
        return _bf16(out)
