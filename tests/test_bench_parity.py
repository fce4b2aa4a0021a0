"""The benchmark's in-run parity leg (bench.inrun_parity) on the CPU: a workspace laid out by the library's own
offsets and filled with the CPU restatement's intermediates must pass every check, and a planted mistake (one
FC2 row, one E4M3 byte of FC1's output) must fail the check it belongs to."""
import os
import sys

import numpy as np
import pytest
import torch

import cases
import k3moe
import oracle

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)
import bench  # noqa: E402


class FakeLayer:
    """What inrun_parity reads of k3moe.MoELayer: dims, offsets() and the workspace (here on the CPU)."""

    def __init__(self, c, inter):
        self.H, self.I, self.E, self.K, self.shared = c.H, c.I, c.E, c.K, c.shared
        self.ws_bytes = k3moe.lib().k3moe_layer_workspace_size(c.T, c.H, c.I, c.E, c.K, c.shared)
        ws = np.zeros(self.ws_bytes, np.uint8)
        self._T = c.T
        off = self.offsets(c.T)
        tb = inter["tables"]

        def put(name, arr):
            b = np.ascontiguousarray(arr).view(np.uint8).reshape(-1)
            ws[off[name]:off[name] + b.size] = b

        put("idx", inter["idx"])
        put("wts", inter["wts"])
        put("counts", tb["counts"])
        put("cta_batch", tb["cta_batch"])
        put("cta_limit", tb["cta_limit"])
        put("meta", tb["meta"])
        put("route_map", tb["route_map"])
        put("exp2perm", tb["exp2perm"])
        put("q_perm", inter["q_perm"])
        put("sf_perm", inter["sf_perm"])
        put("fc1_q", inter["fc1_q"])
        put("fc1_sf", inter["fc1_sf"])
        put("fc2", inter["fc2"])
        self.ws = torch.from_numpy(ws)

    def offsets(self, T=None):
        import ctypes

        arr = (ctypes.c_size_t * 14)()
        k3moe._check(k3moe.lib().k3moe_layer_workspace_offsets(T or self._T, self.H, self.I, self.E, self.K,
                                                              self.shared, ctypes.cast(arr, ctypes.c_void_p)), "off")
        return dict(zip(k3moe.OFFSET_NAMES, list(arr)))


def _case():
    c = cases.make_case(T=200, H=1024, I=512, E=16, K=4, shared=1, rs=2.5, seed=11)
    out, inter = cases.oracle_forward(c)
    host = {"x_bits": c.x_bits, "S": c.S, "bias": c.bias, "rs_bits": c.rs_bits}
    w = {k: torch.from_numpy(np.ascontiguousarray(getattr(c, k))) for k in ("w13", "w13_sf", "w2", "w2_sf")}
    return c, out, inter, host, w


def test_parity_leg_passes_on_the_oracles_own_intermediates():
    c, out, inter, host, w = _case()
    layer = FakeLayer(c, inter)
    nne = int(inter["tables"]["meta"][0])
    res, _, _ = bench.inrun_parity(layer, host, w, torch.from_numpy(out.view(np.int16)), c.T, c.E,
                                   bench.sample_tiles_of(nne, 4), n_tokens=16)
    assert res["ok"], res
    assert res["fc1"]["rel_l2"] == 0.0 and res["fc2"]["rel_l2"] == 0.0


@pytest.mark.parametrize("plant", ["fc2_row", "fc1_byte", "combine_row"])
def test_parity_leg_catches_a_planted_mistake(plant):
    c, out, inter, host, w = _case()
    nne = int(inter["tables"]["meta"][0])
    tiles = bench.sample_tiles_of(nne, 4)
    if plant == "fc2_row":  # a sampled tile's first row of FC2 output scaled by 2
        r = tiles[0] * 128
        inter["fc2"][r] = oracle.bf16_bits(oracle.bf16_to_f32(inter["fc2"][r]) * 2)
    elif plant == "fc1_byte":  # every E4M3 byte of a sampled tile's first FC1 row flipped in sign
        for kt in range(c.I // 128):
            off = (tiles[0] * (c.I // 128) + kt) * 16384
            inter["fc1_q"].reshape(-1)[off:off + 128] ^= 0x80
    else:  # one token's combined output row changed
        out = out.copy()
        out[0] ^= 0x0100
    layer = FakeLayer(c, inter)
    res, _, _ = bench.inrun_parity(layer, host, w, torch.from_numpy(out.view(np.int16)), c.T, c.E, tiles,
                                   n_tokens=16)
    assert not res["ok"]
    key = {"fc2_row": "fc2", "fc1_byte": "fc1"}.get(plant)
    if key:
        assert not res[key]["ok"], res[key]
    else:
        assert not res["combine_tokens_equal"]
