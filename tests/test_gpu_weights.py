"""Load-time re-layout of a checkpoint's MXFP4 expert tensors (k3moe_import_mxfp4 and its module entries
kern_k3_moe_w_tiles / kern_k3_moe_sf_tiles) against the layout the grouped GEMMs read.

The checkpoint binds each expert's `weight_packed` rows (E2M1 two a byte, element 2i in the low nibble) and
`weight_scale` bytes (UE8M0 per 32 along K) row-major, FC1 as [w3 (up); w1 (gate)]
(scripts/gen_stage.py:681-702 of the reference).  The test makes that form on the host from the device
quantiser's own output (tile-major [gate; up], tiled scales), imports it on the device, and requires the
original bytes back: the re-layout is a byte permutation, so parity is exact."""
import numpy as np
import pytest
import torch

import k3moe

pytestmark = pytest.mark.gpu


def untile_packed(p, rows, K):
    """Tile-major packed E2M1 (128 x 128-element tiles of 64-byte rows) -> row-major [rows, K/2]."""
    return np.ascontiguousarray(p.reshape(rows // 128, K // 128, 128, 64).transpose(0, 2, 1, 3).reshape(rows, K // 2))


def untile_scales(s, rows, K):
    """128x4-tiled scales over the rows -> row-major [rows, K/32]."""
    kbn, kg4 = K // 32, K // 128
    r = np.arange(rows, dtype=np.int64)[:, None]
    kb = np.arange(kbn, dtype=np.int64)[None, :]
    off = ((r // 128) * kg4 + kb // 4) * 512 + (r % 32) * 16 + ((r % 128) // 32) * 4 + kb % 4
    return np.ascontiguousarray(s[off])


def checkpoint_form(packed, sf, experts, n, K, gated):
    rm = untile_packed(packed, experts * n, K)
    srm = untile_scales(sf, experts * n, K)
    if gated:  # [gate; up] -> the checkpoint's [w3 (up); w1 (gate)] an expert
        rm = np.ascontiguousarray(rm.reshape(experts, 2, n // 2, K // 2)[:, ::-1].reshape(experts * n, K // 2))
        srm = np.ascontiguousarray(srm.reshape(experts, 2, n // 2, K // 32)[:, ::-1].reshape(experts * n, K // 32))
    return rm, srm


@pytest.mark.parametrize("experts,n,K,gated", [(3, 256, 512, True), (2, 384, 256, False), (2, 4096, 7168, True),
                                               (1, 7168, 2048, False)])
def test_import_restores_gemm_layout(dev, experts, n, K, gated):
    g = torch.Generator(device=dev)
    g.manual_seed(experts * 1000 + n + K)
    w = torch.randn((experts * n, K), generator=g, device=dev) * 0.02
    packed, sf = k3moe.quant_mxfp4(w)
    torch.cuda.synchronize()
    rm, srm = checkpoint_form(packed.cpu().numpy(), sf.cpu().numpy(), experts, n, K, gated)
    ip, isf = k3moe.import_mxfp4(torch.from_numpy(rm).to(dev), torch.from_numpy(srm).to(dev), experts, gated)
    torch.cuda.synchronize()
    assert torch.equal(ip, packed), "packed weights differ after the re-layout"
    assert torch.equal(isf, sf), "scales differ after the re-layout"


def test_import_rejects_bad_shapes(dev):
    L = k3moe.lib()
    buf = torch.zeros(1 << 16, dtype=torch.uint8, device=dev)
    p = buf.data_ptr()
    s = k3moe._stream()
    assert L.k3moe_import_mxfp4(p, p, 1, 100, 256, 0, p, p, s) == -1  # rows not a multiple of 128
    assert L.k3moe_import_mxfp4(p, p, 1, 128, 200, 0, p, p, s) == -1  # K not a multiple of 128
    assert L.k3moe_import_mxfp4(p + 8, p, 1, 128, 256, 0, p, p, s) == -1  # packed rows not 16-byte aligned
    assert L.k3moe_import_mxfp4(p, p, 0, 128, 256, 0, p, p, s) == -1
