"""The reference's own GEMM family on the same GPU — TEST INFRASTRUCTURE ONLY (a baseline and a parity pin).

The reference runs its MoE FC1 / FC2 as TRT-LLM-gen batched-GEMM cubins (kernels.toml:1-9, families
`trtllm_bmm_mxe4m3_mxe2m1_mxe4m3` and `trtllm_bmm_bf16_mxe2m1_mxe4m3`), whose parameter block is packed by the
kern runtime, absent from the reference tree.  Its K14 gate records that the same family run through
FlashInfer's `trtllm_fp4_block_scale_moe` gave byte-identical outputs (docs/k3-kernel-abi.md:567-569).
FlashInfer 0.6.11 (installed, with its `flashinfer_cubin` bundle of that family) is therefore the way to run
the reference's GEMMs here: this module drives `trtllm_fp4_block_scale_routed_moe` (MXFP8 activations x MXFP4
weights, SwiGLU, bf16 out, top-k ids given) on the same quantised operands as k3moe's layer.

Weights go in as the reference binds them: the checkpoint form (row-major E2M1 rows and UE8M0 scales, FC1 as
[w3 (up); w1 (gate)]) through the reference's load-time shuffles (source/k3_moe_prefill.cu:237-259: within
32 rows, row r takes row (r/32)*32 + (r%8)*4 + (r%32)/8; FC1 interleaves the two halves; scales 128x4-tiled an
expert), restated here with torch indexing on the device.  The host launcher of that FlashInfer module is
compiled once into oracle/_fi (`make -C oracle flashinfer`, FlashInfer's JIT with FLASHINFER_WORKSPACE_BASE set
there).  What this pinned: the reference FC1 requantises its output with the OCP MX exponent rule
(floor(log2(amax)) - 8), which the oracle's and k3moe's FC1 now use too.

Only bench.py's baseline legs and tests/ import this; the product never does.
"""
from __future__ import annotations

import glob
import os

import torch

FI_DIR = os.path.join(os.path.dirname(os.path.abspath(__file__)), "_fi")


def available() -> bool:
    """FlashInfer's host launcher of the TRT-LLM-gen MoE has been compiled into oracle/_fi (make -C oracle
    flashinfer): without it the first call would compile it (about 20 minutes), so callers skip instead."""
    return bool(glob.glob(os.path.join(FI_DIR, ".cache", "flashinfer", "*", "*", "cached_ops",
                                       "fused_moe_trtllm_sm100", "fused_moe_trtllm_sm100.so")))


def _use_cache():
    os.environ.setdefault("FLASHINFER_WORKSPACE_BASE", FI_DIR)


def _shuffle_rows(n: int, gated: bool, device) -> torch.Tensor:
    """Source row of every destination row of one expert (the reference's w_shuffle / sf_shuffle map)."""
    r = torch.arange(n, device=device)
    u = (r // 32) * 32 + (r % 8) * 4 + (r % 32) // 8
    if not gated:
        return u
    return torch.where(u % 2 == 1, n // 2, 0) + u // 2


def untile_packed(p: torch.Tensor, rows: int, K: int) -> torch.Tensor:
    """k3moe's tile-major packed E2M1 -> row-major [rows, K/2] (the checkpoint's `weight_packed` form)."""
    return p.reshape(rows // 128, K // 128, 128, 64).permute(0, 2, 1, 3).reshape(rows, K // 2).contiguous()


def _sf_tiled_index(rows: int, kbn: int, device) -> torch.Tensor:
    """Byte offset of scale (r, kb) in the 128x4-tiled layout over `rows` rows, [rows, kbn]."""
    kg4 = kbn // 4
    r = torch.arange(rows, device=device, dtype=torch.int64)[:, None]
    kb = torch.arange(kbn, device=device, dtype=torch.int64)[None, :]
    return ((r // 128) * kg4 + kb // 4) * 512 + (r % 32) * 16 + ((r % 128) // 32) * 4 + kb % 4


def untile_scales(s: torch.Tensor, rows: int, K: int) -> torch.Tensor:
    """128x4-tiled scales -> row-major [rows, K/32] (the checkpoint's `weight_scale` form)."""
    return s[_sf_tiled_index(rows, K // 32, s.device)].contiguous()


def reference_weights(packed: torch.Tensor, sf: torch.Tensor, experts: int, n: int, K: int, gated: bool):
    """k3moe's weights of `experts` experts (tile-major [gate; up] for FC1) -> the reference GEMMs' operands:
    the checkpoint form ([up; gate] for FC1) shuffled as the reference's load-time shuffles do.
    Returns (weights u8 [experts, n, K/2], scales viewed as float8_e4m3fn [experts, n, K/32])."""
    dev = packed.device
    rm = untile_packed(packed, experts * n, K).view(experts, n, K // 2)
    srm = untile_scales(sf, experts * n, K).view(experts, n, K // 32)
    if gated:  # [gate; up] -> the checkpoint's [w3 (up); w1 (gate)]
        rm = torch.cat([rm[:, n // 2:], rm[:, :n // 2]], 1)
        srm = torch.cat([srm[:, n // 2:], srm[:, :n // 2]], 1)
    src = _shuffle_rows(n, gated, dev)
    w = rm[:, src].contiguous()
    s_rows = srm[:, src]                                   # [experts, n, K/32] in GEMM row order
    idx = _sf_tiled_index(n, K // 32, dev)                 # tiled an expert
    s = torch.empty((experts, n * (K // 32)), dtype=torch.uint8, device=dev)
    s[:, idx.reshape(-1)] = s_rows.reshape(experts, -1)
    return w, s.view(experts, n, K // 32).view(torch.float8_e4m3fn)


def pack_topk(idx: torch.Tensor, wts: torch.Tensor) -> torch.Tensor:
    """Top-k ids and weights packed as FlashInfer's routed entry reads them: the expert id in the high 16
    bits, the weight's bf16 bits in the low 16 (the packing FlashInfer's own tuner makes,
    fused_moe/core.py `_init_packed_topk_ids`)."""
    wb = wts.to(torch.bfloat16).view(torch.int16).to(torch.int32) & 0xFFFF
    return ((idx.to(torch.int32) << 16) | wb).contiguous()


class ReferenceMoE:
    """The routed experts (no shared expert) through FlashInfer's TRT-LLM-gen MoE."""

    def __init__(self, w13, w13_sf, w2, w2_sf, E, H, I, K):
        _use_cache()
        import flashinfer.fused_moe as fm

        self.fm = fm
        self.E, self.H, self.I, self.K = E, H, I, K
        self.g1, self.g1s = reference_weights(w13, w13_sf, E, 2 * I, H, True)
        self.g2, self.g2s = reference_weights(w2, w2_sf, E, H, I, False)

    def forward(self, q_fp8, sf_linear, topk_packed, finalize=True, tune_max=8192):
        """q_fp8 [T, H] float8_e4m3fn, sf_linear [T, H/32] (UE8M0 bytes), topk_packed [T, K] int32.
        finalize: the combined bf16 output [T, H]; else (FC2 rows [padded, H], expanded->permuted row map)."""
        out = self.fm.trtllm_fp4_block_scale_routed_moe(
            topk_packed, None, q_fp8, sf_linear.view(torch.float8_e4m3fn), self.g1, self.g1s, None, None, None,
            None, self.g2, self.g2s, None, None, None, None, self.E, self.K, None, None, self.I, 0, self.E, None,
            routing_method_type=1, do_finalize=finalize, tune_max_num_tokens=tune_max)
        return out[0] if finalize else (out[0], out[2])

    def tune(self, q_fp8, sf_linear, topk_packed):
        """FlashInfer's autotuner over this call's token count only (its default sweep of 1..8192 tokens took
        over 20 minutes at the K3 shape)."""
        import flashinfer
        import flashinfer.fused_moe.core as fcore

        T = q_fp8.shape[0]
        orig = fcore.get_hybrid_num_tokens_buckets
        fcore.get_hybrid_num_tokens_buckets = lambda mx, mn=1: (T,)
        try:
            with flashinfer.autotune(True):
                self.forward(q_fp8, sf_linear, topk_packed, finalize=True, tune_max=T)
        finally:
            fcore.get_hybrid_num_tokens_buckets = orig
