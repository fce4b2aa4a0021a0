"""GEMM parity against the reference's own GEMM family on the same GPU.

The reference's FC1 / FC2 are TRT-LLM-gen batched-GEMM cubins; FlashInfer's `trtllm_fp4_block_scale_routed_moe`
runs that family (the reference's own K14 gate compares them byte for byte).  Here it runs on the same
quantised operands as k3moe's layer (weights re-laid out as the reference binds and shuffles them,
oracle/flashinfer_ref.py), and every (token, pick) FC2 result row and the combined output must agree within the
contract (rel-L2 <= 1e-2).  Skipped where FlashInfer's launcher is not prebuilt (make -C oracle flashinfer)."""
import pytest
import torch

import flashinfer_ref
import k3moe

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("T,H,I,E,K", [(512, 2048, 1024, 32, 8), (1024, 7168, 2048, 64, 8)])
def test_gemms_match_the_reference_family(dev, T, H, I, E, K):
    if not flashinfer_ref.available():
        pytest.skip("FlashInfer's TRT-LLM-gen launcher is not prebuilt in oracle/_fi")
    g = torch.Generator(device=dev)
    g.manual_seed(T + E)
    x = torch.randn((T, H), generator=g, device=dev).to(torch.bfloat16)
    S = (x.float() @ (torch.randn((H, E), generator=g, device=dev) / H ** 0.5)).contiguous()
    bias = (torch.rand(E, generator=g, device=dev) * 0.2 - 0.1).float()
    rs = torch.tensor([2.5], dtype=torch.bfloat16, device=dev)
    w13, w13_sf = k3moe.synth_mxfp4(11, E * 2 * I, H, 0.02, device=dev)
    w2, w2_sf = k3moe.synth_mxfp4(12, E * H, I, 0.02, device=dev)
    layer = k3moe.MoELayer(H, I, E, K, 0, w13, w13_sf, w2, w2_sf, bias, rs, max_tokens=T, device=dev)
    out = layer.forward(S, x)
    torch.cuda.synchronize()
    layer.check_device_error(T)
    off = layer.offsets(T)
    ws = layer.ws
    idx = ws[off["idx"]:off["idx"] + T * K * 4].view(torch.int32).view(T, K).clone()
    wts = ws[off["wts"]:off["wts"] + T * K * 4].view(torch.float32).view(T, K).clone()
    e2p = ws[off["exp2perm"]:off["exp2perm"] + T * K * 4].view(torch.int32).view(T, K)
    tp = int(ws[off["meta"]:off["meta"] + 16].view(torch.int32)[1])
    ours = ws[off["fc2"]:off["fc2"] + tp * H * 2].view(torch.bfloat16).view(tp, H)[e2p.reshape(-1).long()].float()
    q, sf = k3moe.quant_mxfp8(x, tiled_sf=False)
    ref = flashinfer_ref.ReferenceMoE(w13, w13_sf, w2, w2_sf, E, H, I, K)
    tk = flashinfer_ref.pack_topk(idx, wts)
    g2, pmap = ref.forward(q.view(torch.float8_e4m3fn), sf, tk, finalize=False)
    y = ref.forward(q.view(torch.float8_e4m3fn), sf, tk, finalize=True)
    torch.cuda.synchronize()
    theirs = g2[pmap.reshape(-1).long()].float()
    rel_rows = float((ours - theirs).norm() / theirs.norm())
    rel_out = float((out.float() - y.float()).norm() / y.float().norm())
    assert rel_rows <= 1e-2, f"FC2 rows rel-L2 {rel_rows:.3e} against the reference family"
    assert rel_out <= 1e-2, f"combined output rel-L2 {rel_out:.3e} against the reference family"
