"""The router GEMM (k3moe_router_gemm: S = x . W_router^T, bf16 x bf16 -> f32 on tcgen05 kind::f16) against an
fp32 matmul of the same bf16 operands.  Products of bf16 values are exact in f32, so the two differ only in the
order of the f32 sums: rel-L2 <= 1e-5 and max-abs <= 1e-4 (values of order 1)."""
import pytest
import torch

import k3moe

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("T,H,E", [(333, 1024, 64), (1000, 7168, 896), (8192, 7168, 896), (128, 2048, 16),
                                   (77, 512, 48)])
def test_router_gemm_matches_fp32_matmul(dev, T, H, E):
    g = torch.Generator(device=dev)
    g.manual_seed(T + H + E)
    x = torch.randn((T, H), generator=g, device=dev).to(torch.bfloat16)
    w = (torch.randn((E, H), generator=g, device=dev) / H ** 0.5).to(torch.bfloat16)
    err = torch.zeros(4, dtype=torch.int32, device=dev)
    S = k3moe.router_gemm(x, w, err)
    ref = x.float() @ w.float().t()
    torch.cuda.synchronize()
    assert err[:2].tolist() == [0, 0]
    rel = float((S - ref).norm() / ref.norm())
    mx = float((S - ref).abs().max())
    assert rel <= 1e-5 and mx <= 1e-4, (rel, mx)


def test_router_gemm_feeds_the_topk(dev):
    """The logits from the router GEMM route the same as fp32 logits wherever the two keep their order: the
    ids agree for all but a handful of near-tied rows."""
    T, H, E, K = 4096, 7168, 896, 8
    g = torch.Generator(device=dev)
    g.manual_seed(7)
    x = torch.randn((T, H), generator=g, device=dev).to(torch.bfloat16)
    w = (torch.randn((E, H), generator=g, device=dev) / H ** 0.5).to(torch.bfloat16)
    bias = torch.rand(E, generator=g, device=dev) * 0.2 - 0.1
    rs = torch.tensor([2.5], dtype=torch.bfloat16, device=dev)
    i1, _ = k3moe.route_topk(k3moe.router_gemm(x, w), bias, rs, K)
    i2, _ = k3moe.route_topk((x.float() @ w.float().t()).contiguous(), bias, rs, K)
    torch.cuda.synchronize()
    differing = int((i1 != i2).any(1).sum())
    assert differing <= T // 200, differing
