"""The device-resident expert-parallel step (k3moe_ep_forward) on one GPU (world 1: no process group, no
peers): its output must equal, bit for bit, the one-GPU layer (k3moe_layer_forward) on the same inputs, step
after step over reused buffers, eagerly and replayed from a CUDA graph that captured the whole step.  The
multi-rank cases run in tests/test_gpu_ep.py (2 GPUs)."""
import ctypes

import numpy as np
import pytest
import torch

import k3moe
import k3moe_ep

pytestmark = pytest.mark.gpu


def _case(T, H, I, E, K, shared, seed, dev):
    w13, w13_sf = k3moe.synth_mxfp4(seed, (E + shared) * 2 * I, H, 0.02, device=dev)
    w2, w2_sf = k3moe.synth_mxfp4(seed + 1, (E + shared) * H, I, 0.02, device=dev)
    rng = np.random.default_rng(seed)
    x = torch.from_numpy(rng.standard_normal((T, H)).astype(np.float32)).to(torch.bfloat16).to(dev)
    S = torch.from_numpy(rng.standard_normal((T, E)).astype(np.float32)).to(dev)
    bias = torch.from_numpy(rng.uniform(-0.1, 0.1, E).astype(np.float32)).to(dev)
    rs = torch.tensor([2.5], dtype=torch.bfloat16, device=dev)
    w = {"w13": w13, "w13_sf": w13_sf, "w2": w2, "w2_sf": w2_sf}
    return x, S, bias, rs, w


@pytest.mark.parametrize("T,H,I,E,K,shared,max_tokens", [
    (100, 512, 256, 16, 4, 1, 128),
    (300, 1024, 512, 32, 8, 0, 300),
    (1, 512, 256, 16, 8, 1, 64),
])
def test_device_step_equals_one_gpu_layer(T, H, I, E, K, shared, max_tokens):
    dev = torch.device("cuda", 0)
    x, S, bias, rs, w = _case(T, H, I, E, K, shared, 31, dev)
    ref = k3moe.MoELayer(H, I, E, K, shared, w["w13"], w["w13_sf"], w["w2"], w["w2_sf"], bias, rs, max_tokens=T,
                         device=dev)
    want = ref.forward(S, x)
    layer = k3moe_ep.DeviceEPMoELayer(H, I, E, K, shared, w, bias, rs, max_tokens=max_tokens, device=dev)
    for _ in range(3):  # reused buffers, the step number advancing
        got = layer.forward(S, x)
        torch.cuda.synchronize()
        assert torch.equal(got.view(torch.int16), want.view(torch.int16))
    rc, words = layer.error_words()
    assert rc == 0 and words == (0, 0)
    assert layer.received_counts() == [T, T if shared else 0]
    layer.close()


def test_device_step_in_a_cuda_graph():
    dev = torch.device("cuda", 0)
    T, H, I, E, K, shared = 64, 512, 256, 16, 8, 1
    x, S, bias, rs, w = _case(T, H, I, E, K, shared, 41, dev)
    ref = k3moe.MoELayer(H, I, E, K, shared, w["w13"], w["w13_sf"], w["w2"], w["w2_sf"], bias, rs, max_tokens=T,
                         device=dev)
    want = ref.forward(S, x)
    layer = k3moe_ep.DeviceEPMoELayer(H, I, E, K, shared, w, bias, rs, max_tokens=T, device=dev)
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        layer.forward(S, x)
    torch.cuda.current_stream().wait_stream(side)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        out = layer.forward(S, x)
    for _ in range(3):
        out.zero_()
        graph.replay()
        torch.cuda.synchronize()
        assert torch.equal(out.view(torch.int16), want.view(torch.int16))
    # the step number lives on the device: one a replay (plus the eager warm-up step)
    epoch = layer.ws[:4].view(torch.int32).item()
    assert epoch == 4
    graph.reset()
    layer.close()


def test_device_step_placed_experts_one_rank():
    """An owner map on one rank is a relabelling of nothing: every expert local, in id order."""
    dev = torch.device("cuda", 0)
    T, H, I, E, K, shared = 77, 512, 256, 16, 4, 1
    x, S, bias, rs, w = _case(T, H, I, E, K, shared, 51, dev)
    ref = k3moe.MoELayer(H, I, E, K, shared, w["w13"], w["w13_sf"], w["w2"], w["w2_sf"], bias, rs, max_tokens=T,
                         device=dev)
    want = ref.forward(S, x)
    layer = k3moe_ep.DeviceEPMoELayer(H, I, E, K, shared, w, bias, rs, max_tokens=T, owner=[0] * E, device=dev)
    got = layer.forward(S, x)
    torch.cuda.synchronize()
    assert torch.equal(got.view(torch.int16), want.view(torch.int16))
    layer.close()


def test_device_step_rejects_more_tokens_than_configured():
    dev = torch.device("cuda", 0)
    T, H, I, E, K, shared = 40, 512, 256, 16, 4, 0
    x, S, bias, rs, w = _case(T, H, I, E, K, shared, 61, dev)
    layer = k3moe_ep.DeviceEPMoELayer(H, I, E, K, shared, w, bias, rs, max_tokens=32, device=dev)
    with pytest.raises(k3moe.K3MoeError):
        layer.forward(S, x)
    layer.close()
