"""The FP8 Llama-shaped stack (the weight-only inference workload): one
layer on a small batch against the same layer computed in float32 from the
dequantised weights. FP8 activations (four per-token e4m3 quantisations per
layer, 3 mantissa bits each) and bf16 intermediates make this an accuracy
bound, not bit parity: the error of the layer's update relative to the update
stays below 10 % (the reference's own bar for FP8 matmul accuracy is a 15 %
relative RMSE, tests/test_fp8_metal.py:52-93)."""
import pytest
import torch
import torch.nn.functional as F

pytestmark = pytest.mark.gpu


def test_one_layer_matches_float32(device):
    from fp4_fp8_for_torch_mps.workloads import LLAMA, Fp8LlamaLayer, _rope, rope_tables
    gen = torch.Generator(device="cuda").manual_seed(0)
    layer = Fp8LlamaLayer(torch.device("cuda"), gen)
    B, S = 2, 256
    h, hd, nkv = LLAMA["hidden"], LLAMA["head_dim"], LLAMA["kv_heads"]
    x = torch.randn(B * S, h, generator=torch.Generator().manual_seed(1)).to(torch.bfloat16).cuda()
    cos, sin = rope_tables(S, "cuda")
    y = layer.forward(x, cos, sin, B, S).float()

    deq = lambda w, s: w.float() * s.float().reshape(-1, 1)
    xf = x.float()
    r = F.rms_norm(xf, (h,), None, LLAMA["eps"])
    q, k, v = (r @ deq(layer.w_qkv, layer.s_qkv).t()).split([h, nkv * hd, nkv * hd], dim=1)
    cf, sf = cos.float(), sin.float()
    q = _rope(q.view(B, S, 32, hd), cf, sf).transpose(1, 2)
    k = _rope(k.view(B, S, nkv, hd), cf, sf).transpose(1, 2)
    v = v.view(B, S, nkv, hd).transpose(1, 2)
    a = F.scaled_dot_product_attention(q, k, v, is_causal=True, enable_gqa=True)
    ref = xf + a.transpose(1, 2).reshape(B * S, h) @ deq(layer.w_o, layer.s_o).t()
    g, u = (F.rms_norm(ref, (h,), None, LLAMA["eps"]) @ deq(layer.w_gu, layer.s_gu).t()).chunk(2, dim=1)
    ref = ref + (F.silu(g) * u) @ deq(layer.w_d, layer.s_d).t()
    rel = ((y - ref).norm() / (ref - xf).norm()).item()   # error relative to the layer's update
    assert torch.isfinite(y).all() and rel < 0.10, rel


def test_graph_replay_matches_eager(device):
    """Two layers captured as one CUDA graph (the benchmark's timed step)
    give the eager forward's bits: the library's launches (tensor maps,
    programmatic dependent launch, clusters) are capture-safe."""
    from fp4_fp8_for_torch_mps import workloads as W
    stack = W.Fp8LlamaStack("cuda", layers=2, seed=0)
    x = W.llama_input(1, 512).cuda()
    eager = stack.forward(x, 1, 512).clone()
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    g = torch.cuda.CUDAGraph()
    with torch.cuda.stream(side):
        with torch.cuda.graph(g, stream=side):
            y = stack.forward(x, 1, 512)
    g.replay()
    torch.cuda.synchronize()
    assert torch.equal(y.view(torch.int16), eager.view(torch.int16))
    x.copy_(W.llama_input(1, 512, seed=3).cuda())         # new input through the same graph
    g.replay()
    torch.cuda.synchronize()
    again = stack.forward(x, 1, 512)
    assert torch.equal(y.view(torch.int16), again.view(torch.int16))
