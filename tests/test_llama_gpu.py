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
