"""Offline pass ``quantize_expert_weights`` (reference
``lightning_router/quantization/quantize_model.py:34-108``), on CPU.

The packed buffers it leaves are exactly ``quantize_tensor`` of the TRANSPOSED
Linear weight (the (K = in, N = out) layout of ``ExpertFFN``), under
``ExpertFFN``'s buffer names, and the expert switches to its quantized path.
The dequantized expert reproduces the float Linear expert within the INT4
error, checked through the oracle's fp32 expert FFN."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import moe_oracle as orc


def _layer(d=256, f=512, E=4, act="swiglu"):
    from lightning_router.config import KernelConfig, ModelConfig, MoEConfig, QuantizationConfig
    from lightning_router.models.moe_layer import MoELayer
    torch.manual_seed(0)
    layer = MoELayer(ModelConfig(hidden_size=d, intermediate_size=f),
                     MoEConfig(num_experts=E, num_experts_per_token=2, expert_activation=act),
                     QuantizationConfig(enabled=False), KernelConfig())
    for m in layer.experts.modules():
        if isinstance(m, torch.nn.Linear):
            torch.nn.init.normal_(m.weight, std=0.02)
    return layer


@pytest.mark.parametrize("act", ["swiglu", "silu"])
def test_quantize_expert_weights_layout_names_and_error(act):
    from lightning_router.quantization.pack_weights import dequantize_tensor, quantize_tensor
    from lightning_router.quantization.quantize_model import quantize_expert_weights
    layer = _layer(act=act)
    lin = {n: m.weight.detach().clone() for n, m in layer.named_modules()
           if isinstance(m, torch.nn.Linear) and "experts." in n}
    stats = quantize_expert_weights(layer, group_size=128)
    assert set(stats) == set(lin)
    assert isinstance(layer.gate.gate_proj, torch.nn.Linear)   # the router stays float
    assert layer.experts.quantized
    for name, w in lin.items():
        parent_name, attr = name.rsplit(".", 1)
        parent = dict(layer.named_modules())[parent_name]
        base = attr[:-len("_proj")]
        assert not hasattr(parent, attr) and parent.quantized
        q, s, z = (getattr(parent, f"{base}_{x}") for x in ("qweight", "scales", "zeros"))
        N, K = w.shape                         # Linear: (out, in)
        assert q.shape == (K, N // 8) and s.shape == (K // 128, N) and z.shape == (K // 128, N // 8)
        q2, s2, z2 = quantize_tensor(w.half().t().contiguous(), 128, "asymmetric")
        assert torch.equal(q, q2) and torch.equal(s, s2) and torch.equal(z, z2)
        rel = stats[name]["quant_error"] / stats[name]["orig_norm"]
        assert 0 < rel < 0.15
        deq = dequantize_tensor(q, s, z, 128, N).float()
        assert (deq - w.t().float()).norm() / w.norm() < 0.15


@pytest.mark.parametrize("act", ["swiglu", "silu"])
def test_quantized_experts_match_float_experts(act):
    """The oracle's fp32 expert FFN on the packed buffers ~= the Linear experts."""
    from lightning_router.quantization.pack_weights import dequantize_tensor
    from lightning_router.quantization.quantize_model import quantize_expert_weights
    layer = _layer(act=act)
    x = torch.randn(64, 256)
    with torch.no_grad():
        ref = [e(x).float().numpy() for e in layer.experts.experts]   # nn.Linear path, fp32
    quantize_expert_weights(layer, group_size=128)
    for e, r in zip(layer.experts.experts, ref):
        deq = {m: dequantize_tensor(getattr(e, f"{m}_qweight"), getattr(e, f"{m}_scales"),
                                    getattr(e, f"{m}_zeros"), 128, getattr(e, f"{m}_N")).numpy()
               for m in (("gate", "up", "down") if act == "swiglu" else ("up", "down"))}
        y = orc.expert_ffn(x.numpy(), deq["up"], deq["down"], deq.get("gate"))
        # three INT4 matrices, ~7 % relative error each (a transposed layout would be ~100 %)
        assert np.linalg.norm(y - r) / np.linalg.norm(r) < 0.25


def test_incompatible_dims_are_skipped():
    from lightning_router.quantization.quantize_model import quantize_expert_weights
    m = torch.nn.Module()
    m.up_proj = torch.nn.Linear(100, 64, bias=False)     # in = 100 not a multiple of 128
    stats = quantize_expert_weights(m, group_size=128)
    assert stats == {} and isinstance(m.up_proj, torch.nn.Linear)


@pytest.mark.gpu
def test_quantized_layer_runs_the_tcgen05_path_and_matches_oracle():
    """A float layer quantized in place runs its experts through the grouped W4A16
    GEMM on the GPU and matches the oracle on the packed buffers (layer bars:
    max-abs 2e-2, rel-L2 1e-3)."""
    from lightning_router.quantization.pack_weights import dequantize_tensor
    from lightning_router.quantization.quantize_model import quantize_expert_weights
    layer = _layer(d=512, f=1024, E=4)
    quantize_expert_weights(layer, group_size=128)
    layer = layer.cuda().half()
    x = torch.randn(300, 512, generator=torch.Generator().manual_seed(3)).half().cuda()
    out, aux = layer(x)
    logits, _ = layer.route(x)
    experts = []
    for e in layer.experts.experts:
        experts.append({m: dequantize_tensor(getattr(e, f"{m}_qweight").cpu(),
                                             getattr(e, f"{m}_scales").cpu(),
                                             getattr(e, f"{m}_zeros").cpu(), 128,
                                             getattr(e, f"{m}_N")).numpy()
                        for m in ("gate", "up", "down")})
    ref, _, _ = orc.moe_layer(x.cpu().numpy(), logits.cpu().numpy(), 2,
                              layer.moe_cfg.expert_capacity_factor, experts)
    o = out.float().cpu().numpy()
    assert np.abs(o - ref).max() <= 2e-2
    assert np.linalg.norm(o - ref) / np.linalg.norm(ref) <= 1e-3
