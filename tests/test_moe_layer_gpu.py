"""End-to-end parity of ``MoELayer.forward`` on the GPU.

* Against the numpy oracle (``oracle.moe_layer``) at the full PR1 size and at
  reduced decode / skewed-routing shapes: routing bit-exact given the kernel's
  fp32 gate logits, outputs within max-abs 2e-2 and relative L2 1e-3 of the fp32
  dequant-then-matmul reference, aux loss within 1e-5 relative.
* At the full decode / prefill / skewed sizes, against a plain fp32 torch
  reference of the same layer on the GPU (same tolerances).
"""

from __future__ import annotations

import dataclasses

import numpy as np
import pytest
import torch

import oracle as orc

pytestmark = pytest.mark.gpu
DEV = "cuda"
MAX_ABS = 2e-2
REL_L2 = 1e-3


def _np(t):
    return t.detach().cpu().numpy()


def _oracle_experts(tensors, w):
    experts = []
    for ex in tensors.experts:
        d = {}
        for name, (q, s, z) in ex.items():
            N = s.shape[1]
            d[name] = orc.dequantize_tensor(_np(q), _np(s), _np(z), w.group_size, N)
        experts.append(d)
    return experts


def _compare(out, ref):
    out = out.astype(np.float32)
    err = np.abs(out - ref).max()
    rel = np.linalg.norm(out - ref) / max(np.linalg.norm(ref), 1e-30)
    assert np.isfinite(out).all()
    assert err <= MAX_ABS, f"max-abs {err:.3e}"
    assert rel <= REL_L2, f"rel-L2 {rel:.3e}"


def _run_vs_oracle(w):
    from lightning_router.workloads import build_layer
    layer, t = build_layer(w, device=DEV)
    x = t.x
    out, aux = layer(x)
    logits, plan = layer.route(x)
    lg = _np(logits)
    # the fp32 gate GEMM agrees with the oracle's to rounding
    ref_logits = orc.gate_logits(_np(x), _np(t.gate_w), None if t.bias is None else _np(t.bias))
    np.testing.assert_allclose(lg, ref_logits, rtol=1e-4, atol=1e-4)
    ref, ref_aux, r = orc.moe_layer(_np(x), lg, w.top_k, w.capacity_factor, _oracle_experts(t, w))
    np.testing.assert_array_equal(_np(plan.expert_ids), r.ids)
    np.testing.assert_array_equal(_np(plan.slot_pos), r.slot_pos)
    np.testing.assert_array_equal(_np(plan.kept_counts), r.kept_counts)
    _compare(_np(out), ref)
    assert abs(float(aux) - ref_aux) <= 1e-5 * abs(ref_aux)


def test_pr1_layer_matches_oracle():
    from lightning_router.workloads import WORKLOADS
    _run_vs_oracle(WORKLOADS["pr1"])


@pytest.mark.parametrize("name,overrides", [
    ("decode", dict(d_model=1024, d_ff=2048)),
    ("decode", dict(d_model=4096, d_ff=7168)),
    ("fine", dict(tokens=1024, d_model=512)),
    ("prefill", dict(tokens=2048, d_model=512, d_ff=1024)),
    ("pr1", dict(tokens=333, capacity_factor=0.5)),
    # shapes off the tcgen05 kernel: group 32 (mma.sync kernel), N = 48 / group 16
    # (up projection on CUDA cores, down projection on mma.sync)
    ("decode", dict(d_model=256, d_ff=512, group_size=32)),
    ("pr1", dict(tokens=300, d_model=96, d_ff=48, group_size=16)),
])
def test_reduced_layers_match_oracle(name, overrides):
    from lightning_router.workloads import WORKLOADS
    _run_vs_oracle(dataclasses.replace(WORKLOADS[name], **overrides))


def torch_reference(layer, t, w, plan, x):
    """fp32 torch evaluation of the layer on the kernel's (verified) routing plan."""
    from lightning_router.quantization.pack_weights import dequantize_tensor
    T, d = x.shape
    out = torch.zeros(T, d, dtype=torch.float32, device=DEV)
    offs = plan.offsets.tolist()
    kept = plan.kept_counts.tolist()
    for e, ex in enumerate(t.experts):
        n = kept[e]
        if n == 0:
            continue
        rows = slice(offs[e], offs[e] + n)
        toks = plan.source_indices[rows].long()
        xe = x[toks].float()
        W = {name: dequantize_tensor(q, s, z, w.group_size, s.shape[1]).float()
             for name, (q, s, z) in ex.items()}
        if "gate" in W:
            h = torch.nn.functional.silu(xe @ W["gate"]) * (xe @ W["up"])
        else:
            h = torch.nn.functional.silu(xe @ W["up"])
        ye = h @ W["down"]
        out.index_add_(0, toks, ye * plan.routing_weights[rows, None])
    return out


@pytest.mark.slow
@pytest.mark.parametrize("name", ["decode", "prefill", "fine"])
def test_full_size_layer_matches_torch_fp32(name):
    from lightning_router.workloads import WORKLOADS, build_layer
    w = WORKLOADS[name]
    torch.backends.cuda.matmul.allow_tf32 = False
    layer, t = build_layer(w, device=DEV, gen_device=DEV)
    out, aux = layer(t.x)
    logits, plan = layer.route(t.x)
    # routing bit-exact against the oracle on the kernel's logits
    ids, wts, probs = orc.topk_gating(_np(logits), w.top_k)
    r = orc.dispatch(ids.reshape(-1), wts.reshape(-1), np.repeat(np.arange(w.tokens), w.top_k),
                     w.experts, plan.capacity)
    np.testing.assert_array_equal(_np(plan.slot_pos), r.slot_pos)
    ref = torch_reference(layer, t, w, plan, t.x)
    _compare(_np(out), _np(ref))


def test_reference_forward_shapes():
    """Mirrors the reference's tests/test_moe_layer.py:71-103 (fp16, unquantized experts)."""
    from lightning_router.config import KernelConfig, ModelConfig, MoEConfig, QuantizationConfig
    from lightning_router.models.moe_layer import MoELayer
    for impl, d, f in (("triton", 128, 256), ("torch", 64, 128)):
        layer = MoELayer(ModelConfig(hidden_size=d, intermediate_size=f),
                         MoEConfig(num_experts=4, num_experts_per_token=2, routing_implementation=impl),
                         QuantizationConfig(enabled=False), KernelConfig()).cuda().half()
        x = torch.randn(2, 8, d, dtype=torch.float16, device=DEV)
        out, loss = layer(x)
        assert out.shape == x.shape and loss.dim() == 0
        assert torch.isfinite(out).all()


def test_reference_gating_properties():
    """Mirrors tests/test_moe_layer.py:24-62 on the GPU."""
    from lightning_router.models.gating import TopKGating
    gate = TopKGating(128, 4, 2).to(DEV)
    x = torch.randn(8, 16, 128, device=DEV)
    ids, w, tok, loss = gate(x)
    assert ids.shape == (256,) and w.shape == (256,) and tok.shape == (256,) and loss.dim() == 0
    assert int(ids.min()) >= 0 and int(ids.max()) < 4
    sums = torch.zeros(128, device=DEV).scatter_add_(0, tok.long(), w)
    torch.testing.assert_close(sums, torch.ones(128, device=DEV), atol=1e-5, rtol=1e-5)
    assert float(loss) > 0


def test_layer_is_deterministic():
    from lightning_router.workloads import WORKLOADS, build_layer
    w = dataclasses.replace(WORKLOADS["fine"], tokens=2048, d_model=512)
    layer, t = build_layer(w, device=DEV)
    a, _ = layer(t.x)
    b, _ = layer(t.x)
    assert torch.equal(a, b)
