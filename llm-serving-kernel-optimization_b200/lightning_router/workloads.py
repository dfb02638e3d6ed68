"""Seeded synthetic workloads for the MoE-layer configurations.

No public dataset is involved: activations are fp16 N(0, 1), the gate weight is
fp16 N(0, 0.02) of shape (E, d), expert weights are fp32 N(0, 0.02) cast to fp16,
stored (K = in, N = out) and packed with :func:`quantize_tensor`.  Tensors are
drawn from one ``torch.Generator`` in a fixed order (x, gate weight, bias, then
per expert gate/up/down), so a CPU run and a GPU run of the same generator
device see identical bits.

The skewed-routing workload adds a per-expert logit bias from a Zipf(s) ranking:
a random permutation assigns ranks 1..E and ``bias_e = -s ln(rank_e)`` minus
its log-sum-exp, i.e. a normalised log-Zipf prior.
"""

from __future__ import annotations

import math
from dataclasses import dataclass, field

import torch

from lightning_router.quantization.pack_weights import quantize_tensor


@dataclass(frozen=True)
class LayerWorkload:
    name: str
    tokens: int
    d_model: int
    d_ff: int
    experts: int
    top_k: int
    group_size: int
    activation: str            # "swiglu" or "silu"
    capacity_factor: float
    seed: int
    zipf_s: float = 0.0        # > 0 adds the Zipf logit bias


WORKLOADS = {
    "pr1": LayerWorkload("pr1", 4096, 1024, 4096, 4, 2, 128, "silu", 1.25, 0),
    "decode": LayerWorkload("decode", 64, 4096, 14336, 8, 2, 128, "swiglu", 1.25, 1),
    "prefill": LayerWorkload("prefill", 16384, 4096, 14336, 8, 2, 128, "swiglu", 1.25, 2),
    "fine": LayerWorkload("fine", 8192, 2048, 1408, 64, 6, 64, "swiglu", 1.5, 3, zipf_s=1.2),
}

SWEEP_TOKENS = (1024, 4096, 16384, 65536, 262144)
SWEEP_D = 4096
SWEEP_E = 8
SWEEP_K = 2


@dataclass
class LayerTensors:
    x: torch.Tensor                 # (T, d) fp16
    gate_w: torch.Tensor            # (E, d) fp16
    bias: torch.Tensor | None       # (E,) fp32
    # per expert: {"gate"/"up"/"down": (qweight, scales, zeros)}
    experts: list = field(default_factory=list)


def zipf_bias(num_experts: int, s: float, gen: torch.Generator) -> torch.Tensor:
    perm = torch.randperm(num_experts, generator=gen, device=gen.device)
    rank = (perm + 1).to(torch.float64)
    logp = -s * torch.log(rank)
    logp = logp - torch.logsumexp(logp, dim=0)
    return logp.float()


def make_layer(w: LayerWorkload, device: str | torch.device = "cuda",
               gen_device: str | torch.device | None = None, tokens: int | None = None,
               experts: int | None = None) -> LayerTensors:
    """Build the workload's tensors on ``device``.

    ``gen_device`` selects where the random numbers are drawn (default: CPU for
    bit-reproducibility against the CPU oracle).  ``tokens`` / ``experts``
    override the token count / the number of experts whose weights are built
    (the others are skipped, for memory-bounded parity checks).
    """
    gdev = torch.device("cpu" if gen_device is None else gen_device)
    g = torch.Generator(device=gdev).manual_seed(w.seed)
    T = w.tokens if tokens is None else tokens
    x = torch.randn(T, w.d_model, generator=g, device=gdev).half()
    gate_w = (torch.randn(w.experts, w.d_model, generator=g, device=gdev) * 0.02).half()
    bias = zipf_bias(w.experts, w.zipf_s, g) if w.zipf_s > 0 else None
    out = LayerTensors(x.to(device), gate_w.to(device), None if bias is None else bias.to(device))
    n_build = w.experts if experts is None else experts
    mats = (("gate", w.d_model, w.d_ff), ("up", w.d_model, w.d_ff), ("down", w.d_ff, w.d_model))
    for e in range(n_build):
        ex = {}
        for name, K, N in mats:
            if name == "gate" and w.activation != "swiglu":
                continue
            W = (torch.randn(K, N, generator=g, device=gdev) * 0.02).half().to(device)
            ex[name] = quantize_tensor(W, w.group_size)
            del W
        out.experts.append(ex)
    return out


def load_into_layer(layer, t: LayerTensors, first_expert: int = 0) -> None:
    """Copy workload tensors into a ``MoELayer`` (gate, bias, expert buffers)."""
    with torch.no_grad():
        layer.gate.gate_proj.weight.copy_(t.gate_w.to(layer.gate.gate_proj.weight.dtype))
        if t.bias is not None:
            layer.gate.logit_bias.copy_(t.bias)
        for i, ex in enumerate(t.experts):
            mod = layer.experts.experts[first_expert + i]
            for name, (q, s, z) in ex.items():
                getattr(mod, f"{name}_qweight").copy_(q)
                getattr(mod, f"{name}_scales").copy_(s)
                getattr(mod, f"{name}_zeros").copy_(z)


def build_layer(w: LayerWorkload, device="cuda", **kw):
    """A ``MoELayer`` for workload ``w`` on ``device`` plus its ``LayerTensors``."""
    from lightning_router.config import KernelConfig, ModelConfig, MoEConfig, QuantizationConfig
    from lightning_router.models.moe_layer import MoELayer
    layer = MoELayer(ModelConfig(hidden_size=w.d_model, intermediate_size=w.d_ff),
                     MoEConfig(num_experts=w.experts, num_experts_per_token=w.top_k,
                               expert_capacity_factor=w.capacity_factor,
                               expert_activation=w.activation, gate_bias=w.zipf_s > 0),
                     QuantizationConfig(group_size=w.group_size), KernelConfig())
    layer = layer.to(device)
    layer.gate.gate_proj.half()
    t = make_layer(w, device=device, **kw)
    load_into_layer(layer, t)
    return layer, t


def sweep_inputs(tokens: int, index: int, device="cuda", gen_device=None):
    """Dispatch-sweep inputs: x (T, 4096) fp16 N(0,1) and logits (T, 8) fp32 N(0,1)."""
    gdev = torch.device("cpu" if gen_device is None else gen_device)
    g = torch.Generator(device=gdev).manual_seed(100 + index)
    x = torch.randn(tokens, SWEEP_D, generator=g, device=gdev).half()
    logits = torch.randn(tokens, SWEEP_E, generator=g, device=gdev)
    return x.to(device), logits.to(device)


def dispatch_bytes(T: int, d: int, E: int, S: int, kept: int) -> int:
    """Algorithmic HBM bytes of one dispatch: read tokens once, write kept rows,
    read logits, write per-slot metadata (ids, weight, position)."""
    return T * d * 2 + kept * d * 2 + T * E * 4 + S * 12


def combine_bytes(T: int, d: int, S: int, kept: int) -> int:
    """Algorithmic HBM bytes of one combine: read kept rows, write tokens, read slot metadata."""
    return kept * d * 2 + T * d * 2 + S * 8


def ffn_flops(kept_rows: int, d: int, f: int, gated: bool) -> int:
    return 2 * kept_rows * (3 if gated else 2) * d * f


def weight_bytes(w: LayerWorkload, active_experts: int | None = None) -> int:
    """Packed INT4 weights + scales + zeros of the active experts."""
    E = w.experts if active_experts is None else active_experts
    n_in = 2 if w.activation == "swiglu" else 1
    per = 0
    for K, N in [(w.d_model, w.d_ff)] * n_in + [(w.d_ff, w.d_model)]:
        per += K * N // 2 + (K // w.group_size) * N * 2 + (K // w.group_size) * (N // 8) * 4
    return E * per
