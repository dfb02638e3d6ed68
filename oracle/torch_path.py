"""PyTorch restatement of the reference's own CPU path of the MoE layer.

TEST INFRASTRUCTURE ONLY -- the timed CPU baseline of ``bench.py`` (its
``cpu_baseline`` leg and ``--impl reference``) and a checker in ``tests/``.
Never imported by the product package.

What ``MoELayer(routing_implementation="torch")`` of the reference runs on a
CPU, operation for operation (the reference cannot be installed where the
benchmark runs, so this port stands in for it; it is pinned against the
reference's own outputs in ``tests/golden/layer_torch.npz``):

* ``TopKGating.forward`` (``lightning_router/models/gating.py:48-101``): fp32
  gate projection, softmax, ``torch.topk`` on the probabilities, renormalised
  by ``sum + 1e-9``, Switch-style auxiliary loss;
* ``MoELayer._torch_routing`` (``lightning_router/models/moe_layer.py:64-86``):
  per expert a mask over the slots, the selected tokens gathered, the expert
  FFN applied and ``index_add_`` of ``out * weight`` into the output -- no
  capacity is applied on this path;
* ``ExpertFFN.forward`` unquantized (``lightning_router/models/experts.py:71-89``):
  ``down(silu(gate x) * up x)``, here with the dequantized INT4 weights in fp32
  held as ``nn.Linear`` holds them, (out, in) row-major, and applied with
  ``F.linear`` (:func:`linear_experts` converts the packed format's (in, out)
  matrices once).  ``gated=False`` gives the ``down(silu(up x))`` expert of the
  non-gated configuration.

The routing-only sweep baseline restates ``vectorized_pytorch_routing``
(``benchmarks/baseline_comparison.py:76-100``): identity experts, one
``index_add_`` per expert in fp32.
"""

from __future__ import annotations

import torch
import torch.nn.functional as F

__all__ = ["gate", "linear_experts", "expert_ffn", "moe_layer", "vectorized_routing"]


def gate(x: torch.Tensor, wg: torch.Tensor, k: int, load_balance_weight: float = 0.01,
         bias: torch.Tensor | None = None):
    """``(expert_ids, gate_weights, token_indices, aux_loss)``, gating.py:48-101.

    ``bias`` is the per-expert logit bias of the skewed-routing workload (the
    reference gate has none; it is added to the logits before the softmax)."""
    T = x.shape[0]
    E = wg.shape[0]
    logits = x @ wg.t()
    if bias is not None:
        logits = logits + bias
    probs = F.softmax(logits, dim=-1)
    w, ids = torch.topk(probs, k, dim=-1)
    w = w / (w.sum(dim=-1, keepdim=True) + 1e-9)
    ids = ids.reshape(-1)
    w = w.reshape(-1).float()
    tok = torch.arange(T).unsqueeze(1).expand(-1, k).reshape(-1)
    f = torch.zeros(E, dtype=torch.float32).scatter_add_(0, ids, torch.ones_like(w)) / (T * k)
    aux = load_balance_weight * E * (f * probs.mean(dim=0)).sum()
    return ids, w, tok, aux


def linear_experts(experts: list) -> list:
    """(in, out) fp32 matrices (the packed format's K x N) -> ``nn.Linear`` weights
    (out, in), contiguous, as the reference's unquantized experts store them."""
    return [{m: W.t().contiguous() for m, W in ex.items()} for ex in experts]


def expert_ffn(x: torch.Tensor, w: dict, gated: bool = True) -> torch.Tensor:
    """experts.py:71-89 with ``nn.Linear`` weights ``w["gate"|"up"|"down"]`` (out, in)."""
    if gated:
        return F.linear(F.silu(F.linear(x, w["gate"])) * F.linear(x, w["up"]), w["down"])
    return F.linear(F.silu(F.linear(x, w["up"])), w["down"])


def moe_layer(x: torch.Tensor, wg: torch.Tensor, experts: list, k: int, gated: bool = True,
              load_balance_weight: float = 0.01, bias: torch.Tensor | None = None):
    """``(out, aux_loss)`` of the reference's torch-routing layer, moe_layer.py:64-135;
    ``experts`` in ``nn.Linear`` layout (:func:`linear_experts`)."""
    ids, w, tok, aux = gate(x, wg, k, load_balance_weight, bias)
    out = torch.zeros_like(x)
    for e in range(len(experts)):
        mask = ids == e
        if not mask.any():
            continue
        slots = mask.nonzero(as_tuple=True)[0]
        toks = tok[slots]
        y = expert_ffn(x[toks], experts[e], gated)
        out.index_add_(0, toks, y * w[slots].unsqueeze(1))
    return out, aux


def vectorized_routing(tokens: torch.Tensor, expert_ids: torch.Tensor, gate_weights: torch.Tensor,
                       token_indices: torch.Tensor, num_experts: int) -> torch.Tensor:
    """Identity-expert dispatch + combine, baseline_comparison.py:76-100."""
    out = torch.zeros(tokens.shape, dtype=torch.float32)
    for e in range(num_experts):
        mask = expert_ids == e
        if not mask.any():
            continue
        slots = mask.nonzero(as_tuple=True)[0]
        toks = token_indices[slots]
        out.index_add_(0, toks, tokens[toks].float() * gate_weights[slots].unsqueeze(1))
    return out.to(tokens.dtype)
