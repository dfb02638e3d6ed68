"""Expert routing: fused top-k gating + capacity-masked dispatch, and combine.

Drop-in for the reference's ``lightning_router/kernels/expert_routing.py``:

* :func:`expert_routing_forward` (reference ``:164-230``) -- histogram, scan and
  placement of precomputed slots.  Returns ``(permuted, offsets, routing_weights,
  source_indices)`` with the reference's layout: ``offsets`` is the UNCAPPED CSR
  over experts (so ``offsets[1:] - offsets[:-1] == bincount(expert_ids)``), expert
  ``e`` owns rows ``[offsets[e], offsets[e+1])`` and its first
  ``min(count, capacity)`` rows are its kept slots in slot order.  Dropped rows
  are zero with ``routing_weight = 0`` and ``source_index`` = their token (the
  reference leaves them uninitialised).  ``capacity = max(int(S / E * cf), 1)``.
* :func:`expert_routing_gather` (reference ``:274-298``) -- weighted return to
  token order, fp32 accumulation in ascending row order, one fp16 store (the
  reference accumulates with fp16 atomics in arbitrary order).
* :func:`topk_gating_dispatch` -- top-k softmax gating from fp32 logits,
  histogram, scan, capacity and permutation in two kernel launches with no host
  synchronisation.
* :func:`gate_topk_gating_dispatch` -- the path used by ``MoELayer``: the gate
  projection followed by the above; up to 256 tokens (decode) the projection
  joins the routing launch.
* :func:`combine` -- token-major weighted combine driven by ``slot_pos``.

Slot ``s = t * k + j`` lists token ``t``'s experts in descending logit order,
ties broken towards the lowest expert index.
"""

from __future__ import annotations

from typing import NamedTuple

import torch

from lightning_router import _ext


# token count up to which the gate projection runs inside the routing launch
SMALL_BATCH_TOKENS = 256


def expert_capacity(num_slots: int, num_experts: int, capacity_factor: float) -> int:
    """``max(int((S / E) * cf), 1)`` -- reference ``expert_routing.py:196-197``."""
    return max(int((num_slots / num_experts) * capacity_factor), 1)


class RoutingPlan(NamedTuple):
    expert_ids: torch.Tensor      # (S,) int32
    gate_weights: torch.Tensor    # (S,) fp32
    token_indices: torch.Tensor   # (S,) int32
    offsets: torch.Tensor         # (E+1,) int32, uncapped CSR
    kept_counts: torch.Tensor     # (E,) int32
    aux_loss: torch.Tensor        # () fp32
    permuted: torch.Tensor        # (S, d) fp16 (empty when routing only)
    routing_weights: torch.Tensor  # (S,) fp32 per row
    source_indices: torch.Tensor  # (S,) int32 per row
    slot_pos: torch.Tensor        # (S,) int32 row of each slot, -1 if dropped
    capacity: int


def topk_gating_dispatch(x: torch.Tensor | None, logits: torch.Tensor, top_k: int,
                         capacity_factor: float = 1.25, load_balance_weight: float = 0.01,
                         fill_dropped: bool = False, capacity: int | None = None) -> RoutingPlan:
    """Fused top-k softmax gating + dispatch from fp32 ``logits`` (T, E).

    ``x`` (T, d) fp16 is permuted into expert-contiguous rows; pass ``None`` for
    routing metadata only.
    """
    _ext.require_cuda(logits, x)
    T, E = logits.shape
    C = expert_capacity(T * top_k, E, capacity_factor) if capacity is None else int(capacity)
    err = _ext.error_word(logits.device.index)
    outs = _ext.ops().topk_gating_dispatch(
        None if x is None else x.contiguous(), logits.contiguous().float(), int(top_k), C,
        float(load_balance_weight), bool(fill_dropped), True, err)
    return RoutingPlan(*outs, capacity=C)


def gate_topk_gating_dispatch(x: torch.Tensor, gate_weight: torch.Tensor,
                              bias: torch.Tensor | None, top_k: int,
                              capacity_factor: float = 1.25, load_balance_weight: float = 0.01,
                              fill_dropped: bool = False, capacity: int | None = None,
                              permute: bool = True) -> tuple[torch.Tensor, RoutingPlan]:
    """Gate projection ``x @ gate_weight.T (+ bias)`` followed by
    :func:`topk_gating_dispatch`; returns ``(logits, plan)``.

    ``x`` (T, d) fp16 is the gate input and the rows to permute (``permute=False``:
    routing metadata only); ``gate_weight`` (E, d) fp16.  Up to 256 tokens the
    projection, top-k and routing run in one kernel launch (plus the row copy);
    the logits are bit-identical to :func:`gate_logits` either way.
    """
    _ext.require_cuda(x, gate_weight)
    T, E = x.shape[0], gate_weight.shape[0]
    C = expert_capacity(T * top_k, E, capacity_factor) if capacity is None else int(capacity)
    err = _ext.error_word(x.device.index)
    outs = _ext.ops().gate_topk_gating_dispatch(
        x.half().contiguous(), gate_weight.half().contiguous(),
        None if bias is None else bias.float().contiguous(), int(top_k), C,
        float(load_balance_weight), bool(fill_dropped), bool(permute), err)
    return outs[0], RoutingPlan(*outs[1:], capacity=C)


def expert_routing_forward(
    tokens: torch.Tensor,
    expert_ids: torch.Tensor,
    gate_weights: torch.Tensor,
    token_indices: torch.Tensor,
    num_experts: int,
    capacity_factor: float = 1.25,
) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor, torch.Tensor]:
    """Route tokens to experts; see the module docstring for the layout."""
    permuted, offsets, rw, src, _kept, _pos = expert_routing_forward_ex(
        tokens, expert_ids, gate_weights, token_indices, num_experts, capacity_factor)
    return permuted, offsets, rw, src


def expert_routing_forward_ex(tokens, expert_ids, gate_weights, token_indices, num_experts,
                              capacity_factor=1.25):
    """:func:`expert_routing_forward` plus ``kept_counts`` (E,) and ``slot_pos`` (S,)."""
    _ext.require_cuda(tokens, expert_ids, gate_weights, token_indices)
    S = expert_ids.numel()
    C = expert_capacity(S, num_experts, capacity_factor)
    err = _ext.error_word(tokens.device.index)
    return tuple(_ext.ops().expert_routing_forward(
        tokens.contiguous(), expert_ids.reshape(-1).to(torch.int32).contiguous(),
        gate_weights.reshape(-1).float().contiguous(),
        token_indices.reshape(-1).to(torch.int32).contiguous(), int(num_experts), C, True, err))


def expert_routing_gather(
    expert_output: torch.Tensor,
    routing_weights: torch.Tensor,
    source_indices: torch.Tensor,
    num_tokens: int,
) -> torch.Tensor:
    """Weighted gather of expert rows back to token order (fp16 out)."""
    _ext.require_cuda(expert_output, routing_weights, source_indices)
    err = _ext.error_word(expert_output.device.index)
    return _ext.ops().expert_routing_gather(
        expert_output.contiguous(), routing_weights.reshape(-1).float().contiguous(),
        source_indices.reshape(-1).to(torch.int32).contiguous(), int(num_tokens), err)


def combine(expert_output: torch.Tensor, gate_weights: torch.Tensor, slot_pos: torch.Tensor,
            num_tokens: int, top_k: int) -> torch.Tensor:
    """``out[t] = sum_j w[t*k+j] * y[slot_pos[t*k+j]]`` over kept slots (fp32 accumulate)."""
    _ext.require_cuda(expert_output, gate_weights, slot_pos)
    return _ext.ops().combine(expert_output.contiguous(), gate_weights.contiguous(),
                              slot_pos.contiguous(), int(num_tokens), int(top_k))


def gate_logits(hidden: torch.Tensor, gate_weight: torch.Tensor,
                bias: torch.Tensor | None = None) -> torch.Tensor:
    """fp32 logits ``hidden @ gate_weight.T (+ bias)`` from fp16 operands."""
    _ext.require_cuda(hidden, gate_weight)
    return _ext.ops().gate_logits(hidden.half().contiguous(), gate_weight.half().contiguous(),
                                  None if bias is None else bias.float().contiguous())
