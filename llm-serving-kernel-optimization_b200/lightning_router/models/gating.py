"""Top-k softmax router, reference ``lightning_router/models/gating.py:15-101``.

Same module interface and parameter name (``gate_proj``, an ``nn.Linear(d, E,
bias=False)``) so reference checkpoints load unchanged.  The forward runs two
sm_100a kernels: the gate projection (fp16 operands, fp32 logits) and the
fused top-k softmax + histogram + aux-loss kernel.  Selection is on the fp32
logits, descending, ties towards the lowest expert index; gate weights are
``p / (sum_topk p + 1e-9)`` (reference ``:75``); the aux loss is the Switch
load-balancing loss ``lbw * E * sum_e f_e P_e`` with the uncapped slot fraction
``f`` (reference ``:91-99``).

``logit_bias`` (optional, enabled by ``bias=True``) is a per-expert fp32 bias
added to the logits, used by the skewed-routing workload.
"""

from __future__ import annotations

import torch
import torch.nn as nn

from lightning_router.kernels.expert_routing import gate_logits, topk_gating_dispatch


class TopKGating(nn.Module):
    def __init__(self, hidden_size: int, num_experts: int, top_k: int = 2,
                 load_balance_weight: float = 0.01, bias: bool = False):
        super().__init__()
        self.num_experts = num_experts
        self.top_k = top_k
        self.load_balance_weight = load_balance_weight
        self.gate_proj = nn.Linear(hidden_size, num_experts, bias=False)
        if bias:
            self.register_buffer("logit_bias", torch.zeros(num_experts, dtype=torch.float32))
        else:
            self.logit_bias = None

    def logits(self, hidden_states: torch.Tensor) -> torch.Tensor:
        h = hidden_states.reshape(-1, hidden_states.shape[-1]).detach()
        # inference path: the kernels have no backward, so no autograd graph is built
        return gate_logits(h, self.gate_proj.weight.detach(), self.logit_bias)

    def forward(self, hidden_states: torch.Tensor):
        """Returns ``(expert_ids (S,) int32, gate_weights (S,) fp32,
        token_indices (S,) int32, aux_loss ())`` with ``S = T * top_k``."""
        logits = self.logits(hidden_states)
        plan = topk_gating_dispatch(None, logits, self.top_k, capacity=1,
                                    load_balance_weight=self.load_balance_weight)
        return plan.expert_ids, plan.gate_weights, plan.token_indices, plan.aux_loss
