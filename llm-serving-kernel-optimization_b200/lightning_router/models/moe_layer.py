"""Mixture-of-Experts layer, reference ``lightning_router/models/moe_layer.py:20-135``.

``MoELayer(model_cfg, moe_cfg, quant_cfg, kernel_cfg).forward(h) -> (out, aux_loss)``
with ``h`` of shape (B, S, d) or (T, d).  One forward is six stream-ordered
launches and no host synchronisation:

1. gate projection             fp16 h . fp16 Wg^T -> fp32 logits        (CUDA cores / mma.sync)
2. top-k softmax + histogram   ids, weights, slot ranks, aux loss, CSR offsets
   (up to 256 tokens, 1 and 2 are one launch: the decode step is five)
3. permute                     token rows -> expert-contiguous rows (kept slots only)
4. grouped W4A16 gate/up GEMM  tcgen05, fused SwiGLU (or SiLU) epilogue
5. grouped W4A16 down GEMM     tcgen05
6. combine                     token-major fp32 weighted sum, one fp16 store

Capacity is ``max(int(T*k/E * cf), 1)`` per expert (reference
``expert_routing.py:196-197``); slots beyond it are dropped in slot order.
``routing_implementation`` is accepted for configuration compatibility; there
is a single (CUDA) implementation.
"""

from __future__ import annotations

import torch
import torch.nn as nn

from lightning_router.config import KernelConfig, ModelConfig, MoEConfig, QuantizationConfig
from lightning_router.kernels.expert_routing import (
    SMALL_BATCH_TOKENS, RoutingPlan, combine, expert_capacity, gate_topk_gating_dispatch,
    topk_gating_dispatch)
from lightning_router.models.experts import ExpertGroup
from lightning_router.models.gating import TopKGating


class MoELayer(nn.Module):
    def __init__(self, model_cfg: ModelConfig, moe_cfg: MoEConfig,
                 quant_cfg: QuantizationConfig, kernel_cfg: KernelConfig):
        super().__init__()
        self.moe_cfg = moe_cfg
        self.kernel_cfg = kernel_cfg
        self.hidden_size = model_cfg.hidden_size
        self.intermediate_size = model_cfg.intermediate_size
        self.num_experts = moe_cfg.num_experts
        self.top_k = moe_cfg.num_experts_per_token
        self.gate = TopKGating(
            hidden_size=model_cfg.hidden_size,
            num_experts=moe_cfg.num_experts,
            top_k=moe_cfg.num_experts_per_token,
            load_balance_weight=moe_cfg.load_balance_loss_weight,
            bias=getattr(moe_cfg, "gate_bias", False),
        )
        self.experts = ExpertGroup(
            num_experts=moe_cfg.num_experts,
            hidden_size=model_cfg.hidden_size,
            intermediate_size=model_cfg.intermediate_size,
            quantized=quant_cfg.enabled and quant_cfg.quantize_experts,
            group_size=quant_cfg.group_size,
            activation=getattr(moe_cfg, "expert_activation", "swiglu"),
        )

        # optional list; when set, each forward appends (stage, cuda.Event) marks
        self.stage_events: list | None = None

    def _mark(self, name: str) -> None:
        if self.stage_events is not None:
            ev = torch.cuda.Event(enable_timing=True)
            ev.record()
            self.stage_events.append((name, ev))

    def capacity(self, num_tokens: int) -> int:
        return expert_capacity(num_tokens * self.top_k, self.num_experts,
                               self.moe_cfg.expert_capacity_factor)

    def route(self, hidden_states: torch.Tensor) -> tuple[torch.Tensor, RoutingPlan]:
        """Gate logits and the dispatch plan (rows permuted) for (T, d) fp16 input."""
        if hidden_states.shape[0] <= SMALL_BATCH_TOKENS:
            # decode-sized batches: projection, top-k and routing in one launch
            logits, plan = gate_topk_gating_dispatch(
                hidden_states, self.gate.gate_proj.weight.detach(), self.gate.logit_bias,
                self.top_k, load_balance_weight=self.gate.load_balance_weight,
                capacity=self.capacity(hidden_states.shape[0]))
            self._mark("gate")
            return logits, plan
        logits = self.gate.logits(hidden_states)
        self._mark("gate")
        plan = topk_gating_dispatch(hidden_states, logits, self.top_k,
                                    load_balance_weight=self.gate.load_balance_weight,
                                    capacity=self.capacity(hidden_states.shape[0]))
        return logits, plan

    def expert_forward(self, plan: RoutingPlan) -> torch.Tensor:
        """Expert outputs for the kept rows of ``plan.permuted``."""
        if self.experts.quantized:
            seg_start = plan.offsets[:-1]
            return self.experts.forward_segments(plan.permuted, seg_start, plan.kept_counts,
                                                 plan.capacity, mark=self._mark)
        # unquantized experts (reference nn.Linear path): per-expert slices
        y = torch.zeros_like(plan.permuted)
        offs = plan.offsets.tolist()
        kept = plan.kept_counts.tolist()
        for e, ex in enumerate(self.experts.experts):
            if kept[e]:
                rows = slice(offs[e], offs[e] + kept[e])
                y[rows] = ex(plan.permuted[rows]).to(y.dtype)
        return y

    def forward(self, hidden_states: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
        orig_shape, orig_dtype = hidden_states.shape, hidden_states.dtype
        h = hidden_states.reshape(-1, orig_shape[-1]).to(torch.float16).contiguous()
        T = h.shape[0]
        self._mark("begin")
        _logits, plan = self.route(h)
        self._mark("dispatch")
        y = self.expert_forward(plan)
        out = combine(y, plan.gate_weights, plan.slot_pos, T, self.top_k)
        self._mark("combine")
        return out.to(orig_dtype).view(orig_shape), plan.aux_loss
