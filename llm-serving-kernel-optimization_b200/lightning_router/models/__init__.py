"""MoE model components: gating, expert FFN and the fused MoE layer."""
