"""Expert-parallel execution of the MoE layer across the GPUs of one node."""
