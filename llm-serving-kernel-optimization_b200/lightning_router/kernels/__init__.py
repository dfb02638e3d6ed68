"""sm_100a kernels for MoE expert routing and W4A16 expert GEMMs."""
