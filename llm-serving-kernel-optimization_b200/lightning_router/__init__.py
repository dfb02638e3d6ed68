"""LightningRouter MoE-layer hot path for NVIDIA B200 (sm_100a).

Drop-in for the reference package's hot path: ``lightning_router.kernels``
(routing + quantized GEMM entry points), ``lightning_router.models``
(``TopKGating``, ``ExpertFFN``/``ExpertGroup``, ``MoELayer``) and the packed
INT4 format of ``lightning_router.quantization``.  All device work runs in the
hand-written CUDA library ``_lib/liblr_kernels.so`` through the torch custom ops
in ``_lib/_lr_torch_ops.so``; there is no CPU or Triton path.
"""

__version__ = "0.2.0"
