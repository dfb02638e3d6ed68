"""Model runner around the B200 MoE layer, with CUDA-graph replay of fixed shapes.

Same interface as the reference's ``LightningModelRunner``
(``lightning_router/serving/model_runner.py:29-118``): constructed from config
dicts, ``load_model(checkpoint_path)``, ``execute_model(input_ids,
hidden_states) -> output`` per step, and ``enable_profiling`` /
``profile_step``.

The single-GPU layer forward has no host synchronisation (routing, expert GEMMs
and combine are all stream-ordered and size their buffers from static
bounds), so a step of a fixed token count can be captured once as a CUDA graph
and replayed: :meth:`LightningModelRunner.capture` records it, and
``execute_model`` replays it whenever the input has a captured shape (decode
steps do), copying the input into the graph's static buffer.  Other shapes run
eagerly.
"""

from __future__ import annotations

import logging
from pathlib import Path
from typing import Any

import torch

logger = logging.getLogger(__name__)


class _Graph:
    def __init__(self, graph: torch.cuda.CUDAGraph, x: torch.Tensor, out: torch.Tensor,
                 aux: torch.Tensor):
        self.graph, self.x, self.out, self.aux = graph, x, out, aux


class LightningModelRunner:
    """Runs one MoE layer on one GPU for a serving engine."""

    def __init__(self, model_config: dict[str, Any], moe_config: dict[str, Any],
                 quant_config: dict[str, Any], kernel_config: dict[str, Any],
                 device: torch.device | str = "cuda"):
        self.device = torch.device(device)
        self.model_config = dict(model_config)
        self.moe_config = dict(moe_config)
        self.quant_config = dict(quant_config)
        self.kernel_config = dict(kernel_config)
        self.moe_layer = None
        self._graphs: dict[tuple, _Graph] = {}
        self._pool = None

    # -- model ------------------------------------------------------------
    def load_model(self, checkpoint_path: str | Path | None = None) -> None:
        """Build the MoE layer on the device; load a state dict (packed INT4 buffers
        included) when ``checkpoint_path`` is given, else keep the initial weights."""
        from lightning_router.config import KernelConfig, ModelConfig, MoEConfig, QuantizationConfig
        from lightning_router.models.moe_layer import MoELayer
        layer = MoELayer(ModelConfig(**self.model_config), MoEConfig(**self.moe_config),
                         QuantizationConfig(**self.quant_config),
                         KernelConfig(**self.kernel_config))
        if checkpoint_path is not None:
            state = torch.load(checkpoint_path, map_location="cpu", weights_only=True)
            missing, unexpected = layer.load_state_dict(state, strict=False)
            if unexpected:
                logger.warning("checkpoint entries not used: %s", unexpected)
            logger.info("Loaded checkpoint from %s", checkpoint_path)
        layer = layer.to(self.device)
        layer.gate.gate_proj.half()  # the gate GEMM reads fp16 weights (bias stays fp32)
        self.moe_layer = layer.eval()
        self._graphs.clear()

    # -- execution --------------------------------------------------------
    @torch.inference_mode()
    def capture(self, num_tokens: int, warmup: int = 2) -> None:
        """Record one forward of ``num_tokens`` tokens as a CUDA graph (after
        ``warmup`` eager runs, which build the weight tables and size the caches)."""
        layer = self._layer()
        d = layer.hidden_size
        key = (num_tokens, d)
        x = torch.zeros(num_tokens, d, dtype=torch.float16, device=self.device)
        side = torch.cuda.Stream(device=self.device)
        side.wait_stream(torch.cuda.current_stream(self.device))
        with torch.cuda.stream(side):
            for _ in range(max(1, warmup)):
                layer(x)
        torch.cuda.current_stream(self.device).wait_stream(side)
        torch.cuda.synchronize(self.device)
        if self._pool is None:
            self._pool = torch.cuda.graph_pool_handle()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, pool=self._pool):
            out, aux = layer(x)
        self._graphs[key] = _Graph(g, x, out, aux)

    @torch.inference_mode()
    def execute_model(self, input_ids: torch.Tensor | None,
                      hidden_states: torch.Tensor) -> torch.Tensor:
        """One step through the MoE layer: (..., hidden) -> (..., hidden).
        ``input_ids`` is accepted for interface compatibility and not used."""
        layer = self._layer()
        shape = hidden_states.shape
        h = hidden_states.reshape(-1, shape[-1])
        gr = self._graphs.get((h.shape[0], h.shape[1]))
        if gr is None:
            out, _ = layer(h)
            return out.view(shape).to(hidden_states.dtype)
        gr.x.copy_(h)
        gr.graph.replay()
        return gr.out.clone().view(shape).to(hidden_states.dtype)

    # -- profiling --------------------------------------------------------
    def enable_profiling(self) -> None:
        self._prof_start = torch.cuda.Event(enable_timing=True)
        self._prof_end = torch.cuda.Event(enable_timing=True)

    def profile_step(self, hidden_states: torch.Tensor) -> dict[str, float]:
        """One step with CUDA-event timing of the whole layer (ms)."""
        if not hasattr(self, "_prof_start"):
            self.enable_profiling()
        self._prof_start.record()
        self.execute_model(None, hidden_states)
        self._prof_end.record()
        torch.cuda.synchronize(self.device)
        return {"moe_layer_ms": self._prof_start.elapsed_time(self._prof_end)}

    def _layer(self):
        if self.moe_layer is None:
            raise RuntimeError("load_model() has not been called")
        return self.moe_layer
