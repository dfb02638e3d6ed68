"""Serving workers: one GPU, or expert-parallel with one process per GPU.

``LightningRouterWorker`` keeps the reference's single-GPU worker interface
(``lightning_router/serving/worker.py:22-78``: ``init_device``, ``load_model``,
``execute_model``) over :class:`LightningModelRunner`; decode shapes listed in
``serving_config["cuda_graph_tokens"]`` are captured as CUDA graphs at load.

The reference's ``TensorParallelGroup`` (``worker.py:81-186``) drives every GPU
from one process, runs every expert on every GPU and adds the copies, which
gives ``tp_size`` times the layer output.  :class:`ExpertParallelWorker` is its
replacement under a one-process-per-GPU launcher (torchrun): rank r holds the
experts ``[r*E/G, (r+1)*E/G)`` of the layer, takes its own token shard and
exchanges tokens with the other ranks
(:class:`lightning_router.serving.ep.ExpertParallelMoE`), so the ranks'
outputs concatenate to the single-GPU layer output.
"""

from __future__ import annotations

import logging
from typing import Any

import torch

from lightning_router.serving.model_runner import LightningModelRunner

logger = logging.getLogger(__name__)


class LightningRouterWorker:
    """One GPU running the MoE layer through :class:`LightningModelRunner`."""

    def __init__(self, model_config: dict[str, Any], moe_config: dict[str, Any],
                 quant_config: dict[str, Any], kernel_config: dict[str, Any],
                 serving_config: dict[str, Any], local_rank: int = 0):
        self.local_rank = local_rank
        self.serving_config = dict(serving_config)
        self.runner = LightningModelRunner(model_config=model_config, moe_config=moe_config,
                                           quant_config=quant_config,
                                           kernel_config=kernel_config,
                                           device=f"cuda:{local_rank}")

    def init_device(self) -> None:
        torch.cuda.set_device(self.local_rank)
        logger.info("Worker %d: GPU %s", self.local_rank,
                    torch.cuda.get_device_name(self.local_rank))

    def load_model(self, checkpoint_path: str | None = None) -> None:
        self.runner.load_model(checkpoint_path)
        for n in self.serving_config.get("cuda_graph_tokens", ()):
            self.runner.capture(int(n))

    @torch.inference_mode()
    def execute_model(self, input_ids: torch.Tensor | None,
                      hidden_states: torch.Tensor) -> torch.Tensor:
        return self.runner.execute_model(input_ids, hidden_states)


class ExpertParallelWorker(LightningRouterWorker):
    """Rank ``rank`` of ``world`` expert-parallel workers (one process per GPU, an
    initialised ``torch.distributed`` NCCL group).  ``execute_model`` takes this
    rank's token shard and returns its output rows."""

    def __init__(self, model_config: dict[str, Any], moe_config: dict[str, Any],
                 quant_config: dict[str, Any], kernel_config: dict[str, Any],
                 serving_config: dict[str, Any], rank: int, world: int,
                 local_rank: int | None = None, group=None):
        super().__init__(model_config, moe_config, quant_config, kernel_config, serving_config,
                         local_rank=rank if local_rank is None else local_rank)
        self.rank, self.world, self.group = rank, world, group
        self.ep = None

    def load_model(self, checkpoint_path: str | None = None) -> None:
        from lightning_router.serving.ep import ExpertParallelMoE
        self.runner.load_model(checkpoint_path)
        self.ep = ExpertParallelMoE.from_layer(
            self.runner.moe_layer, self.world, self.rank, group=self.group,
            exchange=self.serving_config.get("ep_exchange", "peer"))

    @torch.inference_mode()
    def execute_model(self, input_ids: torch.Tensor | None,
                      hidden_states: torch.Tensor) -> torch.Tensor:
        if self.ep is None:
            raise RuntimeError("load_model() has not been called")
        shape = hidden_states.shape
        out, _ = self.ep.forward(hidden_states.reshape(-1, shape[-1]))
        return out.view(shape).to(hidden_states.dtype)

    def shutdown(self) -> None:
        """Unmap the peers' exchange buffers (before destroying the process group)."""
        if self.ep is not None:
            self.ep.close()
