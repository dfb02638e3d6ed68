"""HostPipeline: overlapped host->device / device->host copies give the same
outputs as running each batch on its own, for every batch and buffer reuse."""

from __future__ import annotations

import dataclasses

import pytest
import torch

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("depth", [1, 2, 3])
def test_pipeline_matches_per_batch_runs(depth):
    from lightning_router.serving.pipeline import HostPipeline
    from lightning_router.workloads import WORKLOADS, build_layer
    w = dataclasses.replace(WORKLOADS["pr1"], tokens=512)
    dev = torch.device("cuda", 0)
    layer, t = build_layer(w, device=dev)
    gen = torch.Generator().manual_seed(7)
    inputs = [torch.randn(w.tokens, w.d_model, generator=gen).half().pin_memory()
              for _ in range(5)]
    outputs = [torch.full((w.tokens, w.d_model), 9.0, dtype=torch.float16).pin_memory()
               for _ in range(5)]
    pipe = HostPipeline(layer.forward, inputs[0], dev, depth=depth)
    pipe.run(inputs, outputs)
    for xi, oi in zip(inputs, outputs):
        ref, _ = layer(xi.to(dev))
        assert torch.equal(oi, ref.cpu())
