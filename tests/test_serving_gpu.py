"""Serving runner and worker (reference ``serving/model_runner.py``,
``serving/worker.py`` interfaces): a checkpoint round trip through
``load_model``, eager steps equal to ``MoELayer.forward``, and CUDA-graph
replays of captured decode shapes equal to eager steps bit for bit."""

from __future__ import annotations

import dataclasses

import pytest
import torch

pytestmark = pytest.mark.gpu


def _configs(w):
    model = dict(hidden_size=w.d_model, intermediate_size=w.d_ff)
    moe = dict(num_experts=w.experts, num_experts_per_token=w.top_k,
               expert_capacity_factor=w.capacity_factor, expert_activation=w.activation,
               gate_bias=w.zipf_s > 0)
    quant = dict(group_size=w.group_size)
    return model, moe, quant, {}


@pytest.fixture(scope="module")
def checkpoint(tmp_path_factory):
    from lightning_router.workloads import WORKLOADS, build_layer
    w = dataclasses.replace(WORKLOADS["decode"], d_model=1024, d_ff=2048)
    layer, t = build_layer(w, device="cuda")
    path = tmp_path_factory.mktemp("ckpt") / "moe.pt"
    torch.save({k: v.cpu() for k, v in layer.state_dict().items()}, path)
    return w, layer, path


def test_runner_loads_checkpoint_and_matches_layer(checkpoint):
    from lightning_router.serving.model_runner import LightningModelRunner
    w, layer, path = checkpoint
    r = LightningModelRunner(*_configs(w), device="cuda:0")
    r.load_model(path)
    x = torch.randn(2, 48, w.d_model, device="cuda").half()
    out = r.execute_model(None, x)
    ref, _ = layer(x.reshape(-1, w.d_model))
    assert out.shape == x.shape
    assert torch.equal(out.reshape(-1, w.d_model), ref)
    assert r.profile_step(x)["moe_layer_ms"] > 0


@pytest.mark.parametrize("tokens", [1, 64, 256])
def test_graph_replay_matches_eager(checkpoint, tokens):
    from lightning_router.serving.model_runner import LightningModelRunner
    w, layer, path = checkpoint
    r = LightningModelRunner(*_configs(w), device="cuda:0")
    r.load_model(path)
    r.capture(tokens)
    gen = torch.Generator(device="cuda").manual_seed(tokens)
    for _ in range(3):   # replays with fresh inputs
        x = torch.randn(tokens, w.d_model, device="cuda", generator=gen).half()
        out = r.execute_model(None, x)
        ref, _ = r.moe_layer(x)
        assert torch.equal(out, ref)


def test_worker_interface(checkpoint):
    from lightning_router.serving.worker import LightningRouterWorker
    w, layer, path = checkpoint
    wk = LightningRouterWorker(*_configs(w), serving_config={"cuda_graph_tokens": [32]},
                               local_rank=0)
    wk.init_device()
    wk.load_model(str(path))
    for T in (32, 40):   # a captured shape and an eager one
        x = torch.randn(T, w.d_model, device="cuda").half()
        out = wk.execute_model(None, x)
        ref, _ = layer(x)
        assert torch.equal(out, ref)


@pytest.mark.parametrize("tokens", [64, 200])
def test_runner_steps_match_oracle(checkpoint, tokens):
    """The runner's eager step and its CUDA-graph replay against the CPU oracle:
    routing bit-exact given the kernel's fp32 gate logits, outputs within max-abs
    2e-2 and relative L2 1e-3 of the fp32 dequant-then-matmul layer."""
    import numpy as np

    import oracle as orc
    from lightning_router.serving.model_runner import LightningModelRunner
    w, layer, path = checkpoint
    r = LightningModelRunner(*_configs(w), device="cuda:0")
    r.load_model(path)
    r.capture(tokens)
    x = torch.randn(tokens, w.d_model, device="cuda",
                    generator=torch.Generator(device="cuda").manual_seed(7 + tokens)).half()
    eager, _ = r.moe_layer(x)
    replay = r.execute_model(None, x)
    assert torch.equal(replay, eager)
    logits, plan = r.moe_layer.route(x)
    experts = []
    for ex in r.moe_layer.experts.experts:
        q, s, z = ex.quant_tensors()
        experts.append({m: orc.dequantize_tensor(q[i].cpu().numpy(), s[i].cpu().numpy(),
                                                 z[i].cpu().numpy(), w.group_size, s[i].shape[1])
                        for i, m in enumerate(("gate", "up", "down")) if q[i] is not None})
    ref, _, rr = orc.moe_layer(x.cpu().numpy(), logits.cpu().numpy(), w.top_k,
                               w.capacity_factor, experts)
    np.testing.assert_array_equal(plan.slot_pos.cpu().numpy(), rr.slot_pos)
    got = replay.float().cpu().numpy()
    assert np.abs(got - ref).max() <= 2e-2
    assert np.linalg.norm(got - ref) / np.linalg.norm(ref) <= 1e-3
