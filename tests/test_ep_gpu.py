"""Expert-parallel layer on 2+ GPUs (NCCL) against the single-GPU layer.

Each rank builds the same seeded layer, runs ``ExpertParallelMoE.forward`` on
its token shard, and rank 0 compares the gathered output with
``MoELayer.forward`` on the whole batch: bit-identical (every kept row goes
through the same kernels and the combine sums in the same slot order), with
the same routing and an aux loss equal to 1e-6 relative.  Skipped when fewer
GPUs than ranks are visible.
"""

from __future__ import annotations

import dataclasses
import datetime
import os
import socket
import traceback

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, wname, overrides, exchange, q, shards=None):
    try:
        os.environ["MASTER_ADDR"] = "127.0.0.1"
        os.environ["MASTER_PORT"] = str(port)
        torch.cuda.set_device(rank)
        dev = torch.device("cuda", rank)
        dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev,
                                timeout=datetime.timedelta(seconds=120))
        from lightning_router.serving.ep import ExpertParallelMoE
        from lightning_router.workloads import WORKLOADS, build_layer
        w = dataclasses.replace(WORKLOADS[wname], **overrides)
        layer, t = build_layer(w, device=dev)
        if shards is None:
            shards = [w.tokens // world] * world
        lo = sum(shards[:rank])
        x_l = t.x[lo:lo + shards[rank]]
        ep = ExpertParallelMoE.from_layer(layer, world, rank, exchange=exchange)
        out, aux = ep.forward(x_l)
        out2, _ = ep.forward(x_l)
        same = bool(torch.equal(out, out2))
        # equal-size gather (shards may differ): pad to the largest shard
        pad = torch.zeros(max(shards), w.d_model, dtype=out.dtype, device=dev)
        pad[:out.shape[0]].copy_(out)
        padded = [torch.empty_like(pad) for _ in range(world)]
        dist.all_gather(padded, pad)
        gathered = [p[:n] for p, n in zip(padded, shards)]
        if rank == 0:
            ref, ref_aux = layer(t.x)
            full = torch.cat(gathered)
            q.put(("ok", bool(torch.equal(full, ref)), float((full.float() - ref.float()).abs().max()),
                   float(aux), float(ref_aux), same))
        dist.barrier()
        ep.close()
        dist.destroy_process_group()
    except Exception:
        q.put(("err", traceback.format_exc(), None, None, None, None))


@pytest.mark.parametrize("exchange", ["peer", "nccl"])
@pytest.mark.parametrize("world", [2, 4, 8])
@pytest.mark.parametrize("wname,overrides", [
    ("prefill", dict(tokens=2048, d_model=1024, d_ff=2048)),
    ("fine", dict(tokens=1024, d_model=512)),
])
def test_expert_parallel_matches_single_gpu(world, wname, overrides, exchange):
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, wname, overrides, exchange, q))
             for r in range(world)]
    for p in procs:
        p.start()
    res = q.get(timeout=600)
    for p in procs:
        p.join(timeout=120)
        if p.is_alive():
            p.kill()
    assert res[0] == "ok", res[1]
    _, equal, maxdiff, aux, ref_aux, repeat_same = res
    assert repeat_same
    assert equal, f"EP output differs from single GPU (max |diff| {maxdiff})"
    assert abs(aux - ref_aux) <= 1e-6 * abs(ref_aux)


@pytest.mark.parametrize("exchange", ["peer", "nccl"])
@pytest.mark.parametrize("shards", [[1200, 848], [700, 0, 900, 448]])
def test_expert_parallel_unequal_shards(shards, exchange):
    """Ranks with different (and empty) token shards: the peer exchange decides the
    capacity on the device from the gathered sizes, the NCCL exchange plans on the
    host; both match the single-GPU layer on the whole batch bit for bit (the shard
    limit keeps the GEMM's tile class, so the per-row arithmetic is the same)."""
    world = len(shards)
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    over = dict(tokens=sum(shards), d_model=1024, d_ff=2048)
    procs = [ctx.Process(target=_worker, args=(r, world, port, "prefill", over, exchange, q, shards))
             for r in range(world)]
    for p in procs:
        p.start()
    res = q.get(timeout=600)
    for p in procs:
        p.join(timeout=120)
        if p.is_alive():
            p.kill()
    assert res[0] == "ok", res[1]
    _, equal, maxdiff, aux, ref_aux, repeat_same = res
    assert repeat_same
    assert equal, f"EP output differs from single GPU (max |diff| {maxdiff})"
    assert abs(aux - ref_aux) <= 1e-6 * abs(ref_aux)


def _worker_ep(rank, world, port, ckpt_dir, q):
    """One rank of ExpertParallelWorker (the replacement of the reference's
    TensorParallelGroup, serving/worker.py:81-186) loading a checkpoint through
    its own interface."""
    try:
        os.environ["MASTER_ADDR"] = "127.0.0.1"
        os.environ["MASTER_PORT"] = str(port)
        torch.cuda.set_device(rank)
        dev = torch.device("cuda", rank)
        dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev,
                                timeout=datetime.timedelta(seconds=120))
        from lightning_router.serving.worker import ExpertParallelWorker
        from lightning_router.workloads import WORKLOADS, build_layer
        w = dataclasses.replace(WORKLOADS["prefill"], tokens=1024, d_model=1024, d_ff=2048)
        layer, t = build_layer(w, device=dev)
        path = os.path.join(ckpt_dir, f"moe{rank}.pt")
        torch.save({k: v.cpu() for k, v in layer.state_dict().items()}, path)
        cfg = (dict(hidden_size=w.d_model, intermediate_size=w.d_ff),
               dict(num_experts=w.experts, num_experts_per_token=w.top_k,
                    expert_capacity_factor=w.capacity_factor, expert_activation=w.activation),
               dict(group_size=w.group_size), {}, {"ep_exchange": "peer"})
        wk = ExpertParallelWorker(*cfg, rank=rank, world=world)
        wk.init_device()
        wk.load_model(path)
        Tl = w.tokens // world
        out = wk.execute_model(None, t.x[rank * Tl:(rank + 1) * Tl].view(1, Tl, -1))
        gathered = [torch.empty(Tl, w.d_model, dtype=out.dtype, device=dev) for _ in range(world)]
        dist.all_gather(gathered, out.reshape(Tl, -1).contiguous())
        if rank == 0:
            ref, _ = layer(t.x)
            full = torch.cat(gathered)
            q.put(("ok", bool(torch.equal(full, ref)),
                   float((full.float() - ref.float()).abs().max()), None, None, True))
        wk.shutdown()
        dist.destroy_process_group()
    except Exception:
        q.put(("err", traceback.format_exc(), None, None, None, None))


def test_expert_parallel_worker_matches_single_gpu(tmp_path):
    world = 2
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker_ep, args=(r, world, port, str(tmp_path), q))
             for r in range(world)]
    for p in procs:
        p.start()
    res = q.get(timeout=600)
    for p in procs:
        p.join(timeout=120)
        if p.is_alive():
            p.kill()
    assert res[0] == "ok", res[1]
    assert res[1], f"ExpertParallelWorker output differs from single GPU (max |diff| {res[2]})"
