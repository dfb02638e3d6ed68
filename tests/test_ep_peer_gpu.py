"""Expert-parallel peer exchange kernels, with G ranks emulated on one GPU.

Every "rank" gets its own token, row-map and output buffers on the same device,
and the address arrays the kernels take point at those buffers, so the device
plan (``lr_ep_plan``), the owner-side gather (``lr_ep_gather``) and the
token-side combine (``lr_ep_combine``) run exactly as across GPUs, one rank
after the other (none of them waits on another rank).  The concatenated
outputs must equal ``MoELayer.forward`` on the whole batch bit for bit, and the
plan must equal a numpy restatement of the global slot-order capacity rule.
"""

from __future__ import annotations

import dataclasses

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def _plan_reference(counts: np.ndarray, rank: int, C: int) -> np.ndarray:
    """numpy restatement of the plan layout documented in ``lr_ep_plan``."""
    G, E = counts.shape
    El = E // G
    base = np.cumsum(counts, axis=0) - counts
    kept = np.clip(C - base, 0, counts)
    seg_start, seg_len = np.zeros(El, np.int64), np.zeros(El, np.int64)
    row_base, src_off, kp = (np.zeros((El, G), np.int64) for _ in range(3))
    row = 0
    for el in range(El):
        e = rank * El + el
        seg_start[el] = row
        for r in range(G):
            row_base[el, r] = row + seg_len[el]
            src_off[el, r] = counts[r, :e].sum()
            kp[el, r] = kept[r, e]
            seg_len[el] += kept[r, e]
        row += seg_len[el]
    my_off = np.cumsum(counts[rank]) - counts[rank]
    my_kept = kept[rank]
    dst_row = np.zeros(E, np.int64)
    for e in range(E):
        o, el = divmod(e, El)
        dst_row[e] = kept[:, o * El:o * El + el].sum() + kept[:rank, e].sum()
    return np.concatenate([seg_start, seg_len, row_base.ravel(), src_off.ravel(), kp.ravel(),
                           my_off, my_kept, dst_row, [C]]).astype(np.int32)


@pytest.mark.parametrize("world", [1, 2, 4, 8])
@pytest.mark.parametrize("wname,overrides", [
    ("prefill", dict(tokens=2048, d_model=1024, d_ff=2048)),
    ("fine", dict(tokens=1024, d_model=512)),
    ("decode", dict(tokens=64, d_model=1024, d_ff=2048)),
    ("decode", dict(tokens=64, d_model=4096, d_ff=1024)),
])
def test_peer_exchange_emulated_matches_single_gpu(world, wname, overrides):
    from lightning_router import _ext
    from lightning_router.kernels.expert_routing import expert_capacity
    from lightning_router.workloads import WORKLOADS, build_layer
    w = dataclasses.replace(WORKLOADS[wname], **overrides)
    dev = torch.device("cuda", 0)
    layer, t = build_layer(w, device=dev)
    ops = _ext.ops()
    err = _ext.error_word(0)
    _ext.check_device_errors()
    E, k, G = w.experts, w.top_k, world
    El, T_l, d = E // G, w.tokens // G, w.d_model
    C = expert_capacity(w.tokens * k, E, w.capacity_factor)
    rows_max = El * C
    ranks = []
    for r in range(G):
        x = t.x[r * T_l:(r + 1) * T_l].contiguous()
        logits = layer.gate.logits(x)
        ids, gw, _tok, offs, _kept, _aux, psum, pos, ws = ops.topk_route(
            logits, k, 1, float(layer.gate.load_balance_weight), err)
        src = torch.zeros(T_l * k, dtype=torch.int32, device=dev)
        ops.route_rows(ids, gw, offs, pos, ws, T_l, E, src)
        ranks.append(dict(x=x, ids=ids, gw=gw, offs=offs, pos=pos, src=src,
                          y=torch.empty(rows_max, d, dtype=torch.float16, device=dev),
                          a=torch.empty(rows_max, d, dtype=torch.float16, device=dev)))
    counts = torch.stack([(rk["offs"][1:] - rk["offs"][:-1]) for rk in ranks]).int().contiguous()
    px = torch.tensor([rk["x"].data_ptr() for rk in ranks], dtype=torch.int64, device=dev)
    psrc = torch.tensor([rk["src"].data_ptr() for rk in ranks], dtype=torch.int64, device=dev)
    py = torch.tensor([rk["y"].data_ptr() for rk in ranks], dtype=torch.int64, device=dev)
    cnt_h = counts.cpu().numpy().astype(np.int64)
    for r, rk in enumerate(ranks):
        plan = ops.ep_plan(counts, r, C, err)
        assert np.array_equal(plan.cpu().numpy(), _plan_reference(cnt_h, r, C))
        a = ops.ep_gather(px, psrc, plan, E, r, T_l, T_l * k, d, rk["a"], err)
        layer.experts.forward_segments(a, plan[0:El], plan[El:2 * El], C, first_expert=r * El,
                                       num_local=El, out=rk["y"])
        rk["plan"] = plan
    outs = [ops.ep_combine(py, rk["plan"], rk["ids"], rk["gw"], rk["pos"], T_l, E, rows_max, d,
                           err) for rk in ranks]
    _ext.check_device_errors()
    full = torch.cat(outs)
    ref, _ = layer(t.x)
    assert torch.equal(full, ref), f"max |diff| {(full.float() - ref.float()).abs().max()}"


@pytest.mark.parametrize("shards,wname,overrides", [
    ([300, 212], "prefill", dict(d_model=1024, d_ff=2048)),
    ([1, 40, 0, 37], "fine", dict(d_model=512)),
    ([5, 27], "decode", dict(d_model=1024, d_ff=2048)),
])
def test_peer_exchange_unequal_shards_emulated(shards, wname, overrides):
    """Ranks with different (and empty) shards: the capacity is decided on the device
    from the gathered shard sizes (``lr_ep_plan_tokens``), buffers are sized for the
    largest shard, and the result equals the single-GPU layer on the whole batch."""
    from lightning_router import _ext
    from lightning_router.kernels.expert_routing import expert_capacity
    from lightning_router.workloads import WORKLOADS, build_layer
    T = sum(shards)
    w = dataclasses.replace(WORKLOADS[wname], tokens=T, **overrides)
    dev = torch.device("cuda", 0)
    layer, t = build_layer(w, device=dev)
    ops = _ext.ops()
    err = _ext.error_word(0)
    _ext.check_device_errors()
    E, k, G, d = w.experts, w.top_k, len(shards), w.d_model
    El = E // G
    T_max = max(shards)
    C = expert_capacity(T * k, E, w.capacity_factor)
    C_max = expert_capacity(T_max * G * k, E, w.capacity_factor)
    rows_max = El * C_max
    ranks, lo = [], 0
    for r, Tl in enumerate(shards):
        rk = dict(T=Tl, x=torch.zeros(T_max, d, dtype=torch.float16, device=dev),
                  src=torch.zeros(T_max * k, dtype=torch.int32, device=dev),
                  y=torch.empty(rows_max, d, dtype=torch.float16, device=dev),
                  a=torch.empty(rows_max, d, dtype=torch.float16, device=dev),
                  cnt=torch.zeros(E, dtype=torch.int32, device=dev))
        if Tl:
            x = t.x[lo:lo + Tl].contiguous()
            logits = layer.gate.logits(x)
            ids, gw, _tok, offs, _kept, _aux, _psum, pos, ws = ops.topk_route(
                logits, k, 1, float(layer.gate.load_balance_weight), err)
            rk["x"][:Tl].copy_(x)
            ops.route_rows(ids, gw, offs, pos, ws, Tl, E, rk["src"])
            rk.update(ids=ids, gw=gw, pos=pos, cnt=(offs[1:] - offs[:-1]).int())
        ranks.append(rk)
        lo += Tl
    counts = torch.stack([rk["cnt"] for rk in ranks]).contiguous()
    sizes = torch.tensor(shards, dtype=torch.int32, device=dev)
    px = torch.tensor([rk["x"].data_ptr() for rk in ranks], dtype=torch.int64, device=dev)
    psrc = torch.tensor([rk["src"].data_ptr() for rk in ranks], dtype=torch.int64, device=dev)
    py = torch.tensor([rk["y"].data_ptr() for rk in ranks], dtype=torch.int64, device=dev)
    cnt_h = counts.cpu().numpy().astype(np.int64)
    for r, rk in enumerate(ranks):
        plan = ops.ep_plan_tokens(counts, sizes, r, k, float(w.capacity_factor), C_max, err)
        assert np.array_equal(plan.cpu().numpy(), _plan_reference(cnt_h, r, C))
        a = ops.ep_gather(px, psrc, plan, E, r, T_max, T_max * k, d, rk["a"], err)
        layer.experts.forward_segments(a, plan[0:El], plan[El:2 * El], C_max,
                                       first_expert=r * El, num_local=El, out=rk["y"])
        rk["plan"] = plan
    outs = [ops.ep_combine(py, rk["plan"], rk["ids"], rk["gw"], rk["pos"], rk["T"], E, rows_max,
                           d, err) for rk in ranks if rk["T"]]
    _ext.check_device_errors()
    full = torch.cat(outs)
    ref, _ = layer(t.x)
    # the GEMM's tile class is chosen from the buffers' row bound (C_max); these
    # cases keep it equal to the single-GPU one, so the rows match bit for bit
    assert torch.equal(full, ref), f"max |diff| {(full.float() - ref.float()).abs().max()}"


@pytest.mark.parametrize("world", [1, 2, 4, 8])
@pytest.mark.parametrize("wname,overrides", [
    ("prefill", dict(tokens=2048, d_model=1024, d_ff=2048)),
    ("fine", dict(tokens=1024, d_model=512)),
    ("decode", dict(tokens=64, d_model=1024, d_ff=2048)),
])
def test_peer_flag_exchange_emulated(world, wname, overrides):
    """The peer step as ExpertParallelMoE runs it -- publish, plan after every rank's
    flag, gather, GEMMs, outputs flag, combine after every owner's flag -- with the
    ranks emulated on one GPU: every rank's publish runs before any plan and every
    signal before any combine, so no wait depends on a later launch.  Plans equal the
    numpy restatement, aux equals the single-GPU aux, outputs equal the single GPU's."""
    from lightning_router import _ext
    from lightning_router.kernels.expert_routing import expert_capacity
    from lightning_router.workloads import WORKLOADS, build_layer
    w = dataclasses.replace(WORKLOADS[wname], **overrides)
    dev = torch.device("cuda", 0)
    layer, t = build_layer(w, device=dev)
    ops = _ext.ops()
    err = _ext.error_word(0)
    _ext.check_device_errors()
    E, k, G, d = w.experts, w.top_k, world, w.d_model
    El, T_l = E // G, w.tokens // G
    C = expert_capacity(w.tokens * k, E, w.capacity_factor)
    rows_max = El * C
    W = 1 + 2 * E
    lbw = float(layer.gate.load_balance_weight)
    ranks = []
    for r in range(G):
        x = t.x[r * T_l:(r + 1) * T_l].contiguous()
        logits = layer.gate.logits(x)
        ids, gw, _tok, offs, _kept, _aux, psum, pos, ws = ops.topk_route(logits, k, 1, lbw, err)
        src = torch.zeros(T_l * k, dtype=torch.int32, device=dev)
        ops.route_rows(ids, gw, offs, pos, ws, T_l, E, src)
        ranks.append(dict(x=x, ids=ids, gw=gw, offs=offs, psum=psum, pos=pos, src=src,
                          y=torch.empty(rows_max, d, dtype=torch.float16, device=dev),
                          a=torch.empty(rows_max, d, dtype=torch.float16, device=dev),
                          stats=torch.zeros(G, W, dtype=torch.float64, device=dev),
                          flags=torch.zeros(2 * G, dtype=torch.int32, device=dev)))
    addr = lambda key: torch.tensor([rk[key].data_ptr() for rk in ranks], dtype=torch.int64,
                                    device=dev)
    px, psrc, py, pstats, pflags = (addr(n) for n in ("x", "src", "y", "stats", "flags"))
    counts = torch.stack([(rk["offs"][1:] - rk["offs"][:-1]) for rk in ranks]).int()
    cnt_h = counts.cpu().numpy().astype(np.int64)
    ref, ref_aux = layer(t.x)
    for epoch in (1, 2):  # the flags carry the step number: a second step reuses them
        for r, rk in enumerate(ranks):
            ops.ep_publish(pstats, pflags, rk["offs"], rk["psum"], T_l, E, r, epoch)
        for r, rk in enumerate(ranks):
            plan, aux = ops.ep_plan_wait(rk["stats"], rk["flags"], E, r, k,
                                         float(w.capacity_factor), C, lbw, epoch, err)
            assert np.array_equal(plan.cpu().numpy(), _plan_reference(cnt_h, r, C))
            assert abs(float(aux) - float(ref_aux)) <= 1e-5 * abs(float(ref_aux))
            a = ops.ep_gather(px, psrc, plan, E, r, T_l, T_l * k, d, rk["a"], err)
            layer.experts.forward_segments(a, plan[0:El], plan[El:2 * El], C,
                                           first_expert=r * El, num_local=El, out=rk["y"])
            rk["plan"] = plan
        for r in range(G):
            ops.ep_signal(pflags, r, epoch)
        outs = [ops.ep_combine(py, rk["plan"], rk["ids"], rk["gw"], rk["pos"], T_l, E, rows_max,
                               d, err, rk["flags"][G:], epoch) for rk in ranks]
        _ext.check_device_errors()
        full = torch.cat(outs)
        assert torch.equal(full, ref), f"max |diff| {(full.float() - ref.float()).abs().max()}"


def test_missing_peer_flag_times_out_with_an_error():
    """A rank whose peers never publish: the bounded wait ends with
    LR_DEVERR_PEER_TIMEOUT and a plan that keeps no rows (no hang, no fault)."""
    import time

    from lightning_router import _ext
    dev = torch.device("cuda", 0)
    ops = _ext.ops()
    err = _ext.error_word(0)
    _ext.check_device_errors()
    G, E = 2, 8
    stats = torch.zeros(G, 1 + 2 * E, dtype=torch.float64, device=dev)
    flags = torch.zeros(2 * G, dtype=torch.int32, device=dev)
    flags[0] = 1  # this rank published; rank 1 never does
    t0 = time.time()
    plan, aux = ops.ep_plan_wait(stats, flags, E, 0, 2, 1.25, 64, 0.01, 1, err)
    torch.cuda.synchronize()
    assert time.time() - t0 < 60
    v = int(err.item())
    err.zero_()
    assert v & 0x10, hex(v)
    El = E // G
    assert int(plan[El:2 * El].sum()) == 0 and float(aux) == 0.0
