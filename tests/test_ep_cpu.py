"""Expert-parallel exchange logic on CPU ``gloo`` ranks (no GPU).

Each rank routes its token shard with the oracle's gating, applies the global
slot-order capacity through ``plan_exchange``, exchanges kept rows with
``all_to_all_single``, runs its local experts (oracle FFN), returns the rows
and combines.  The gathered result must equal the single-process oracle:
routing (kept slots) exactly, outputs to fp32 rounding.

A second test makes a rank fail on the host before the exchange and checks
that the surviving rank's collective ends with an error within the process
group timeout instead of waiting forever.
"""

from __future__ import annotations

import datetime
import os
import socket
import traceback

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

import oracle as orc


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _problem(T, d, f, E, k, seed):
    rng = np.random.default_rng(seed)
    x = rng.standard_normal((T, d)).astype(np.float16)
    logits = (rng.standard_normal((T, E)) + np.linspace(1.0, -1.0, E)).astype(np.float32)
    experts = []
    for _ in range(E):
        experts.append({
            "gate": (rng.standard_normal((d, f)) * 0.05).astype(np.float16),
            "up": (rng.standard_normal((d, f)) * 0.05).astype(np.float16),
            "down": (rng.standard_normal((f, d)) * 0.05).astype(np.float16),
        })
    return x, logits, experts


def _rank_main(rank, world, port, cfg, q):
    try:
        from lightning_router.serving.ep import plan_exchange
        os.environ["MASTER_ADDR"] = "127.0.0.1"
        os.environ["MASTER_PORT"] = str(port)
        dist.init_process_group("gloo", rank=rank, world_size=world,
                                timeout=datetime.timedelta(seconds=30))
        T, d, f, E, k, cf, seed = cfg
        x, logits, experts = _problem(T, d, f, E, k, seed)
        Tl = T // world
        xs, ls = x[rank * Tl:(rank + 1) * Tl], logits[rank * Tl:(rank + 1) * Tl]
        ids, w, probs = orc.topk_gating(ls, k)
        ids, w = ids.reshape(-1), w.reshape(-1)
        counts = np.bincount(ids, minlength=E)
        stats_l = np.concatenate([[Tl], counts, probs.astype(np.float64).sum(0)]).astype(np.float64)
        stats = torch.zeros(world * (1 + 2 * E), dtype=torch.float64)
        dist.all_gather_into_tensor(stats, torch.from_numpy(stats_l))
        plan = plan_exchange(stats.view(world, -1).numpy(), rank, world, E, k, cf, 0.01)
        # local slot ranks in slot order, kept iff base + rank < C, compact rows
        order = np.argsort(ids, kind="stable")
        local_rank = np.empty_like(ids)
        starts = np.concatenate([[0], np.cumsum(counts)])
        local_rank[order] = np.arange(ids.size) - starts[ids[order]]
        kept = plan.rank_base[ids] + local_rank < plan.capacity
        send = np.zeros((plan.n_send, d), np.float16)
        pos = np.full(ids.size, -1, np.int64)
        tok = np.repeat(np.arange(Tl), k)
        for s in np.nonzero(kept)[0]:
            pos[s] = plan.koff[ids[s]] + local_rank[s]
            send[pos[s]] = xs[tok[s]]
        recv = torch.zeros(plan.n_recv, d, dtype=torch.float16)
        dist.all_to_all_single(recv, torch.from_numpy(send), plan.recv_rows, plan.send_rows)
        rr = recv.numpy()
        a = rr[plan.reorder] if plan.reorder is not None else rr
        El = E // world
        y = np.zeros((plan.n_recv, d), np.float32)
        for el in range(El):
            st, n = int(plan.seg_start[el]), int(plan.seg_len[el])
            if n:
                ex = experts[rank * El + el]
                y[st:st + n] = orc.expert_ffn(a[st:st + n], ex["up"], ex["down"], ex["gate"])
        if plan.reorder is not None:
            y_send = np.empty_like(y)
            y_send[plan.reorder] = y
        else:
            y_send = y
        back = torch.zeros(plan.n_send, d, dtype=torch.float32)
        dist.all_to_all_single(back, torch.from_numpy(y_send), plan.send_rows, plan.recv_rows)
        bk = back.numpy()
        out = np.zeros((Tl, d), np.float32)
        for s in np.nonzero(kept)[0]:
            out[tok[s]] += w[s] * bk[pos[s]]
        full = [torch.zeros(Tl, d) for _ in range(world)]
        dist.all_gather(full, torch.from_numpy(out))
        kept_all = [torch.zeros(Tl * k, dtype=torch.int64) for _ in range(world)]
        dist.all_gather(kept_all, torch.from_numpy(kept.astype(np.int64)))
        if rank == 0:
            q.put(("ok", torch.cat(full).numpy(), torch.cat(kept_all).numpy(), plan.aux_loss))
        dist.destroy_process_group()
    except Exception:
        q.put(("err", traceback.format_exc(), None, None))


@pytest.mark.parametrize("world,E,k,cf", [(2, 4, 2, 1.0), (2, 8, 2, 1.25), (4, 8, 3, 0.75),
                                          (2, 2, 1, 2.0)])
def test_ep_exchange_matches_single_process_oracle(world, E, k, cf):
    T, d, f = 48 * world, 32, 48
    cfg = (T, d, f, E, k, cf, 1234 + world + E)
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, world, port, cfg, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = q.get(timeout=120)
    for p in procs:
        p.join(timeout=60)
    assert res[0] == "ok", res[1]
    _, got, kept_got, aux_got = res
    x, logits, experts = _problem(T, d, f, E, k, cfg[-1])
    ref, aux, r = orc.moe_layer(x, logits, k, cf, experts)
    np.testing.assert_array_equal(kept_got.astype(bool), r.kept)
    np.testing.assert_allclose(got, ref, rtol=1e-5, atol=1e-5)
    assert abs(aux_got - aux) <= 1e-9 + 1e-7 * abs(aux)


def _failing_rank(rank, world, port, q):
    try:
        os.environ["MASTER_ADDR"] = "127.0.0.1"
        os.environ["MASTER_PORT"] = str(port)
        dist.init_process_group("gloo", rank=rank, world_size=world,
                                timeout=datetime.timedelta(seconds=4))
        if rank == 1:
            raise SystemExit(3)  # host-side failure before the exchange
        t = torch.zeros(4)
        try:
            dist.all_to_all_single(t, torch.ones(4), [2, 2], [2, 2])
            q.put(("no-error", None))
        except Exception as e:  # the peer is gone: the collective must fail, not hang
            q.put(("error", type(e).__name__))
    except SystemExit:
        raise
    except Exception:
        q.put(("setup-error", traceback.format_exc()))


def test_dead_rank_is_detected_by_timeout():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_failing_rank, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    status, info = q.get(timeout=90)
    for p in procs:
        p.join(timeout=30)
        if p.is_alive():
            p.kill()
    assert status == "error", (status, info)


@pytest.mark.parametrize("world,nchunks,E,k,cf", [(2, 2, 4, 2, 1.0), (4, 2, 8, 2, 0.8),
                                                  (8, 2, 64, 6, 1.5), (2, 3, 8, 3, 1.25)])
def test_microbatch_plans_follow_global_slot_order(world, nchunks, E, k, cf):
    """Kept slots of every (rank, micro-batch) shard equal the single-process capacity rule,
    and the exchange sizes agree between senders and receivers."""
    from lightning_router.serving.ep import plan_exchanges
    rng = np.random.default_rng(world * 100 + E)
    Ts = rng.integers(5, 60, size=world * nchunks)
    logits = [rng.standard_normal((int(t), E)).astype(np.float32) + np.linspace(1, -1, E)
              for t in Ts]
    ids = [orc.topk_gating(l, k)[0].reshape(-1) for l in logits]
    stats = np.stack([np.concatenate([[ids_i.size // k], np.bincount(ids_i, minlength=E),
                                      np.zeros(E)]) for ids_i in ids]).astype(np.float64)
    plans = [plan_exchanges(stats, r, world, E, k, cf, 0.01, nchunks) for r in range(world)]
    all_ids = np.concatenate(ids)
    C = orc.capacity(all_ids.size, E, cf)
    r_ref = orc.dispatch(all_ids, np.ones(all_ids.size, np.float32),
                         np.zeros(all_ids.size, np.int32), E, C)
    got, El = [], E // world
    for r in range(world):
        for c in range(nchunks):
            p = plans[r][c]
            assert p.capacity == C
            loc = ids[r * nchunks + c]
            order = np.argsort(loc, kind="stable")
            cnt = np.bincount(loc, minlength=E)
            lr = np.empty_like(loc)
            lr[order] = np.arange(loc.size) - (np.cumsum(cnt) - cnt)[loc[order]]
            kept = p.rank_base[loc] + lr < C
            got.append(kept)
            assert p.n_send == int(kept.sum())
            # what rank r sends to q in micro-batch c is what q receives from r
            for q in range(world):
                assert plans[q][c].recv_rows[r] == p.send_rows[q]
            if p.reorder is not None:
                assert sorted(p.reorder.tolist()) == list(range(p.n_recv))
            assert int(p.seg_len.sum()) == p.n_recv
    np.testing.assert_array_equal(np.concatenate(got), r_ref.kept)


def _rank_main_chunks(rank, world, port, cfg, q):
    """One rank of the NCCL exchange's host logic with unequal shards and
    micro-batches: every rank splits its shard with ``microbatch_bounds`` into the
    same number of micro-batches (some may be empty), gathers one statistics row
    per micro-batch, and exchanges each micro-batch's kept rows."""
    try:
        from lightning_router.serving.ep import microbatch_bounds, plan_exchanges
        os.environ["MASTER_ADDR"] = "127.0.0.1"
        os.environ["MASTER_PORT"] = str(port)
        dist.init_process_group("gloo", rank=rank, world_size=world,
                                timeout=datetime.timedelta(seconds=30))
        shards, nc, d, f, E, k, cf, seed = cfg
        T = sum(shards)
        x, logits, experts = _problem(T, d, f, E, k, seed)
        lo0 = sum(shards[:rank])
        xs, ls = x[lo0:lo0 + shards[rank]], logits[lo0:lo0 + shards[rank]]
        bounds = microbatch_bounds(shards[rank], nc)
        routes, stats_l = [], []
        for c in range(nc):
            lo, hi = bounds[c], bounds[c + 1]
            if hi == lo:
                routes.append(None)
                stats_l.append(np.zeros(1 + 2 * E))
                continue
            ids, w, probs = orc.topk_gating(ls[lo:hi], k)
            ids, w = ids.reshape(-1), w.reshape(-1)
            routes.append((ids, w))
            stats_l.append(np.concatenate([[hi - lo], np.bincount(ids, minlength=E),
                                           probs.astype(np.float64).sum(0)]))
        stats_l = torch.from_numpy(np.concatenate(stats_l).astype(np.float64))
        stats = torch.zeros(world * stats_l.numel(), dtype=torch.float64)
        dist.all_gather_into_tensor(stats, stats_l)  # equal sizes on every rank
        plans = plan_exchanges(stats.view(world * nc, -1).numpy(), rank, world, E, k, cf, 0.01,
                               nc)
        out = np.zeros((shards[rank], d), np.float32)
        kept_l = []
        El = E // world
        for c, plan in enumerate(plans):
            lo, hi = bounds[c], bounds[c + 1]
            send = np.zeros((plan.n_send, d), np.float16)
            if routes[c] is not None:
                ids, w = routes[c]
                counts = np.bincount(ids, minlength=E)
                order = np.argsort(ids, kind="stable")
                local_rank = np.empty_like(ids)
                local_rank[order] = np.arange(ids.size) - (np.cumsum(counts) - counts)[ids[order]]
                kept = plan.rank_base[ids] + local_rank < plan.capacity
                pos = np.full(ids.size, -1, np.int64)
                tok = np.repeat(np.arange(hi - lo), k)
                for s_ in np.nonzero(kept)[0]:
                    pos[s_] = plan.koff[ids[s_]] + local_rank[s_]
                    send[pos[s_]] = xs[lo + tok[s_]]
                kept_l.append(kept)
            recv = torch.zeros(plan.n_recv, d, dtype=torch.float16)
            dist.all_to_all_single(recv, torch.from_numpy(send), plan.recv_rows, plan.send_rows)
            rr = recv.numpy()
            a = rr[plan.reorder] if plan.reorder is not None else rr
            y = np.zeros((plan.n_recv, d), np.float32)
            for el in range(El):
                st, n = int(plan.seg_start[el]), int(plan.seg_len[el])
                if n:
                    ex = experts[rank * El + el]
                    y[st:st + n] = orc.expert_ffn(a[st:st + n], ex["up"], ex["down"], ex["gate"])
            y_send = np.empty_like(y)
            if plan.reorder is not None:
                y_send[plan.reorder] = y
            else:
                y_send = y
            back = torch.zeros(plan.n_send, d, dtype=torch.float32)
            dist.all_to_all_single(back, torch.from_numpy(y_send), plan.send_rows,
                                   plan.recv_rows)
            if routes[c] is not None:
                bk = back.numpy()
                for s_ in np.nonzero(kept)[0]:
                    out[lo + tok[s_]] += w[s_] * bk[pos[s_]]
        full = [None] * world
        dist.all_gather_object(full, (out, np.concatenate(kept_l) if kept_l else
                                      np.zeros(0, bool), plans[0].aux_loss))
        if rank == 0:
            q.put(("ok", np.concatenate([f_[0] for f_ in full]),
                   np.concatenate([f_[1] for f_ in full]), full[0][2]))
        dist.destroy_process_group()
    except Exception:
        q.put(("err", traceback.format_exc(), None, None))


@pytest.mark.parametrize("shards,nc,E,k,cf", [([70, 9], 2, 4, 2, 1.0), ([0, 96], 2, 8, 2, 1.25),
                                              ([33, 1, 50, 2], 2, 8, 2, 0.9),
                                              ([5, 40], 3, 4, 1, 1.5)])
def test_unequal_shards_with_microbatches_match_oracle(shards, nc, E, k, cf):
    """Unequal (and empty) shards with several micro-batches: the statistics rows
    agree in number across ranks, and the result equals the single-process oracle."""
    world = len(shards)
    cfg = (shards, nc, 32, 48, E, k, cf, 4321 + sum(shards))
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_main_chunks, args=(r, world, port, cfg, q))
             for r in range(world)]
    for p in procs:
        p.start()
    res = q.get(timeout=120)
    for p in procs:
        p.join(timeout=60)
    assert res[0] == "ok", res[1]
    _, got, kept_got, aux_got = res
    x, logits, experts = _problem(sum(shards), 32, 48, E, k, cfg[-1])
    ref, aux, r = orc.moe_layer(x, logits, k, cf, experts)
    np.testing.assert_array_equal(kept_got.astype(bool), r.kept)
    np.testing.assert_allclose(got, ref, rtol=1e-5, atol=1e-5)
    assert abs(aux_got - aux) <= 1e-9 + 1e-7 * abs(aux)


def test_microbatch_bounds_are_rank_independent():
    from lightning_router.serving.ep import microbatch_bounds
    for T in (0, 1, 5, 255, 256, 4096):
        for nc in (1, 2, 3):
            b = microbatch_bounds(T, nc)
            assert len(b) == nc + 1 and b[0] == 0 and b[-1] == T
            assert all(b[i] <= b[i + 1] for i in range(nc))
