"""Expert-parallel MoE layer over NCCL (one process per GPU).

Replaces the reference's ``TensorParallelGroup.execute``
(``lightning_router/serving/worker.py:156-186``).  That runs the whole layer on
every GPU and sums the copies on the host, so its answer is ``tp_size`` times
the single-GPU output.  Here the experts are sharded and tokens move:

* rank r owns experts ``[r*E/G, (r+1)*E/G)`` and its own contiguous shard of
  the tokens (global token order = rank-major);
* every rank gates its tokens (fp32 logits, top-k, slot ranks: kernel phase 1)
  and all-gathers ``(T_r, per-expert counts, per-expert probability sums)``;
* capacity follows the GLOBAL slot order, exactly as on one GPU: rank r's base
  for expert e is the count of lower ranks, and a slot is kept iff
  ``base + local rank < C`` with ``C`` from the global slot count;
* kept rows are permuted into a compact send buffer grouped by owner rank
  (kernel phase 2), exchanged with ``all_to_all_single``, run through the
  local grouped W4A16 FFN, sent back with ``all_to_all_single`` and combined in
  token order by the same combine kernel as on one GPU.

Every kept row goes through the same per-row arithmetic as on one GPU, so the
output equals the single-GPU output bit for bit.  The exchange needs the split
sizes on the host: one device->host read of the gathered counts per forward.

:func:`plan_exchange` is the pure host part (no GPU); it is exercised by CPU
``gloo`` tests against the oracle.
"""

from __future__ import annotations

from dataclasses import dataclass

import numpy as np
import torch
import torch.distributed as dist

from lightning_router import _ext
from lightning_router.kernels.expert_routing import combine, expert_capacity


@dataclass
class ExchangePlan:
    T_total: int
    capacity: int
    rank_base: np.ndarray      # (E,) int32: slots of each expert on lower ranks
    kept: np.ndarray           # (G, E) int64: kept slots per (rank, expert)
    koff: np.ndarray           # (E+1,) int32: this rank's compact send offsets per expert
    send_rows: list            # rows this rank sends to each rank
    recv_rows: list            # rows this rank receives from each rank
    reorder: np.ndarray | None  # (n_recv,) receive position of each row in [expert][rank] order
    seg_start: np.ndarray      # (E_local,) int32 in [expert][rank] order
    seg_len: np.ndarray        # (E_local,) int32
    aux_loss: float

    @property
    def n_send(self) -> int:
        return int(sum(self.send_rows))

    @property
    def n_recv(self) -> int:
        return int(sum(self.recv_rows))


def plan_exchange(stats: np.ndarray, rank: int, world: int, num_experts: int, top_k: int,
                  capacity_factor: float, load_balance_weight: float) -> ExchangePlan:
    """Host plan from the all-gathered ``stats`` (G, 1 + 2E) float64 rows of
    ``[T_r, count_r[0..E), prob_sum_r[0..E)]``."""
    G, E = world, num_experts
    if E % G:
        raise ValueError(f"num_experts {E} must be divisible by the world size {G}")
    El = E // G
    T_r = stats[:, 0].astype(np.int64)
    counts = np.rint(stats[:, 1:1 + E]).astype(np.int64)
    psum = stats[:, 1 + E:1 + 2 * E]
    T = int(T_r.sum())
    S = T * top_k
    C = expert_capacity(S, E, capacity_factor)
    base = np.zeros_like(counts)
    base[1:] = np.cumsum(counts, axis=0)[:-1]
    kept = np.clip(C - base, 0, counts)
    koff = np.zeros(E + 1, np.int64)
    koff[1:] = np.cumsum(kept[rank])
    send_rows = [int(kept[rank, q * El:(q + 1) * El].sum()) for q in range(G)]
    mine = slice(rank * El, (rank + 1) * El)
    recv_rows = [int(kept[q, mine].sum()) for q in range(G)]
    # receive layout: [source rank][local expert]; GEMM layout: [local expert][source rank]
    recv_off = np.zeros(G + 1, np.int64)
    recv_off[1:] = np.cumsum(recv_rows)
    tot = kept[:, mine].sum(axis=0)
    seg_len = tot.astype(np.int32)
    seg_start = np.zeros(El, np.int32)
    seg_start[1:] = np.cumsum(tot)[:-1]
    reorder = None
    if El > 1:
        idx = []
        for el in range(El):
            for q in range(G):
                within = int(kept[q, rank * El:rank * El + el].sum())
                st = int(recv_off[q]) + within
                idx.append(np.arange(st, st + int(kept[q, rank * El + el]), dtype=np.int64))
        reorder = np.concatenate(idx) if idx else np.zeros(0, np.int64)
    f = counts.sum(axis=0) / float(max(S, 1))
    P = psum.sum(axis=0) / float(max(T, 1))
    aux = float(load_balance_weight * E * float((f * P).sum()))
    return ExchangePlan(T, C, base[rank].astype(np.int32), kept, koff.astype(np.int32),
                        send_rows, recv_rows, reorder, seg_start, seg_len, aux)


class ExpertParallelMoE:
    """Expert-parallel forward of a ``MoELayer`` (one rank per GPU).

    ``layer`` must hold at least this rank's experts; the other experts'
    buffers are not read.  ``forward(x_local)`` takes this rank's token shard
    (T_r, d) fp16 and returns ``(out_local, aux_loss)`` for the whole job's
    routing (aux is the global load-balancing loss).
    """

    def __init__(self, layer, world: int, rank: int, group=None):
        if layer.num_experts % world:
            raise ValueError("num_experts must be divisible by the world size")
        self.layer = layer
        self.world = world
        self.rank = rank
        self.group = group
        self.E = layer.num_experts
        self.El = self.E // world
        self.k = layer.top_k
        self.cf = layer.moe_cfg.expert_capacity_factor
        self.lbw = layer.gate.load_balance_weight
        self.stage_events: list | None = None
        self._last_recv = 0

    @classmethod
    def from_layer(cls, layer, world: int, rank: int, group=None) -> "ExpertParallelMoE":
        return cls(layer, world, rank, group)

    def _mark(self, name):
        if self.stage_events is not None:
            ev = torch.cuda.Event(enable_timing=True)
            ev.record()
            self.stage_events.append((name, ev))

    def last_kept_rows(self) -> int:
        return self._last_recv

    @torch.no_grad()
    def forward(self, x: torch.Tensor):
        ops = _ext.ops()
        dev = x.device
        x = x.reshape(-1, x.shape[-1]).to(torch.float16).contiguous()
        T_l, d = x.shape
        E, G = self.E, self.world
        err = _ext.error_word(dev.index)
        self._mark("begin")
        logits = self.layer.gate.logits(x)
        self._mark("gate")
        ids, gw, _tok, offs, _kept, _aux, psum, pos, ws = ops.topk_route(
            logits, self.k, 1, float(self.lbw), err)
        stats_l = torch.cat([torch.full((1,), float(T_l), dtype=torch.float64, device=dev),
                             (offs[1:] - offs[:-1]).double(), psum])
        stats = torch.empty(G * (1 + 2 * E), dtype=torch.float64, device=dev)
        dist.all_gather_into_tensor(stats, stats_l, group=self.group)
        plan = plan_exchange(stats.view(G, -1).cpu().numpy(), self.rank, G, E, self.k, self.cf,
                             self.lbw)
        meta_h = np.concatenate([plan.rank_base, plan.koff, plan.seg_start, plan.seg_len])
        meta = torch.from_numpy(meta_h.astype(np.int32)).pin_memory().to(dev, non_blocking=True)
        rank_base = meta[:E]
        koff = meta[E:2 * E + 1]
        seg_start = meta[2 * E + 1:2 * E + 1 + self.El]
        seg_len = meta[2 * E + 1 + self.El:]
        n_send, n_recv = plan.n_send, plan.n_recv
        send, _rw, _src = ops.permute_tokens(x, ids, gw, koff, rank_base, plan.capacity, True,
                                             False, pos, ws, n_send, E)
        self._mark("dispatch")
        recv = torch.empty(max(n_recv, 1), d, dtype=torch.float16, device=dev)
        dist.all_to_all_single(recv[:n_recv], send[:n_send], plan.recv_rows, plan.send_rows,
                               group=self.group)
        self._mark("a2a_dispatch")
        if plan.reorder is not None and n_recv:
            idx = torch.from_numpy(plan.reorder).pin_memory().to(dev, non_blocking=True)
            a = recv[:n_recv].index_select(0, idx)
        else:
            idx, a = None, recv[:max(n_recv, 1)]
        y = self.layer.experts.forward_segments(a, seg_start, seg_len, plan.capacity,
                                                first_expert=self.rank * self.El,
                                                num_local=self.El, mark=self._mark)
        if idx is not None:
            y_send = torch.empty_like(y)
            y_send.index_copy_(0, idx, y)
        else:
            y_send = y
        back = torch.empty(max(n_send, 1), d, dtype=torch.float16, device=dev)
        dist.all_to_all_single(back[:n_send], y_send[:n_recv], plan.send_rows, plan.recv_rows,
                               group=self.group)
        self._mark("a2a_combine")
        out = combine(back, gw, pos, T_l, self.k)
        self._mark("combine")
        self._last_recv = n_recv
        return out, torch.tensor(plan.aux_loss, dtype=torch.float32, device=dev)
