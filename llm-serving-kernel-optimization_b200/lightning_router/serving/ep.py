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
  token order by the same combine kernel as on one GPU;
* each rank's tokens are split into ``microbatches`` contiguous micro-batches
  whose exchanges are issued asynchronously, so one micro-batch's all-to-all
  overlaps another's expert GEMMs (capacity still follows the global slot order
  over all ranks and micro-batches).

Every kept row goes through the same per-row arithmetic as on one GPU, so the
output equals the single-GPU output bit for bit.

Two exchanges implement the moves:

* ``exchange="peer"`` (default with one process per GPU on one node): every rank
  keeps its tokens, the row -> token map of its expert segments, its expert
  outputs, a statistics table and a few flags in buffers the other ranks map
  through CUDA IPC.  A step calls no collective library: each rank writes its
  statistics row into every rank's table and raises a flag there
  (``lr_ep_publish``); the plan kernel waits for every rank's flag and decides
  the capacity and the row layouts on the device (``lr_ep_plan_wait``); the
  expert owner pulls its kept rows over NVLink (``lr_ep_gather``), runs its
  GEMMs and raises an "outputs" flag on every rank (``lr_ep_signal``); the token
  owner waits for those flags and pulls the output rows back while it combines
  them (``lr_ep_combine``).  Flags carry the step number; every wait is bounded
  in time and reports through the device error word.  No host synchronisation.
  The buffers are sized once for a per-rank shard limit, so shard sizes may
  differ between ranks and change from step to step (each rank up to the
  limit).
* ``exchange="nccl"``: kept rows are permuted into a compact send buffer grouped
  by owner rank, exchanged with ``all_to_all_single`` and sent back the same
  way.  The split sizes need one device->host read of the gathered counts per
  forward (:func:`plan_exchange`, the pure host part, exercised by CPU ``gloo``
  tests against the oracle).
"""

from __future__ import annotations

import ctypes
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


def plan_exchanges(stats: np.ndarray, rank: int, world: int, num_experts: int, top_k: int,
                   capacity_factor: float, load_balance_weight: float,
                   nchunks: int = 1) -> list:
    """Host plans for this rank's ``nchunks`` exchanges from the all-gathered ``stats``.

    ``stats`` has ``world * nchunks`` float64 rows ``[T, count[0..E), prob_sum[0..E)]``,
    one per token shard, in global token order: rank-major, then micro-batch
    (each rank's tokens may be split into ``nchunks`` contiguous micro-batches).
    Plan ``c`` covers the exchange of micro-batch ``c``: every rank sends its
    micro-batch-``c`` rows and receives the same micro-batch's rows of its
    experts.  Capacity follows the global slot order over all shards.
    """
    G, E = world, num_experts
    if E % G:
        raise ValueError(f"num_experts {E} must be divisible by the world size {G}")
    El = E // G
    counts = np.rint(stats[:, 1:1 + E]).astype(np.int64)
    T = int(stats[:, 0].sum())
    S = T * top_k
    C = expert_capacity(S, E, capacity_factor)
    base = np.cumsum(counts, axis=0) - counts         # exclusive, over shards in order
    kept_all = np.clip(C - base, 0, counts)           # (G*nchunks, E)
    f = counts.sum(axis=0) / float(max(S, 1))
    P = stats[:, 1 + E:1 + 2 * E].sum(axis=0) / float(max(T, 1))
    aux = float(load_balance_weight * E * float((f * P).sum()))
    # per destination rank / per local expert sums, shaped (G*nchunks, G, El)
    per_dst = kept_all.reshape(G * nchunks, G, El)
    send_tot = per_dst.sum(axis=2)                    # (G*nchunks, G) rows to each rank
    mine = per_dst[:, rank, :]                        # (G*nchunks, El) rows for my experts
    plans = []
    for c in range(nchunks):
        me = rank * nchunks + c
        kept = kept_all[c::nchunks]                   # (G, E)
        koff = np.zeros(E + 1, np.int32)
        koff[1:] = np.cumsum(kept_all[me])
        recv_m = mine[c::nchunks]                     # (G, El) from each source rank
        recv_rows = recv_m.sum(axis=1).tolist()
        tot = recv_m.sum(axis=0)
        seg_start = np.zeros(El, np.int32)
        seg_start[1:] = np.cumsum(tot)[:-1]
        reorder = None
        if El > 1:
            # receive layout [source rank][local expert] -> GEMM layout [local expert][rank]
            flat = recv_m.reshape(-1)
            starts = (np.cumsum(flat) - flat).reshape(G, El).T.reshape(-1)
            lens = recv_m.T.reshape(-1)
            dst0 = np.cumsum(lens) - lens
            reorder = (np.repeat(starts - dst0, lens) + np.arange(int(lens.sum()))).astype(np.int64)
        plans.append(ExchangePlan(T, C, base[me].astype(np.int32), kept, koff,
                                  send_tot[me].tolist(), recv_rows, reorder, seg_start,
                                  tot.astype(np.int32), aux))
    return plans


def microbatch_bounds(num_tokens: int, nchunks: int) -> list:
    """Token bounds of a shard's ``nchunks`` contiguous micro-batches.

    ``nchunks`` is the same on every rank whatever its shard size (the gathered
    statistics hold ``world * nchunks`` rows), so a small shard may have empty
    micro-batches."""
    return [num_tokens * c // nchunks for c in range(nchunks + 1)]


def plan_exchange(stats: np.ndarray, rank: int, world: int, num_experts: int, top_k: int,
                  capacity_factor: float, load_balance_weight: float, chunk: int = 0,
                  nchunks: int = 1) -> ExchangePlan:
    """The plan of one micro-batch; see :func:`plan_exchanges`."""
    return plan_exchanges(stats, rank, world, num_experts, top_k, capacity_factor,
                          load_balance_weight, nchunks)[chunk]


class _PeerBuffers:
    """Per-rank exchange buffers mapped by every rank of the group (CUDA IPC).

    ``x`` (T_max, d) tokens and ``src`` (T_max*k) row -> token map are read by the
    expert owners; ``y`` (rows_max, d) expert outputs are read by the token owners;
    ``stats`` (G, 1 + 2E) float64 and ``flags`` (2G,) int32 are written by every
    rank; ``a`` (rows_max, d) is this rank's GEMM input (local).  ``p*`` hold the
    G ranks' addresses of each mapped buffer (int64, on the device).
    """

    def __init__(self, group, world: int, rank: int, dev, T_max: int, k: int, d: int,
                 rows_max: int, num_experts: int):
        self.T_max, self.rows_max = T_max, rows_max
        # one allocation holds every mapped buffer, so each rank exports (and every
        # peer opens) exactly one IPC handle
        parts = [("x", torch.float16, (T_max, d)), ("src", torch.int32, (T_max * k,)),
                 ("y", torch.float16, (max(rows_max, 1), d)),
                 ("stats", torch.float64, (world, 1 + 2 * num_experts)),
                 ("flags", torch.int32, (2 * world,))]
        offs, total = [], 0
        for _name, dt, shape in parts:
            n = int(np.prod(shape)) * torch.empty(0, dtype=dt).element_size()
            offs.append(total)
            total += (n + 255) // 256 * 256
        self._mem = torch.empty(total, dtype=torch.uint8, device=dev)
        views = []
        for (_name, dt, shape), off in zip(parts, offs):
            n = int(np.prod(shape)) * torch.empty(0, dtype=dt).element_size()
            views.append(self._mem.narrow(0, off, n).view(dt).view(shape))
        self.x, self.src, self.y, self.stats, self.flags = views
        self.src.zero_()
        self.stats.zero_()
        self.flags.zero_()
        self.a = torch.empty(max(rows_max, 1), d, dtype=torch.float16, device=dev)
        # zeroed before any peer can map (and write) them
        torch.cuda.synchronize(dev)
        lib = _ext.clib()
        h = ctypes.create_string_buffer(64)
        base_off = ctypes.c_uint64(0)
        _check(lib.lr_ipc_export(ctypes.c_void_p(self._mem.data_ptr()), h, ctypes.byref(base_off)),
               "lr_ipc_export")
        allh = [None] * world
        dist.all_gather_object(allh, (h.raw, int(base_off.value)), group=group)
        self._bases = []
        ptrs = [[0] * world for _ in parts]
        for r in range(world):
            if r == rank:
                base = self._mem.data_ptr()
            else:
                hb, off = allh[r]
                p, mb = ctypes.c_void_p(), ctypes.c_void_p()
                _check(lib.lr_ipc_import(ctypes.create_string_buffer(hb, 64), ctypes.c_uint64(off),
                                         ctypes.byref(p), ctypes.byref(mb)), "lr_ipc_import")
                self._bases.append(mb.value)
                base = p.value
            for b, off in enumerate(offs):
                ptrs[b][r] = base + off
        self.px, self.psrc, self.py, self.pstats, self.pflags = (
            torch.tensor(p, dtype=torch.int64, device=dev) for p in ptrs)

    def close(self) -> None:
        lib = _ext.clib()
        for b in self._bases:
            lib.lr_ipc_close(ctypes.c_void_p(b))
        self._bases = []


def _check(status: int, what: str) -> None:
    if status != 0:
        msg = _ext.clib().lr_status_string(status)
        raise RuntimeError(f"{what} failed: {msg.decode() if isinstance(msg, bytes) else msg}")


class ExpertParallelMoE:
    """Expert-parallel forward of a ``MoELayer`` (one rank per GPU).

    ``layer`` must hold at least this rank's experts; the other experts'
    buffers are not read.  ``forward(x_local)`` takes this rank's token shard
    (T_r, d) fp16 and returns ``(out_local, aux_loss)`` for the whole job's
    routing (aux is the global load-balancing loss).  ``exchange`` selects the
    token exchange ("peer" or "nccl", see the module notes); ``microbatches``
    applies to the NCCL exchange.

    Shard sizes may differ between ranks and from one forward to the next.
    The peer exchange sizes its mapped buffers once, for ``max_tokens_per_rank``
    tokens per rank (when None: the largest shard of the first forward, agreed
    by a collective that every rank enters in its first forward).  A shard above
    that limit raises ``ValueError`` on its rank before any collective of the
    step; the other ranks then fail at the process group's timeout, as after any
    rank's error.  Every rank issues the same collectives in the same order in
    every forward, whatever the sizes (an empty shard included).
    """

    def __init__(self, layer, world: int, rank: int, group=None, microbatches: int = 1,
                 exchange: str = "peer", max_tokens_per_rank: int | None = None):
        if layer.num_experts % world:
            raise ValueError("num_experts must be divisible by the world size")
        if exchange not in ("peer", "nccl"):
            raise ValueError(f"exchange must be 'peer' or 'nccl', got {exchange!r}")
        self.exchange = exchange
        self.layer = layer
        self.world = world
        self.rank = rank
        self.group = group
        self.E = layer.num_experts
        self.El = self.E // world
        self.k = layer.top_k
        self.cf = layer.moe_cfg.expert_capacity_factor
        self.lbw = layer.gate.load_balance_weight
        self.microbatches = max(1, int(microbatches))
        self.stage_events: list | None = None
        self._last_recv = 0
        self._last_kept_e: list = []
        self._pinned: torch.Tensor | None = None  # reused host staging for per-step metadata
        self.max_tokens_per_rank = max_tokens_per_rank
        self._epoch = 0  # steps of the peer exchange (the same on every rank)
        self._peer: _PeerBuffers | None = None
        self._plan: torch.Tensor | None = None

    def _to_device(self, arr: np.ndarray, dev, dtype) -> torch.Tensor:
        """Copy a small host array to the device through a persistent pinned buffer."""
        t = torch.from_numpy(np.ascontiguousarray(arr)).to(dtype)
        nbytes = t.numel() * t.element_size()
        if self._pinned is None or self._pinned.numel() < nbytes:
            self._pinned = torch.empty(max(nbytes, 1 << 16), dtype=torch.uint8).pin_memory()
        # the previous step's copy out of the staging buffer must be finished
        if getattr(self, "_staging_event", None) is not None:
            self._staging_event.synchronize()
        stage = self._pinned[:nbytes].view(dtype)
        stage.copy_(t.view(-1))
        out = stage.to(dev, non_blocking=True)
        self._staging_event = torch.cuda.Event()
        self._staging_event.record()
        return out

    @classmethod
    def from_layer(cls, layer, world: int, rank: int, group=None, microbatches: int = 1,
                   exchange: str = "peer",
                   max_tokens_per_rank: int | None = None) -> "ExpertParallelMoE":
        return cls(layer, world, rank, group, microbatches, exchange, max_tokens_per_rank)

    def close(self) -> None:
        """Unmap the peers' exchange buffers (every rank calls it, before destroying
        the group): a barrier first, so that no rank frees buffers a peer still reads."""
        if self._peer is not None:
            torch.cuda.synchronize()
            dist.barrier(group=self.group)
            self._peer.close()
            self._peer = None

    def _mark(self, name):
        if self.stage_events is not None:
            ev = torch.cuda.Event(enable_timing=True)
            ev.record()
            self.stage_events.append((name, ev))

    def last_kept_rows(self) -> int:
        return int(sum(self.last_kept_per_expert()))

    def last_kept_per_expert(self) -> list:
        """Kept rows of each local expert in the last forward."""
        if self.exchange == "peer" and self._plan is not None:
            return self._plan[self.El:2 * self.El].cpu().tolist()
        return list(self._last_kept_e)

    def _peer_buffers(self, T_l: int, d: int, dev) -> _PeerBuffers:
        """The mapped exchange buffers, created in the first forward (a collective
        every rank enters then) for the per-rank shard limit."""
        if self._peer is None:
            T_max = self.max_tokens_per_rank
            if T_max is None:
                sizes = [None] * self.world
                dist.all_gather_object(sizes, int(T_l), group=self.group)
                T_max = max(sizes)
            T_max = max(int(T_max), 1)
            C_max = expert_capacity(T_max * self.world * self.k, self.E, self.cf)
            self._peer = _PeerBuffers(self.group, self.world, self.rank, dev, T_max, self.k, d,
                                      self.El * C_max, self.E)
            self._peer_C = C_max
        if T_l > self._peer.T_max:
            raise ValueError(f"shard of {T_l} tokens exceeds the expert-parallel limit of "
                             f"{self._peer.T_max} tokens per rank (max_tokens_per_rank)")
        return self._peer

    @torch.no_grad()
    def forward(self, x: torch.Tensor):
        if self.exchange == "peer" and self.world > 1:
            xf = x.reshape(-1, x.shape[-1])
            return self._forward_peer(xf, self._peer_buffers(xf.shape[0], xf.shape[1], xf.device))
        return self._forward_nccl(x)

    def _forward_peer(self, x: torch.Tensor, bufs: _PeerBuffers):
        ops = _ext.ops()
        dev = x.device
        x = x.to(torch.float16).contiguous()
        T_l, d = x.shape
        E, El, k = self.E, self.El, self.k
        C_max = self._peer_C
        err = _ext.error_word(dev.index)
        self._epoch += 1
        epoch = self._epoch
        self._mark("begin")
        offs = psum = None
        if T_l:
            logits = self.layer.gate.logits(x)
            self._mark("gate")
            ids, gw, _tok, offs, _kept, _aux, psum, pos, ws = ops.topk_route(
                logits, k, 1, float(self.lbw), err)
            # this rank's tokens and its uncapped row -> token map, readable by the owners
            bufs.x[:T_l].copy_(x)
            ops.route_rows(ids, gw, offs, pos, ws, T_l, E, bufs.src)
        else:  # an empty shard still publishes (zeros) and owns its experts
            self._mark("gate")
        # statistics to every rank, then the plan once every rank's row is in
        ops.ep_publish(bufs.pstats, bufs.pflags, offs, psum, T_l, E, self.rank, epoch)
        plan, aux = ops.ep_plan_wait(bufs.stats, bufs.flags, E, self.rank, k, float(self.cf),
                                     C_max, float(self.lbw), epoch, err)
        a = ops.ep_gather(bufs.px, bufs.psrc, plan, E, self.rank, bufs.T_max, bufs.T_max * k,
                          d, bufs.a, err)
        self._mark("dispatch")
        self.layer.experts.forward_segments(a, plan[0:El], plan[El:2 * El], C_max,
                                            first_expert=self.rank * El, num_local=El,
                                            mark=self._mark, out=bufs.y)
        # this rank's outputs are written: raise its flag on every rank
        ops.ep_signal(bufs.pflags, self.rank, epoch)
        self._mark("a2a_combine")
        if T_l:
            out = ops.ep_combine(bufs.py, plan, ids, gw, pos, T_l, E, bufs.rows_max, d, err,
                                 bufs.flags[self.world:], epoch)
        else:
            out = torch.empty(0, d, dtype=torch.float16, device=dev)
        self._mark("combine")
        self._plan = plan
        return out, aux

    @torch.no_grad()
    def _forward_nccl(self, x: torch.Tensor):
        ops = _ext.ops()
        dev = x.device
        x = x.reshape(-1, x.shape[-1]).to(torch.float16).contiguous()
        T_l, d = x.shape
        E, G, El = self.E, self.world, self.El
        # the same micro-batch count on every rank (the gathered statistics have
        # G * nc rows); a micro-batch of a small shard may be empty
        nc = self.microbatches
        bounds = microbatch_bounds(T_l, nc)
        err = _ext.error_word(dev.index)
        self._mark("begin")
        logits = self.layer.gate.logits(x) if T_l else None
        self._mark("gate")
        # phase 1 for every micro-batch, then one gather of all shard statistics
        routes, stats_l = [], []
        for c in range(nc):
            lo, hi = bounds[c], bounds[c + 1]
            if hi == lo:
                routes.append(None)
                stats_l.append(torch.zeros(1 + 2 * E, dtype=torch.float64, device=dev))
                continue
            r = ops.topk_route(logits[lo:hi], self.k, 1, float(self.lbw), err)
            ids, gw, _tok, offs, _kept, _aux, psum, pos, ws = r
            routes.append((ids, gw, pos, ws))
            stats_l.append(torch.cat([torch.full((1,), float(hi - lo), dtype=torch.float64,
                                                 device=dev),
                                      (offs[1:] - offs[:-1]).double(), psum]))
        stats_l = torch.cat(stats_l)
        stats = torch.empty(G * stats_l.numel(), dtype=torch.float64, device=dev)
        dist.all_gather_into_tensor(stats, stats_l, group=self.group)
        stats_h = stats.view(G * nc, -1).cpu().numpy()  # the one host synchronisation
        plans = plan_exchanges(stats_h, self.rank, G, E, self.k, self.cf, self.lbw, nc)
        # phase 2 + dispatch exchange for every micro-batch (asynchronous collectives)
        sends, recvs, metas, dwork = [], [], [], []
        for c, plan in enumerate(plans):
            idx_h = plan.reorder if (plan.reorder is not None and plan.n_recv) else \
                np.zeros(0, np.int64)
            meta = self._to_device(np.concatenate([plan.rank_base, plan.koff, plan.seg_start,
                                                   plan.seg_len, idx_h]).astype(np.int32),
                                   dev, torch.int32)
            metas.append(meta)
            if routes[c] is not None:
                ids, gw, pos, ws = routes[c]
                xs = x[bounds[c]:bounds[c + 1]]
                send, _rw, _src = ops.permute_tokens(xs, ids, gw, meta[E:2 * E + 1], meta[:E],
                                                     plan.capacity, True, False, pos, ws,
                                                     plan.n_send, E)
            else:  # an empty micro-batch sends nothing
                send = torch.empty(1, d, dtype=torch.float16, device=dev)
            recv = torch.empty(max(plan.n_recv, 1), d, dtype=torch.float16, device=dev)
            sends.append(send)
            recvs.append(recv)
            dwork.append(dist.all_to_all_single(recv[:plan.n_recv], send[:plan.n_send],
                                                plan.recv_rows, plan.send_rows,
                                                group=self.group, async_op=True))
        self._mark("dispatch")
        # expert FFN per micro-batch as soon as its rows arrived; combine exchange async
        backs, cwork = [], []
        for c, plan in enumerate(plans):
            dwork[c].wait()
            if c == 0:
                self._mark("a2a_dispatch")
            meta = metas[c]
            seg_start = meta[2 * E + 1:2 * E + 1 + El]
            seg_len = meta[2 * E + 1 + El:2 * E + 1 + 2 * El]
            n_recv, n_send = plan.n_recv, plan.n_send
            if plan.reorder is not None and n_recv:
                idx = meta[2 * E + 1 + 2 * El:].long()
                a = recvs[c][:n_recv].index_select(0, idx)
            else:
                idx, a = None, recvs[c]
            y = self.layer.experts.forward_segments(
                a, seg_start, seg_len, plan.capacity, first_expert=self.rank * El,
                num_local=El, mark=self._mark if c == nc - 1 else None)
            if idx is not None:
                y_send = torch.empty_like(y)
                y_send.index_copy_(0, idx, y)
            else:
                y_send = y
            back = torch.empty(max(n_send, 1), d, dtype=torch.float16, device=dev)
            backs.append(back)
            cwork.append(dist.all_to_all_single(back[:n_send], y_send[:n_recv], plan.send_rows,
                                                plan.recv_rows, group=self.group,
                                                async_op=True))
        outs = []
        for c in range(nc):
            cwork[c].wait()
            if c == 0:
                self._mark("a2a_combine")
            if routes[c] is None:
                outs.append(torch.empty(0, d, dtype=torch.float16, device=dev))
                continue
            _ids, gw, pos, _ws = routes[c]
            outs.append(combine(backs[c], gw, pos, bounds[c + 1] - bounds[c], self.k))
        out = outs[0] if nc == 1 else torch.cat(outs)
        self._mark("combine")
        self._last_recv = sum(p.n_recv for p in plans)
        self._last_kept_e = [int(sum(int(p.seg_len[el]) for p in plans)) for el in range(El)]
        return out, torch.tensor(plans[0].aux_loss, dtype=torch.float32, device=dev)
