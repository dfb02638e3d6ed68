"""numpy restatement of the LightningRouter MoE-layer hot path (CPU oracle).

TEST INFRASTRUCTURE ONLY -- imported by tests/, by __graft_entry__.smoke() as
the checker, and by bench.py's CPU-baseline / reference arm.  Never imported by
the product package.

Every function cites the reference (AlexanderLeonida/LLM-Serving-Kernel-
Optimization) file:line it restates.  Where the reference leaves a behaviour
undefined the contract chosen here is stated in the docstring:

* top-k is selected on fp32 logits, descending, ties to the lowest expert index
  (the reference's ``torch.topk`` on softmax probabilities does not fix the tie
  order);
* capacity keeps the first ``C`` slots of each expert in slot order (the intent
  of the reference's atomic-claim scatter, and what its Triton kernel does when
  run serially under ``TRITON_INTERPRET=1``);
* dropped slots are written as zero rows with ``routing_w = 0`` and
  ``source_idx = token`` (the reference leaves those rows uninitialised);
* the combine accumulates in fp32 (the reference uses fp16 atomics).
"""

from __future__ import annotations

import numpy as np

__all__ = [
    "capacity", "gate_logits", "softmax_f32", "topk_gating", "aux_loss",
    "dispatch", "permute_rows", "combine_slots", "gather_rows",
    "quantize_tensor", "pack_int4", "unpack_int4", "dequantize_tensor",
    "silu", "expert_ffn", "moe_layer", "RouteResult",
]


# --------------------------------------------------------------------------
# capacity / gating
# --------------------------------------------------------------------------

def capacity(num_slots: int, num_experts: int, capacity_factor: float) -> int:
    """Per-expert capacity, ``lightning_router/kernels/expert_routing.py:196-197``.

    ``max(int((S / E) * cf), 1)`` evaluated in Python double precision.
    """
    return max(int((num_slots / num_experts) * capacity_factor), 1)


def gate_logits(h: np.ndarray, wg: np.ndarray, bias: np.ndarray | None = None) -> np.ndarray:
    """fp32 gate logits ``h @ wg.T (+ bias)``.

    ``lightning_router/models/gating.py:46,69`` (``nn.Linear(d, E, bias=False)``),
    computed in fp32 from the fp16 operands.  ``bias`` is the per-expert logit
    bias of the skewed-routing workload (the reference gate has none).
    """
    out = h.astype(np.float32) @ wg.astype(np.float32).T
    if bias is not None:
        out = out + bias.astype(np.float32)[None, :]
    return out.astype(np.float32)


def softmax_f32(logits: np.ndarray) -> np.ndarray:
    """Row softmax in fp32, ``lightning_router/models/gating.py:70``."""
    logits = logits.astype(np.float32)
    m = logits.max(axis=1, keepdims=True)
    e = np.exp(logits - m).astype(np.float32)
    s = np.zeros((logits.shape[0], 1), np.float32)
    for j in range(logits.shape[1]):          # sequential sum, expert order
        s = (s + e[:, j:j + 1]).astype(np.float32)
    return (e / s).astype(np.float32)


def topk_gating(logits: np.ndarray, k: int):
    """Top-k selection and renormalisation, ``lightning_router/models/gating.py:70-85``.

    Returns ``(ids (T,k) int32, weights (T,k) fp32, probs (T,E) fp32)``.
    Selection is on the fp32 logits, descending, lowest index first on ties
    (softmax is monotone, so this is the reference's selection on
    probabilities with a fixed tie order).  ``w = p / (sum_topk p + 1e-9)``
    with the sum taken in selection order (``gating.py:75``).
    """
    probs = softmax_f32(logits)
    ids = np.argsort(-logits.astype(np.float32), axis=1, kind="stable")[:, :k].astype(np.int32)
    p_sel = np.take_along_axis(probs, ids.astype(np.int64), axis=1).astype(np.float32)
    s = np.zeros((logits.shape[0], 1), np.float32)
    for j in range(k):
        s = (s + p_sel[:, j:j + 1]).astype(np.float32)
    denom = (s + np.float32(1e-9)).astype(np.float32)
    w = (p_sel / denom).astype(np.float32)
    return ids, w, probs


def aux_loss(ids_flat: np.ndarray, probs: np.ndarray, num_experts: int, k: int,
             load_balance_weight: float = 0.01) -> float:
    """Switch-style load-balancing loss, ``lightning_router/models/gating.py:91-99``.

    ``lbw * E * sum_e f_e * P_e`` with the UNCAPPED slot fraction ``f`` and the
    mean softmax probability ``P``.  Evaluated in float64.
    """
    T = probs.shape[0]
    counts = np.bincount(ids_flat.astype(np.int64), minlength=num_experts).astype(np.float64)
    f = counts / float(T * k)
    P = probs.astype(np.float64).mean(axis=0)
    return float(load_balance_weight * num_experts * float((f * P).sum()))


# --------------------------------------------------------------------------
# dispatch / combine
# --------------------------------------------------------------------------

class RouteResult:
    """Routing metadata for S slots (slot s = t*k + j for gated routing)."""

    def __init__(self, ids, weights, token_idx, counts, offsets, kept_counts,
                 rank, kept, dst, src_idx, routing_w, slot_pos, capacity):
        self.ids = ids                    # (S,) int32 expert per slot
        self.weights = weights            # (S,) fp32 gate weight per slot
        self.token_idx = token_idx        # (S,) int32 source token per slot
        self.counts = counts              # (E,) int32 uncapped per-expert count
        self.offsets = offsets            # (E+1,) int32 uncapped CSR offsets
        self.kept_counts = kept_counts    # (E,) int32 min(count, C)
        self.rank = rank                  # (S,) int64 slot-order rank inside its expert
        self.kept = kept                  # (S,) bool rank < C
        self.dst = dst                    # (S,) int64 row of the slot in the permuted layout
        self.src_idx = src_idx            # (S,) int32 per row: source token
        self.routing_w = routing_w        # (S,) fp32 per row: gate weight (0 if dropped)
        self.slot_pos = slot_pos          # (S,) int32 per slot: row, or -1 if dropped
        self.capacity = capacity


def dispatch(expert_ids: np.ndarray, gate_weights: np.ndarray, token_indices: np.ndarray,
             num_experts: int, cap: int) -> RouteResult:
    """Histogram, exclusive scan and capacity-masked placement.

    ``lightning_router/kernels/expert_routing.py:39-84`` (histogram, scan into
    the uncapped CSR ``offsets``), ``:196-204`` (capacity, ``offsets[-1]`` rows)
    and ``:135-156`` (placement at ``offsets[e] + position``, kept iff
    ``position < capacity``), with positions assigned in slot order.
    """
    ids = expert_ids.astype(np.int64).reshape(-1)
    S = ids.shape[0]
    counts = np.bincount(ids, minlength=num_experts).astype(np.int64)
    offsets = np.zeros(num_experts + 1, np.int64)
    offsets[1:] = np.cumsum(counts)
    order = np.argsort(ids, kind="stable")
    rank = np.empty(S, np.int64)
    rank[order] = np.arange(S, dtype=np.int64) - offsets[ids[order]]
    kept = rank < cap
    dst = offsets[ids] + rank
    src_idx = np.empty(S, np.int32)
    routing_w = np.empty(S, np.float32)
    src_idx[dst] = token_indices.astype(np.int32).reshape(-1)
    routing_w[dst] = np.where(kept, gate_weights.astype(np.float32).reshape(-1), np.float32(0))
    slot_pos = np.where(kept, dst, -1).astype(np.int32)
    return RouteResult(
        ids=ids.astype(np.int32), weights=gate_weights.astype(np.float32).reshape(-1),
        token_idx=token_indices.astype(np.int32).reshape(-1),
        counts=counts.astype(np.int32), offsets=offsets.astype(np.int32),
        kept_counts=np.minimum(counts, cap).astype(np.int32), rank=rank, kept=kept,
        dst=dst, src_idx=src_idx, routing_w=routing_w, slot_pos=slot_pos, capacity=cap)


def permute_rows(x: np.ndarray, r: RouteResult) -> np.ndarray:
    """Permuted token matrix, ``lightning_router/kernels/expert_routing.py:150-156``.

    Row ``dst[s]`` holds ``x[token_idx[s]]`` for kept slots and zeros for dropped
    slots.
    """
    S = r.ids.shape[0]
    out = np.zeros((S, x.shape[1]), x.dtype)
    keep = r.kept
    out[r.dst[keep]] = x[r.token_idx[keep].astype(np.int64)]
    return out


def combine_slots(y: np.ndarray, r: RouteResult, num_tokens: int) -> np.ndarray:
    """Weighted combine in token order, fp32.

    ``lightning_router/models/moe_layer.py:80-84`` semantics (``index_add_`` of
    ``y * w``) restricted to kept slots, accumulated in fp32.
    """
    out = np.zeros((num_tokens, y.shape[1]), np.float32)
    keep = np.nonzero(r.kept)[0]
    contrib = y[r.dst[keep]].astype(np.float32) * r.weights[keep][:, None]
    np.add.at(out, r.token_idx[keep].astype(np.int64), contrib)
    return out


def gather_rows(y: np.ndarray, routing_w: np.ndarray, src_idx: np.ndarray,
                num_tokens: int) -> np.ndarray:
    """Row-wise weighted gather, ``lightning_router/kernels/expert_routing.py:238-298``.

    ``out[src[r]] += w[r] * y[r]`` over rows with ``w[r] != 0`` (a dropped row
    carries ``w = 0`` and contributes nothing), accumulated in fp32.
    """
    out = np.zeros((num_tokens, y.shape[1]), np.float32)
    live = np.nonzero(routing_w != 0)[0]
    np.add.at(out, src_idx[live].astype(np.int64),
              y[live].astype(np.float32) * routing_w[live].astype(np.float32)[:, None])
    return out


# --------------------------------------------------------------------------
# INT4 format
# --------------------------------------------------------------------------

def pack_int4(q: np.ndarray) -> np.ndarray:
    """``lightning_router/quantization/pack_weights.py:81-89``: nibble i of word j is column 8j+i."""
    *lead, N = q.shape
    assert N % 8 == 0
    qv = q.reshape(*lead, N // 8, 8).astype(np.uint32) & 0xF
    out = np.zeros((*lead, N // 8), np.uint32)
    for i in range(8):
        out |= qv[..., i] << np.uint32(4 * i)
    return out.view(np.int32)


def unpack_int4(packed: np.ndarray, N: int) -> np.ndarray:
    """``lightning_router/quantization/pack_weights.py:92-105``."""
    *lead, pn = packed.shape
    assert pn == N // 8
    pu = packed.view(np.uint32)
    out = np.empty((*lead, N), np.int32)
    for i in range(8):
        out[..., i::8] = ((pu >> np.uint32(4 * i)) & 0xF).astype(np.int32)
    return out


def quantize_tensor(weight: np.ndarray, group_size: int = 128, scheme: str = "asymmetric"):
    """``lightning_router/quantization/pack_weights.py:23-78``, fp32 arithmetic.

    Returns ``(qweight (K,N/8) int32, scales (K/g,N) fp16, zeros (K/g,N/8) int32)``.
    """
    K, N = weight.shape
    assert K % group_size == 0, f"K={K} must be divisible by group_size={group_size}"
    assert N % 8 == 0, f"N={N} must be divisible by 8 for INT4 packing"
    w = weight.astype(np.float32).reshape(K // group_size, group_size, N)
    if scheme == "asymmetric":
        wmin = w.min(axis=1)
        wmax = w.max(axis=1)
        scales = ((wmax - wmin) / np.float32(15.0)).astype(np.float32)
        scales = np.maximum(scales, np.float32(1e-8))
        zeros = np.clip(np.round((-wmin / scales).astype(np.float32)), 0, 15).astype(np.float32)
    else:
        absmax = np.abs(w).max(axis=1)
        scales = np.maximum((absmax / np.float32(7.0)).astype(np.float32), np.float32(1e-8))
        zeros = np.full_like(scales, 8.0)
    q = np.round((w / scales[:, None, :]).astype(np.float32) + zeros[:, None, :]).astype(np.float32)
    q = np.clip(q, 0, 15).astype(np.int32).reshape(K, N)
    return pack_int4(q), scales.astype(np.float16), pack_int4(zeros.astype(np.int32))


def dequantize_tensor(qweight: np.ndarray, scales: np.ndarray, zeros: np.ndarray,
                      group_size: int, N: int) -> np.ndarray:
    """``lightning_router/quantization/pack_weights.py:108-130``: fp16(fp32(scale) * (q - z))."""
    K = qweight.shape[0]
    G = scales.shape[0]
    q = unpack_int4(qweight, N).astype(np.float32).reshape(G, group_size, N)
    z = unpack_int4(zeros, N).astype(np.float32)
    w = scales.astype(np.float32)[:, None, :] * (q - z[:, None, :])
    return w.reshape(K, N).astype(np.float16)


# --------------------------------------------------------------------------
# expert FFN / layer
# --------------------------------------------------------------------------

def silu(v: np.ndarray) -> np.ndarray:
    v = v.astype(np.float32)
    return (v / (np.float32(1.0) + np.exp(-v))).astype(np.float32)


def expert_ffn(x: np.ndarray, w_up: np.ndarray, w_down: np.ndarray,
               w_gate: np.ndarray | None = None) -> np.ndarray:
    """Expert FFN in fp32 on dequantized weights.

    Gated (SwiGLU): ``down(silu(gate x) * up x)``, ``lightning_router/models/experts.py:84-89``.
    Non-gated (``w_gate is None``): ``down(silu(up x))``.
    Weights are (K=in, N=out) as stored by ``ExpertFFN`` (``experts.py:50-56``).
    """
    x32 = x.astype(np.float32)
    up = x32 @ w_up.astype(np.float32)
    if w_gate is not None:
        hid = silu(x32 @ w_gate.astype(np.float32)) * up
    else:
        hid = silu(up)
    return (hid.astype(np.float32) @ w_down.astype(np.float32)).astype(np.float32)


def moe_layer(x: np.ndarray, logits: np.ndarray, k: int, capacity_factor: float,
              experts, load_balance_weight: float = 0.01, cap: int | None = None):
    """MoE layer, ``lightning_router/models/moe_layer.py:90-135``, fp32.

    ``experts[e]`` is a dict with dequantized ``up``, ``down`` and optional
    ``gate`` (K,N) arrays.  Routing follows :func:`topk_gating` /
    :func:`dispatch`; only kept slots reach the experts.  Returns
    ``(out (T,d) fp32, aux_loss, RouteResult)``.
    """
    T = x.shape[0]
    E = logits.shape[1]
    ids, w, probs = topk_gating(logits, k)
    S = T * k
    C = capacity(S, E, capacity_factor) if cap is None else cap
    tok = np.repeat(np.arange(T, dtype=np.int32), k)
    r = dispatch(ids.reshape(-1), w.reshape(-1), tok, E, C)
    y = np.zeros((S, x.shape[1]), np.float32)
    for e in range(E):
        start = int(r.offsets[e])
        n = int(r.kept_counts[e])
        if n == 0:
            continue
        rows = slice(start, start + n)
        toks = r.src_idx[rows].astype(np.int64)
        ex = experts[e]
        y[rows] = expert_ffn(x[toks], ex["up"], ex["down"], ex.get("gate"))
    out = combine_slots(y, r, T)
    aux = aux_loss(ids.reshape(-1), probs, E, k, load_balance_weight)
    return out, aux, r
