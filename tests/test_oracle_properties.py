"""Property checks of the CPU oracle (the checker the GPU parity tests rely on),
on random sizes and values:

* top-k: k distinct experts per token that are a valid top-k of the fp32
  softmax probabilities (computed here independently, as the reference's
  ``torch.topk`` on probabilities selects them), in descending probability
  order; where probabilities are equal the documented contract decides --
  the larger fp32 logit first, then the lowest expert index; weights
  p / (sum of selected p + 1e-9);
* dispatch: uncapped CSR offsets = exclusive scan of the expert histogram, the
  kept slots of an expert are its first ``capacity`` slots in slot order and sit
  at ``offsets[e] + rank``, dropped slots have no row (slot_pos -1);
* combine over an identity expert returns sum_j w_j * x[t].
"""

from __future__ import annotations

import numpy as np
from hypothesis import given, settings, strategies as st

import oracle as orc


@st.composite
def routing_case(draw):
    T = draw(st.integers(1, 300))
    E = draw(st.integers(1, 64))
    k = draw(st.integers(1, min(8, E)))
    cf = draw(st.sampled_from([0.25, 0.5, 1.0, 1.25, 2.0]))
    seed = draw(st.integers(0, 2**31 - 1))
    ties = draw(st.booleans())
    rng = np.random.default_rng(seed)
    logits = rng.standard_normal((T, E)).astype(np.float32)
    if ties:  # coarse values: many exact ties
        logits = np.round(logits * 2).astype(np.float32) / 2
    return T, E, k, cf, logits


@settings(max_examples=60, deadline=None)
@given(routing_case())
def test_topk_order_ties_and_weights(case):
    T, E, k, cf, logits = case
    ids, w, probs = orc.topk_gating(logits, k)
    assert ids.shape == (T, k) and w.shape == (T, k)
    # fp32 probabilities computed independently of the oracle (float64 softmax, rounded)
    z = logits.astype(np.float64)
    pr = np.exp(z - z.max(axis=1, keepdims=True))
    pr = (pr / pr.sum(axis=1, keepdims=True)).astype(np.float32)
    for t in range(T):
        row, prow = logits[t], pr[t]
        sel = ids[t].tolist()
        assert len(set(sel)) == k
        rest = [e for e in range(E) if e not in sel]
        # a valid top-k of the probabilities (what the reference's torch.topk returns)...
        if rest:
            assert min(prow[sel]) >= max(prow[rest]) - 2e-7 * max(prow[rest])
        # ...in descending order, equal probabilities ordered by the contract
        for a, b in zip(sel, sel[1:]):
            assert prow[a] >= prow[b] - 2e-7 * prow[b]
            if row[a] == row[b]:
                assert a < b
    p = probs[np.arange(T)[:, None], ids]
    np.testing.assert_allclose(w, p / (p.sum(axis=1, keepdims=True) + np.float32(1e-9)),
                               rtol=1e-6, atol=1e-7)


@settings(max_examples=60, deadline=None)
@given(routing_case())
def test_dispatch_capacity_in_slot_order(case):
    T, E, k, cf, logits = case
    ids, w, _ = orc.topk_gating(logits, k)
    S = T * k
    C = orc.capacity(S, E, cf)
    tok = np.repeat(np.arange(T, dtype=np.int32), k)
    r = orc.dispatch(ids.reshape(-1), w.reshape(-1), tok, E, C)
    flat = ids.reshape(-1)
    counts = np.bincount(flat, minlength=E)
    assert r.offsets.tolist() == [0] + np.cumsum(counts).tolist()
    assert r.kept_counts.tolist() == np.minimum(counts, C).tolist()
    seen = np.zeros(E, np.int64)
    rows = set()
    for s in range(S):
        e = int(flat[s])
        if seen[e] < C:
            assert r.slot_pos[s] == r.offsets[e] + seen[e]
            rows.add(int(r.slot_pos[s]))
            assert r.src_idx[r.slot_pos[s]] == s // k
            assert r.routing_w[r.slot_pos[s]] == w.reshape(-1)[s]
        else:
            assert r.slot_pos[s] == -1
        seen[e] += 1
    assert len(rows) == int(np.minimum(counts, C).sum())


@settings(max_examples=30, deadline=None)
@given(routing_case(), st.integers(1, 64))
def test_identity_expert_combine(case, d):
    T, E, k, cf, logits = case
    ids, w, _ = orc.topk_gating(logits, k)
    C = orc.capacity(T * k, E, cf)
    tok = np.repeat(np.arange(T, dtype=np.int32), k)
    r = orc.dispatch(ids.reshape(-1), w.reshape(-1), tok, E, C)
    x = np.random.default_rng(T * 131 + d).standard_normal((T, d)).astype(np.float32)
    y = orc.permute_rows(x, r)            # identity experts: y = permuted rows
    out = orc.combine_slots(y, r, T)
    kept = (r.slot_pos >= 0).reshape(T, k)
    want = (np.where(kept, w, 0).sum(axis=1, dtype=np.float64))[:, None] * x
    np.testing.assert_allclose(out, want, rtol=1e-5, atol=1e-5)


def test_topk_logits_one_ulp_apart():
    """Logits one fp32 ulp apart can round to the same probability, where the
    reference's topk on probabilities leaves the order open; the contract takes
    the larger logit first (and the lowest index only for equal logits)."""
    x = np.float32(0.75)
    up = np.nextafter(x, np.float32(np.inf))
    logits = np.array([[x, up, np.float32(-3), x]], np.float32)
    ids, _, probs = orc.topk_gating(logits, 3)
    assert ids[0].tolist() == [1, 0, 3]
