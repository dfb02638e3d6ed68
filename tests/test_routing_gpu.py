"""GPU parity of gating, dispatch, gather and combine against the CPU oracle.

Integer outputs (expert ids, counts, offsets, slot positions, source indices,
permuted rows) must match bit for bit; gate weights within 1e-6 relative (fp32
``exp`` differs by ulps between CPU and GPU); aux loss within 1e-5 relative.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

import oracle as orc
from conftest import golden

pytestmark = pytest.mark.gpu

DEV = "cuda"


def _np(t):
    return t.detach().cpu().numpy()


def check_plan(plan, x, logits, k, cf, fill=True):
    T, E = logits.shape
    lg = _np(logits)
    ids, w, probs = orc.topk_gating(lg, k)
    C = orc.capacity(T * k, E, cf)
    tok = np.repeat(np.arange(T, dtype=np.int32), k)
    r = orc.dispatch(ids.reshape(-1), w.reshape(-1), tok, E, C)
    assert plan.capacity == C
    np.testing.assert_array_equal(_np(plan.expert_ids), ids.reshape(-1))
    np.testing.assert_allclose(_np(plan.gate_weights), w.reshape(-1), rtol=1e-6, atol=1e-12)
    np.testing.assert_array_equal(_np(plan.token_indices), tok)
    np.testing.assert_array_equal(_np(plan.offsets), r.offsets)
    np.testing.assert_array_equal(_np(plan.kept_counts), r.kept_counts)
    np.testing.assert_array_equal(_np(plan.slot_pos), r.slot_pos)
    np.testing.assert_array_equal(_np(plan.source_indices), r.src_idx)
    rw = _np(plan.routing_weights)
    kept_rows = r.dst[r.kept]
    np.testing.assert_allclose(rw[kept_rows], r.routing_w[kept_rows], rtol=1e-6, atol=1e-12)
    assert (rw[r.dst[~r.kept]] == 0).all()
    aux = orc.aux_loss(ids.reshape(-1), probs, E, k, 0.01)
    assert abs(float(plan.aux_loss) - aux) <= 1e-5 * abs(aux) + 1e-12
    if x is not None and plan.permuted.numel():
        perm = _np(plan.permuted).view(np.uint16)
        ref = orc.permute_rows(_np(x), r).view(np.uint16)
        if fill:
            np.testing.assert_array_equal(perm, ref)
        else:
            np.testing.assert_array_equal(perm[kept_rows], ref[kept_rows])
    return r


CASES = [
    # T, d, E, k, cf
    (1000, 256, 8, 2, 1.0),
    (1000, 256, 8, 2, 2.0),
    (777, 64, 4, 2, 1.25),
    (513, 128, 64, 6, 1.5),
    (1, 64, 8, 2, 1.0),
    (300, 32, 16, 8, 0.5),
    (2048, 64, 32, 1, 1.0),
    (4099, 8, 8, 2, 1.0),
]


@pytest.mark.parametrize("T,d,E,k,cf", CASES)
def test_topk_gating_dispatch_matches_oracle(T, d, E, k, cf):
    from lightning_router.kernels.expert_routing import topk_gating_dispatch
    g = torch.Generator().manual_seed(T * 31 + E)
    x = torch.randn(T, d, generator=g).half()
    logits = torch.randn(T, E, generator=g)
    if E == 64:  # skewed: Zipf-like bias produces heavy drops
        logits = logits + torch.linspace(3, -3, E)
    plan = topk_gating_dispatch(x.to(DEV), logits.to(DEV), k, cf, fill_dropped=True)
    check_plan(plan, x, logits, k, cf)


def test_ties_break_to_lowest_expert():
    from lightning_router.kernels.expert_routing import topk_gating_dispatch
    T, E, k = 257, 8, 3
    g = torch.Generator().manual_seed(7)
    logits = torch.randint(-2, 3, (T, E), generator=g).float()  # many exact ties
    logits[0] = 0.0
    plan = topk_gating_dispatch(None, logits.to(DEV), k, 1.0)
    check_plan(plan, None, logits, k, 1.0)
    assert _np(plan.expert_ids)[:3].tolist() == [0, 1, 2]


def test_all_tokens_to_one_expert_drop_in_slot_order():
    from lightning_router.kernels.expert_routing import topk_gating_dispatch
    T, E, k, d = 600, 8, 2, 64
    logits = torch.zeros(T, E)
    logits[:, 3] = 10.0
    logits[:, 5] = 5.0
    x = torch.randn(T, d).half()
    plan = topk_gating_dispatch(x.to(DEV), logits.to(DEV), k, 1.0, fill_dropped=True)
    r = check_plan(plan, x, logits, k, 1.0)
    C = plan.capacity
    assert r.kept_counts[3] == C and r.kept_counts[5] == C
    pos = _np(plan.slot_pos).reshape(T, k)
    assert (pos[:C, 0] >= 0).all() and (pos[C:, 0] == -1).all()


def test_fill_dropped_false_leaves_kept_rows_exact():
    from lightning_router.kernels.expert_routing import topk_gating_dispatch
    T, E, k, d = 1500, 8, 2, 128
    g = torch.Generator().manual_seed(3)
    x = torch.randn(T, d, generator=g).half()
    logits = torch.randn(T, E, generator=g) + torch.linspace(1, -1, E)
    plan = topk_gating_dispatch(x.to(DEV), logits.to(DEV), k, 0.8, fill_dropped=False)
    check_plan(plan, x, logits, k, 0.8, fill=False)


# ---------------------------------------------------------------------------
# reference API: expert_routing_forward / expert_routing_gather
# ---------------------------------------------------------------------------

def _make_test_data(num_tokens=64, hidden=256, num_experts=4, top_k=2, seed=0):
    g = torch.Generator().manual_seed(seed)
    tokens = torch.randn(num_tokens, hidden, generator=g).half()
    ids = torch.randint(0, num_experts, (num_tokens * top_k,), generator=g, dtype=torch.int32)
    w = torch.rand(num_tokens * top_k, generator=g)
    w = w / w.view(num_tokens, top_k).sum(-1, keepdim=True).repeat(1, top_k).view(-1)
    tok = torch.arange(num_tokens).unsqueeze(1).expand(-1, top_k).reshape(-1).int()
    return tokens, ids, w, tok


@pytest.mark.parametrize("T,d,E,k,cf", [(64, 256, 4, 2, 1.25), (1000, 64, 8, 2, 1.0),
                                        (333, 128, 64, 6, 1.5), (4096, 32, 1000, 1, 1.0)])
def test_expert_routing_forward_matches_oracle(T, d, E, k, cf):
    from lightning_router.kernels.expert_routing import expert_routing_forward_ex
    tokens, ids, w, tok = _make_test_data(T, d, E, k, seed=T)
    perm, offs, rw, src, kept, pos = expert_routing_forward_ex(
        tokens.to(DEV), ids.to(DEV), w.to(DEV), tok.to(DEV), E, cf)
    C = orc.capacity(T * k, E, cf)
    r = orc.dispatch(_np(ids), _np(w), _np(tok), E, C)
    np.testing.assert_array_equal(_np(offs), r.offsets)
    np.testing.assert_array_equal(_np(kept), r.kept_counts)
    np.testing.assert_array_equal(_np(pos), r.slot_pos)
    np.testing.assert_array_equal(_np(src), r.src_idx)
    np.testing.assert_array_equal(_np(rw), r.routing_w)
    np.testing.assert_array_equal(_np(perm).view(np.uint16),
                                  orc.permute_rows(_np(tokens), r).view(np.uint16))


def test_reference_histogram_matches_bincount():
    """Mirrors the reference's tests/test_expert_routing.py:85-101."""
    from lightning_router.kernels.expert_routing import expert_routing_forward
    tokens, ids, w, tok = _make_test_data()
    _, offsets, _, _ = expert_routing_forward(tokens.to(DEV), ids.to(DEV), w.to(DEV), tok.to(DEV), 4)
    ref = torch.bincount(ids.long(), minlength=4)
    torch.testing.assert_close((offsets[1:] - offsets[:-1]).cpu().long(), ref)


def test_reference_sources_in_range_and_gather_shape():
    """Mirrors tests/test_expert_routing.py:103-132."""
    from lightning_router.kernels.expert_routing import expert_routing_forward, expert_routing_gather
    tokens, ids, w, tok = _make_test_data()
    perm, offs, rw, src = expert_routing_forward(tokens.to(DEV), ids.to(DEV), w.to(DEV), tok.to(DEV), 4)
    assert int(src.min()) >= 0 and int(src.max()) < tokens.shape[0]
    out = expert_routing_gather(perm, rw, src, tokens.shape[0])
    assert out.shape == tokens.shape


def test_reference_round_trip():
    """Mirrors tests/test_expert_routing.py:134-160 (with capacity large enough to keep all)."""
    from lightning_router.kernels.expert_routing import expert_routing_forward, expert_routing_gather
    T, d, E, k = 32, 128, 4, 2
    tokens, ids, w, tok = _make_test_data(T, d, E, k, seed=5)
    perm, offs, rw, src = expert_routing_forward(tokens.to(DEV), ids.to(DEV), w.to(DEV),
                                                 tok.to(DEV), E, capacity_factor=float(E))
    out = expert_routing_gather(perm, rw, src, T)
    ref = torch.zeros(T, d)
    for s in range(ids.numel()):
        ref[tok[s]] += w[s] * tokens[tok[s]].float()
    torch.testing.assert_close(out.float().cpu(), ref, atol=1e-2, rtol=1e-2)
    # tighter: fp32 accumulation and a single fp16 rounding
    torch.testing.assert_close(out.float().cpu(), ref, atol=2e-3, rtol=1e-3)


@pytest.mark.parametrize("name", ["r_drop", "r_nodrop", "r_e8"])
def test_matches_reference_triton_kernel_fixtures(name):
    from lightning_router.kernels.expert_routing import expert_routing_forward, expert_routing_gather
    z = golden("routing_interp")
    E = int(z[f"{name}_E"])
    x, ids, w, tok = (torch.from_numpy(z[f"{name}_{n}"]) for n in ("x", "ids", "w", "tok"))
    perm, offs, rw, src = expert_routing_forward(x.to(DEV), ids.to(DEV), w.to(DEV), tok.to(DEV), E,
                                                 float(z[f"{name}_cf"]))
    np.testing.assert_array_equal(_np(offs), z[f"{name}_offsets"])
    C = orc.capacity(ids.numel(), E, float(z[f"{name}_cf"]))
    r = orc.dispatch(z[f"{name}_ids"], z[f"{name}_w"], z[f"{name}_tok"], E, C)
    kr = r.dst[r.kept]
    np.testing.assert_array_equal(_np(src)[kr], z[f"{name}_src"][kr])
    np.testing.assert_array_equal(_np(rw)[kr], z[f"{name}_rw"][kr])
    np.testing.assert_array_equal(_np(perm)[kr].view(np.uint16), z[f"{name}_perm"][kr].view(np.uint16))
    if f"{name}_gather" in z:
        out = expert_routing_gather(perm, rw, src, x.shape[0])
        np.testing.assert_allclose(_np(out).astype(np.float32), z[f"{name}_gather"].astype(np.float32),
                                   rtol=2e-3, atol=2e-3)


@pytest.mark.parametrize("R,T,d", [(500, 200, 64), (1, 5, 8), (3000, 700, 256), (0, 4, 16)])
def test_gather_general_matches_oracle(R, T, d):
    from lightning_router.kernels.expert_routing import expert_routing_gather
    g = torch.Generator().manual_seed(R + T)
    y = torch.randn(max(R, 1), d, generator=g).half()[:R]
    src = torch.randint(0, T, (R,), generator=g, dtype=torch.int32)
    rw = torch.rand(R, generator=g)
    rw[torch.rand(R, generator=g) < 0.2] = 0.0
    out = expert_routing_gather(y.to(DEV), rw.to(DEV), src.to(DEV), T)
    ref = orc.gather_rows(_np(y), _np(rw), _np(src), T)
    np.testing.assert_allclose(_np(out).astype(np.float32), ref, rtol=1e-3, atol=1e-3)
    # deterministic: a second call is bit-identical
    out2 = expert_routing_gather(y.to(DEV), rw.to(DEV), src.to(DEV), T)
    assert torch.equal(out, out2)


@pytest.mark.parametrize("T,d,E,k,cf", [(1000, 256, 8, 2, 1.0), (513, 128, 64, 6, 1.5), (64, 4096, 8, 2, 1.25)])
def test_combine_matches_oracle(T, d, E, k, cf):
    from lightning_router.kernels.expert_routing import combine, topk_gating_dispatch
    g = torch.Generator().manual_seed(11)
    x = torch.randn(T, d, generator=g).half()
    logits = torch.randn(T, E, generator=g)
    plan = topk_gating_dispatch(x.to(DEV), logits.to(DEV), k, cf, fill_dropped=False)
    y = torch.randn(T * k, d, generator=g).half()
    out = combine(y.to(DEV), plan.gate_weights, plan.slot_pos, T, k)
    ids, w, _ = orc.topk_gating(_np(logits), k)
    r = orc.dispatch(ids.reshape(-1), w.reshape(-1), np.repeat(np.arange(T), k), E, plan.capacity)
    ref = orc.combine_slots(_np(y), r, T)
    np.testing.assert_allclose(_np(out).astype(np.float32), ref, rtol=2e-3, atol=2e-3)


def test_bad_expert_id_is_flagged_not_fatal():
    from lightning_router import _ext
    from lightning_router.kernels.expert_routing import expert_routing_forward_ex
    tokens, ids, w, tok = _make_test_data(64, 64, 4, 2)
    ids[5] = 9
    _ext.check_device_errors()
    perm, offs, rw, src, kept, pos = expert_routing_forward_ex(
        tokens.to(DEV), ids.to(DEV), w.to(DEV), tok.to(DEV), 4, 4.0)
    assert int(pos[5]) == -1
    assert int(offs[-1]) == ids.numel() - 1
    with pytest.raises(RuntimeError, match="expert id"):
        _ext.check_device_errors()


def test_gate_logits_matches_fp32_reference():
    from lightning_router.kernels.expert_routing import gate_logits
    for T, d, E in [(100, 256, 8), (37, 64, 64), (5, 4096, 4), (300, 2048, 33)]:
        g = torch.Generator().manual_seed(T)
        h = torch.randn(T, d, generator=g).half()
        wg = (torch.randn(E, d, generator=g) * 0.02).half()
        bias = torch.randn(E, generator=g)
        out = gate_logits(h.to(DEV), wg.to(DEV), bias.to(DEV))
        ref = orc.gate_logits(_np(h), _np(wg), _np(bias))
        np.testing.assert_allclose(_np(out), ref, rtol=1e-4, atol=1e-4)


@pytest.mark.slow
@pytest.mark.parametrize("T,cf", [(262144, 1.0), (262144, 2.0), (16384, 1.0)])
def test_dispatch_sweep_full_size_properties(T, cf):
    """Sweep sizes (d=4096, E=8, k=2): routing bit-exact vs the oracle, rows by property."""
    from lightning_router.kernels.expert_routing import combine, topk_gating_dispatch
    from lightning_router.workloads import SWEEP_TOKENS, sweep_inputs
    x, logits = sweep_inputs(T, SWEEP_TOKENS.index(T) if T in SWEEP_TOKENS else 0, gen_device=DEV)
    plan = topk_gating_dispatch(x, logits, 2, cf, fill_dropped=True)
    r = check_plan(plan, None, logits.cpu(), 2, cf)
    kept_rows = torch.from_numpy(r.dst[r.kept]).to(DEV)
    src = plan.source_indices[kept_rows].long()
    assert torch.equal(plan.permuted[kept_rows], x[src])
    drop_rows = torch.from_numpy(r.dst[~r.kept]).to(DEV)
    assert int(plan.permuted[drop_rows].abs().sum()) == 0 if drop_rows.numel() else True
    # identity experts: combine == sum_j w_j x_t over kept slots (fp32), one rounding
    out = combine(plan.permuted, plan.gate_weights, plan.slot_pos, T, 2)
    wk = torch.where(plan.slot_pos >= 0, plan.gate_weights, torch.zeros_like(plan.gate_weights))
    ref = (x.float() * wk.view(T, 2).sum(1, keepdim=True))
    torch.testing.assert_close(out.float(), ref, rtol=2e-3, atol=2e-3)


GATE_DISPATCH_CASES = [
    # T, d, E, k, cf, bias, fill
    (64, 4096, 8, 2, 1.25, False, False),     # decode layer shape
    (1, 64, 4, 1, 1.0, False, True),
    (37, 256, 64, 6, 1.5, True, True),
    (256, 1024, 33, 8, 0.5, True, False),     # the one-block limit, heavy drops
    (200, 8192, 16, 2, 1.0, False, True),     # two shared-memory pieces per d-chunk
    (130, 16, 8, 2, 1.0, True, True),         # d smaller than the 8 chunks
    (257, 512, 8, 2, 1.25, False, True),      # just above the limit: two-kernel path
    (1000, 256, 64, 6, 1.5, True, False),
]


@pytest.mark.parametrize("T,d,E,k,cf,use_bias,fill", GATE_DISPATCH_CASES)
def test_gate_topk_dispatch_equals_two_kernel_path(T, d, E, k, cf, use_bias, fill):
    """Gate projection + dispatch in one call: logits bit-identical to gate_logits,
    every plan output identical to topk_gating_dispatch on those logits, and the
    routing bit-exact against the oracle."""
    from lightning_router.kernels.expert_routing import (
        gate_logits, gate_topk_gating_dispatch, topk_gating_dispatch)
    g = torch.Generator().manual_seed(T * 7 + E)
    x = torch.randn(T, d, generator=g).half().to(DEV)
    wg = (torch.randn(E, d, generator=g) * 0.05).half().to(DEV)
    bias = torch.randn(E, generator=g).to(DEV) if use_bias else None
    logits, plan = gate_topk_gating_dispatch(x, wg, bias, k, cf, fill_dropped=fill)
    ref_logits = gate_logits(x, wg, bias)
    assert torch.equal(logits, ref_logits)
    ref = topk_gating_dispatch(x, ref_logits, k, cf, fill_dropped=fill)
    for name in ("expert_ids", "gate_weights", "token_indices", "offsets", "kept_counts",
                 "routing_weights", "source_indices", "slot_pos"):
        assert torch.equal(getattr(plan, name), getattr(ref, name)), name
    assert torch.equal(plan.aux_loss, ref.aux_loss)
    kept = plan.slot_pos >= 0
    rows = plan.slot_pos[kept].long()
    assert torch.equal(plan.permuted[rows], ref.permuted[rows])
    if fill:
        assert torch.equal(plan.permuted, ref.permuted)
    check_plan(plan, x.cpu(), logits.cpu(), k, cf, fill=fill)
    # routing metadata only
    logits2, plan2 = gate_topk_gating_dispatch(x, wg, bias, k, cf, permute=False)
    assert torch.equal(logits2, logits) and plan2.permuted.numel() == 0
    assert torch.equal(plan2.slot_pos, plan.slot_pos)


def test_combine_small_batch_split_rows_bit_identical():
    """Small batches spread each token's row over several warps; every output
    element keeps its slot-order fp32 accumulation, so the result equals the
    one-warp-per-token combine of a large batch holding the same tokens."""
    from lightning_router.kernels.expert_routing import combine, topk_gating_dispatch
    T, d, E, k, reps = 64, 4096, 8, 2, 40
    g = torch.Generator().manual_seed(5)
    x = torch.randn(T, d, generator=g).half().to(DEV)
    logits = torch.randn(T, E, generator=g).to(DEV)
    plan = topk_gating_dispatch(x, logits, k, 1.0)
    y = torch.randn(T * k, d, generator=g).half().to(DEV)
    small = combine(y, plan.gate_weights, plan.slot_pos, T, k)
    big = combine(y, plan.gate_weights.repeat(reps), plan.slot_pos.repeat(reps), T * reps, k)
    assert torch.equal(big[:T], small)
    assert torch.equal(big[T * (reps - 1):], small)
