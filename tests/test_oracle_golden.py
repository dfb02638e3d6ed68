"""Pin the CPU oracle against golden vectors produced by the reference itself.

The fixtures in ``tests/golden`` come from ``tests/golden/make_golden.py``, which
runs the reference's own PyTorch code and its Triton kernels (interpreted on
the CPU) on seeded inputs.
"""

from __future__ import annotations

import numpy as np
import pytest

import oracle as orc
from conftest import golden


def test_pack_unpack_matches_reference():
    z = golden("pack_weights")
    np.testing.assert_array_equal(orc.pack_int4(z["pack_q"]), z["pack_packed"])
    np.testing.assert_array_equal(orc.unpack_int4(z["pack_packed"], 64), z["pack_unpacked"])
    np.testing.assert_array_equal(z["pack_unpacked"], z["pack_q"])


@pytest.mark.parametrize("name", ["q128", "q64", "q32"])
def test_quantize_dequantize_bit_exact(name):
    z = golden("pack_weights")
    gs = int(z[f"{name}_gs"])
    qw, s, zz = orc.quantize_tensor(z[f"{name}_w"], gs)
    np.testing.assert_array_equal(qw, z[f"{name}_qweight"])
    np.testing.assert_array_equal(s.view(np.uint16), z[f"{name}_scales"].view(np.uint16))
    np.testing.assert_array_equal(zz, z[f"{name}_zeros"])
    N = z[f"{name}_w"].shape[1]
    deq = orc.dequantize_tensor(z[f"{name}_qweight"], z[f"{name}_scales"], z[f"{name}_zeros"], gs, N)
    np.testing.assert_array_equal(deq.view(np.uint16), z[f"{name}_deq"].view(np.uint16))


def test_quantize_rejects_bad_group():
    with pytest.raises(AssertionError):
        orc.quantize_tensor(np.zeros((100, 64), np.float16), 128)


@pytest.mark.parametrize("name", ["g4", "g8", "g64"])
def test_gating_matches_reference(name):
    z = golden("gating")
    k = int(z[f"{name}_k"])
    logits = z[f"{name}_logits"]
    ids, w, probs = orc.topk_gating(logits, k)
    np.testing.assert_array_equal(ids.reshape(-1), z[f"{name}_ids"])
    np.testing.assert_allclose(w.reshape(-1), z[f"{name}_w"], rtol=1e-6, atol=0)
    T = logits.shape[0]
    np.testing.assert_array_equal(np.repeat(np.arange(T), k), z[f"{name}_tok"])
    aux = orc.aux_loss(ids.reshape(-1), probs, logits.shape[1], k, 0.01)
    assert abs(aux - float(z[f"{name}_aux"])) <= 1e-5 * abs(float(z[f"{name}_aux"]))
    # the fp32 gate GEMM restatement agrees with nn.Linear to fp32 rounding
    np.testing.assert_allclose(orc.gate_logits(z[f"{name}_x"], z[f"{name}_wg"]), logits, rtol=1e-5, atol=1e-5)


@pytest.mark.parametrize("name", ["r_drop", "r_nodrop", "r_e8"])
def test_dispatch_matches_reference_triton_kernels(name):
    z = golden("routing_interp")
    E = int(z[f"{name}_E"])
    ids, w, tok, x = z[f"{name}_ids"], z[f"{name}_w"], z[f"{name}_tok"], z[f"{name}_x"]
    C = orc.capacity(ids.size, E, float(z[f"{name}_cf"]))
    r = orc.dispatch(ids, w, tok, E, C)
    np.testing.assert_array_equal(r.offsets, z[f"{name}_offsets"])
    kept_rows = r.dst[r.kept]
    # kept rows are fully defined by the reference; dropped rows are left uninitialised there
    np.testing.assert_array_equal(r.src_idx[kept_rows], z[f"{name}_src"][kept_rows])
    np.testing.assert_array_equal(r.routing_w[kept_rows], z[f"{name}_rw"][kept_rows])
    perm = orc.permute_rows(x, r)
    np.testing.assert_array_equal(perm[kept_rows].view(np.uint16), z[f"{name}_perm"][kept_rows].view(np.uint16))
    if f"{name}_gather" in z:
        assert r.kept.all()
        ref = z[f"{name}_gather"].astype(np.float32)
        ours = orc.gather_rows(perm, r.routing_w, r.src_idx, x.shape[0])
        # reference accumulates with fp16 atomics; the oracle in fp32
        np.testing.assert_allclose(ours, ref, rtol=2e-3, atol=2e-3)


@pytest.mark.parametrize("name", ["m1", "m2"])
def test_quantized_matmul_matches_reference_kernel(name):
    z = golden("qmm_interp")
    gs, N = int(z[f"{name}_gs"]), int(z[f"{name}_N"])
    w = orc.dequantize_tensor(z[f"{name}_qweight"], z[f"{name}_scales"], z[f"{name}_zeros"], gs, N)
    c = z[f"{name}_a"].astype(np.float32) @ w.astype(np.float32)
    ref = z[f"{name}_c"].astype(np.float32)
    err = np.linalg.norm(c - ref) / np.linalg.norm(c)
    assert err < 1e-3, err


@pytest.mark.parametrize("name", ["l4", "l8"])
def test_layer_matches_reference_torch_path(name):
    z = golden("layer_torch")
    B, Sq, d, f, E, k, gs = (int(v) for v in z[f"{name}_dims"])
    experts = []
    for e in range(E):
        ex = {}
        for mat, (K, N) in {"gate": (d, f), "up": (d, f), "down": (f, d)}.items():
            ex[mat] = orc.dequantize_tensor(z[f"{name}_e{e}_{mat}_qweight"], z[f"{name}_e{e}_{mat}_scales"],
                                            z[f"{name}_e{e}_{mat}_zeros"], gs, N)
        experts.append(ex)
    x = z[f"{name}_x"].reshape(-1, d)
    logits = z[f"{name}_logits"]
    T = x.shape[0]
    # the reference torch path applies no capacity: use C = S
    out, aux, r = orc.moe_layer(x, logits, k, 1.0, experts, cap=T * k)
    ref = z[f"{name}_out"].reshape(-1, d)
    np.testing.assert_allclose(out, ref, rtol=1e-4, atol=1e-5)
    assert abs(aux - float(z[f"{name}_aux"])) <= 1e-5 * abs(float(z[f"{name}_aux"]))


@pytest.mark.parametrize("name", ["l4", "l8"])
def test_torch_path_port_matches_reference_layer(name):
    """The timed CPU baseline (a port of the reference's torch-routing MoELayer)
    reproduces the reference's own outputs and aux loss on its fixture."""
    import torch

    from oracle import torch_path
    z = golden("layer_torch")
    B, Sq, d, f, E, k, gs = (int(v) for v in z[f"{name}_dims"])
    experts = []
    for e in range(E):
        ex = {}
        for m in ("gate", "up", "down"):
            N = f if m != "down" else d
            ex[m] = torch.from_numpy(orc.dequantize_tensor(
                z[f"{name}_e{e}_{m}_qweight"], z[f"{name}_e{e}_{m}_scales"],
                z[f"{name}_e{e}_{m}_zeros"], gs, N).astype(np.float32))
        experts.append(ex)
    x = torch.from_numpy(z[f"{name}_x"]).reshape(-1, d)
    wg = torch.from_numpy(z[f"{name}_wg"])
    out, aux = torch_path.moe_layer(x, wg, torch_path.linear_experts(experts), k)
    ref = z[f"{name}_out"].reshape(-1, d)
    np.testing.assert_allclose(out.numpy(), ref, rtol=1e-5, atol=1e-6)
    assert abs(float(aux) - float(z[f"{name}_aux"])) <= 1e-6 * abs(float(z[f"{name}_aux"]))


def test_vectorized_routing_port_is_weighted_identity():
    """Identity experts: the sweep baseline returns sum_j w_j * x_t per token."""
    import torch

    from oracle import torch_path
    g = torch.Generator().manual_seed(5)
    T, d, E, k = 37, 16, 4, 2
    x = torch.randn(T, d, generator=g).half()
    ids, w, _ = orc.topk_gating(torch.randn(T, E, generator=g).numpy(), k)
    ids, w = torch.from_numpy(ids.reshape(-1)).long(), torch.from_numpy(w.reshape(-1))
    tok = torch.arange(T).repeat_interleave(k)
    out = torch_path.vectorized_routing(x, ids, w, tok, E)
    ref = (x.float() * w.view(T, k).sum(1, keepdim=True)).half()
    assert torch.allclose(out.float(), ref.float(), atol=2e-3)
