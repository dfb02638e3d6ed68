"""Generate golden vectors from the reference implementation itself.

Run where a checkout of the reference is available (read-only is enough):

    LR_REFERENCE_PATH=<reference checkout> python tests/golden/make_golden.py

It imports the reference package ``lightning_router`` from that checkout and
runs, on seeded inputs:

* ``quantization/pack_weights.py``: ``_pack_int4``/``_unpack_int4``,
  ``quantize_tensor``/``dequantize_tensor``;
* ``models/gating.py``: ``TopKGating.forward`` in fp32;
* ``models/moe_layer.py``: ``MoELayer.forward`` on the torch routing path
  (fp32, experts loaded with the dequantized INT4 weights);
* ``kernels/expert_routing.py`` and ``kernels/quantized_matmul.py``: the
  reference's Triton kernels, executed on the CPU by ``TRITON_INTERPRET=1``
  (slot-ordered capacity drops, uncapped CSR offsets).

The outputs are stored as ``.npz`` files beside this script.  The test suite
never imports the reference; it reads these fixtures only.
"""

from __future__ import annotations

import os
import sys
from pathlib import Path

os.environ.setdefault("TRITON_INTERPRET", "1")

import numpy as np
import torch

REF = os.environ.get("LR_REFERENCE_PATH")
if not REF:
    raise SystemExit("set LR_REFERENCE_PATH to a checkout of the reference repository")
OUT = Path(__file__).resolve().parent


def _import_reference():
    # The product package has the same import name; make sure the reference wins here.
    for m in [m for m in sys.modules if m == "lightning_router" or m.startswith("lightning_router.")]:
        del sys.modules[m]
    sys.path.insert(0, REF)
    import lightning_router  # noqa: F401
    assert os.path.realpath(lightning_router.__file__).startswith(os.path.realpath(REF)), lightning_router.__file__
    return lightning_router


def gen_pack(g: torch.Generator):
    from lightning_router.quantization.pack_weights import (
        _pack_int4, _unpack_int4, quantize_tensor, dequantize_tensor)
    out = {}
    q = torch.randint(0, 16, (4, 64), dtype=torch.int32, generator=g)
    out["pack_q"] = q.numpy()
    out["pack_packed"] = _pack_int4(q).numpy()
    out["pack_unpacked"] = _unpack_int4(_pack_int4(q), 64).numpy()
    for name, (K, N, gs) in {"q128": (256, 64, 128), "q64": (256, 128, 64), "q32": (128, 48, 32)}.items():
        w = (torch.randn(K, N, generator=g) * 0.02).half()
        qw, s, z = quantize_tensor(w, group_size=gs)
        out[f"{name}_w"] = w.numpy()
        out[f"{name}_qweight"] = qw.numpy()
        out[f"{name}_scales"] = s.numpy()
        out[f"{name}_zeros"] = z.numpy()
        out[f"{name}_deq"] = dequantize_tensor(qw, s, z, gs, N).numpy()
        out[f"{name}_gs"] = np.int64(gs)
    np.savez_compressed(OUT / "pack_weights.npz", **out)


def gen_gating(g: torch.Generator):
    from lightning_router.models.gating import TopKGating
    out = {}
    for name, (T, d, E, k) in {"g4": (40, 64, 4, 2), "g8": (96, 128, 8, 2), "g64": (64, 96, 64, 6)}.items():
        gate = TopKGating(d, E, k, load_balance_weight=0.01)
        with torch.no_grad():
            gate.gate_proj.weight.copy_(torch.randn(E, d, generator=g) * 0.05)
        x = torch.randn(T, d, generator=g)
        with torch.no_grad():
            logits = gate.gate_proj(x)
            ids, w, tok, aux = gate(x)
        out[f"{name}_x"] = x.numpy()
        out[f"{name}_wg"] = gate.gate_proj.weight.detach().numpy()
        out[f"{name}_logits"] = logits.numpy()
        out[f"{name}_ids"] = ids.numpy()
        out[f"{name}_w"] = w.numpy()
        out[f"{name}_tok"] = tok.numpy()
        out[f"{name}_aux"] = np.float64(aux.item())
        out[f"{name}_k"] = np.int64(k)
    np.savez_compressed(OUT / "gating.npz", **out)


def gen_routing_interp(g: torch.Generator):
    from lightning_router.kernels.expert_routing import expert_routing_forward, expert_routing_gather
    out = {}
    cases = {"r_drop": (16, 32, 4, 2, 1.0), "r_nodrop": (24, 64, 4, 2, 4.0), "r_e8": (48, 32, 8, 2, 1.25)}
    for name, (T, d, E, k, cf) in cases.items():
        x = torch.randn(T, d, generator=g).half()
        ids = torch.randint(0, E, (T * k,), dtype=torch.int32, generator=g)
        w = torch.rand(T * k, generator=g)
        tok = torch.arange(T).unsqueeze(1).expand(-1, k).reshape(-1).int()
        perm, offs, rw, src = expert_routing_forward(x, ids, w, tok, E, capacity_factor=cf)
        out[f"{name}_x"] = x.numpy()
        out[f"{name}_ids"] = ids.numpy()
        out[f"{name}_w"] = w.numpy()
        out[f"{name}_tok"] = tok.numpy()
        out[f"{name}_cf"] = np.float64(cf)
        out[f"{name}_E"] = np.int64(E)
        out[f"{name}_perm"] = perm.numpy()
        out[f"{name}_offsets"] = offs.numpy()
        out[f"{name}_rw"] = rw.numpy()
        out[f"{name}_src"] = src.numpy()
        if cf >= E:  # no drops: every row is defined, so the reference gather is well defined
            y = perm
            gat = expert_routing_gather(y, rw, src, T)
            out[f"{name}_gather"] = gat.numpy()
    np.savez_compressed(OUT / "routing_interp.npz", **out)


def gen_qmm_interp(g: torch.Generator):
    from lightning_router.quantization.pack_weights import quantize_tensor
    from lightning_router.kernels.quantized_matmul import quantized_matmul
    out = {}
    for name, (M, K, N, gs) in {"m1": (32, 256, 64, 128), "m2": (40, 128, 128, 64)}.items():
        a = torch.randn(M, K, generator=g).half()
        w = (torch.randn(K, N, generator=g) * 0.02).half()
        qw, s, z = quantize_tensor(w, group_size=gs)
        c = quantized_matmul(a, qw, s, z, N=N, group_size=gs)
        out[f"{name}_a"] = a.numpy()
        out[f"{name}_qweight"] = qw.numpy()
        out[f"{name}_scales"] = s.numpy()
        out[f"{name}_zeros"] = z.numpy()
        out[f"{name}_c"] = c.numpy()
        out[f"{name}_gs"] = np.int64(gs)
        out[f"{name}_N"] = np.int64(N)
    np.savez_compressed(OUT / "qmm_interp.npz", **out)


def gen_layer_torch(g: torch.Generator):
    """Reference MoELayer (torch routing, fp32) with experts holding dequantized INT4 weights."""
    from lightning_router.config import ModelConfig, MoEConfig, QuantizationConfig, KernelConfig
    from lightning_router.models.moe_layer import MoELayer
    from lightning_router.quantization.pack_weights import quantize_tensor, dequantize_tensor
    out = {}
    for name, (B, Sq, d, f, E, k, gs) in {"l4": (2, 8, 64, 128, 4, 2, 64), "l8": (3, 16, 128, 256, 8, 2, 128)}.items():
        layer = MoELayer(ModelConfig(hidden_size=d, intermediate_size=f),
                         MoEConfig(num_experts=E, num_experts_per_token=k, routing_implementation="torch"),
                         QuantizationConfig(enabled=False), KernelConfig())
        with torch.no_grad():
            layer.gate.gate_proj.weight.copy_(torch.randn(E, d, generator=g) * 0.05)
            for e in range(E):
                ex = layer.experts.experts[e]
                for mat, (K, N) in {"gate": (d, f), "up": (d, f), "down": (f, d)}.items():
                    w = (torch.randn(K, N, generator=g) * 0.02).half()
                    qw, s, z = quantize_tensor(w, group_size=gs)
                    deq = dequantize_tensor(qw, s, z, gs, N)
                    getattr(ex, f"{mat}_proj").weight.copy_(deq.float().t())
                    out[f"{name}_e{e}_{mat}_qweight"] = qw.numpy()
                    out[f"{name}_e{e}_{mat}_scales"] = s.numpy()
                    out[f"{name}_e{e}_{mat}_zeros"] = z.numpy()
        x = torch.randn(B, Sq, d, generator=g).half().float()
        with torch.no_grad():
            logits = layer.gate.gate_proj(x.view(-1, d))
            y, aux = layer(x)
        out[f"{name}_x"] = x.numpy()
        out[f"{name}_wg"] = layer.gate.gate_proj.weight.detach().numpy()
        out[f"{name}_logits"] = logits.numpy()
        out[f"{name}_out"] = y.numpy()
        out[f"{name}_aux"] = np.float64(aux.item())
        out[f"{name}_dims"] = np.array([B, Sq, d, f, E, k, gs], np.int64)
    np.savez_compressed(OUT / "layer_torch.npz", **out)


def main():
    _import_reference()
    g = torch.Generator().manual_seed(20261201)
    gen_pack(g)
    gen_gating(g)
    gen_routing_interp(g)
    gen_qmm_interp(g)
    gen_layer_torch(g)
    for p in sorted(OUT.glob("*.npz")):
        print(p.name, p.stat().st_size)


if __name__ == "__main__":
    main()
