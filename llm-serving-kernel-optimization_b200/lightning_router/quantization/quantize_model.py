"""Offline INT4 quantization of a model's expert weights, in place.

Same entry point, arguments and return value as the reference pass
(``lightning_router/quantization/quantize_model.py:34-108``): every
``nn.Linear`` whose qualified name contains one of ``target_substrings`` is
quantized with :func:`quantize_tensor` and replaced by packed buffers, and a
``{name: {"orig_norm", "quant_error"}}`` dict is returned for QA.

Three behaviours differ from the reference, where its output did not load into
its own expert module (``models/experts.py:50-56``):

* ``nn.Linear.weight`` is (out_features, in_features); the packed format is
  (K = in, N = out) (``experts.py:52`` builds ``qweight`` as (in, out/8)), so the
  weight is transposed before quantization.  The reference quantized the
  (out, in) matrix directly, which gives the transposed layer.
* the buffers are named like ``ExpertFFN``'s (``gate_qweight``, ...: the
  ``_proj`` suffix dropped) rather than ``gate_proj_qweight``, and an
  ``ExpertFFN`` (or ``ExpertGroup``) whose linears were all replaced switches
  to its quantized forward;
* the router's projection (``TopKGating.gate_proj``, whose name also contains
  ``gate_proj``) stays a float Linear: routing decisions are taken on its
  fp32 logits and the gate kernel reads it as fp16.

Layers whose dimensions do not fit the format (``in % group_size``,
``out % 8``) are skipped with a warning, as in the reference.
"""

from __future__ import annotations

import logging
from typing import Iterator

import torch
import torch.nn as nn

from lightning_router.quantization.pack_weights import dequantize_tensor, quantize_tensor

logger = logging.getLogger(__name__)


def _iter_linear_layers(module: nn.Module, prefix: str = "") -> Iterator[tuple[str, nn.Linear]]:
    """(qualified name, nn.Linear) for every Linear in the tree, depth first."""
    for name, child in module.named_children():
        full = f"{prefix}.{name}" if prefix else name
        if isinstance(child, nn.Linear):
            yield full, child
        else:
            yield from _iter_linear_layers(child, full)


def _buffer_base(attr: str) -> str:
    """``gate_proj`` -> ``gate`` (the expert module's buffer prefix)."""
    return attr[:-len("_proj")] if attr.endswith("_proj") else attr


@torch.no_grad()
def quantize_expert_weights(
    model: nn.Module,
    group_size: int = 128,
    scheme: str = "asymmetric",
    target_substrings: tuple[str, ...] = ("gate_proj", "up_proj", "down_proj"),
) -> dict[str, dict]:
    """Quantize the expert ``nn.Linear`` layers of ``model`` to packed INT4 in place.

    Returns ``{qualified_name: {"orig_norm": ||W||, "quant_error": ||W - dequant||}}``
    (Frobenius norms of the fp16 weight as stored by the Linear, (out, in)).
    """
    from lightning_router.models.experts import ExpertFFN, ExpertGroup
    from lightning_router.models.gating import TopKGating

    stats: dict[str, dict] = {}
    modules = dict(model.named_modules())
    touched: set[int] = set()
    for name, linear in list(_iter_linear_layers(model)):
        if not any(sub in name for sub in target_substrings):
            continue
        parent_name, _, attr = name.rpartition(".")
        parent = modules[parent_name] if parent_name else model
        if isinstance(parent, TopKGating):
            continue
        w = linear.weight.data.half()           # (out, in)
        N, K = w.shape
        if K % group_size != 0 or N % 8 != 0:
            logger.warning("Skipping %s (in=%d, out=%d): incompatible dims", name, K, N)
            continue
        wk = w.t().contiguous()                 # (K = in, N = out)
        qweight, scales, zeros = quantize_tensor(wk, group_size, scheme)
        recon = dequantize_tensor(qweight, scales, zeros, group_size, N)
        orig_norm = w.norm().item()
        error_norm = (wk - recon).norm().item()
        stats[name] = {"orig_norm": orig_norm, "quant_error": error_norm}
        logger.info("Quantized %-40s  error/norm = %.4f", name,
                    error_norm / (orig_norm + 1e-12))

        dev = linear.weight.device
        delattr(parent, attr)
        base = _buffer_base(attr)
        for suffix, t in (("qweight", qweight), ("scales", scales), ("zeros", zeros)):
            key = f"{base}_{suffix}"
            if key in parent._buffers:
                del parent._buffers[key]
            parent.register_buffer(key, t.to(dev))
        setattr(parent, f"{base}_N", N)
        touched.add(id(parent))

    # modules whose linears are now all packed run their quantized path
    for mod in modules.values():
        if isinstance(mod, ExpertFFN) and id(mod) in touched:
            mats = ("gate", "up", "down") if mod.gated else ("up", "down")
            if all(hasattr(mod, f"{m}_qweight") and not hasattr(mod, f"{m}_proj") for m in mats):
                mod.quantized = True
                mod.group_size = group_size
                mod._tables.clear()
    for mod in modules.values():
        if isinstance(mod, ExpertGroup) and all(e.quantized for e in mod.experts):
            mod.quantized = True
            mod.group_size = group_size
            mod._tables.clear()
    return stats
