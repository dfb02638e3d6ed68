"""Packed INT4 weight format (asymmetric / symmetric, per group along K).

Format contract of the reference, ``lightning_router/quantization/pack_weights.py:23-130``:

* ``qweight`` (K, N/8) int32 -- nibble ``i`` (bits ``4i..4i+3``) of word ``j`` holds
  column ``8j + i``;
* ``scales`` (K/g, N) fp16, ``zeros`` (K/g, N/8) int32 packed like ``qweight``;
* ``scale = max((max - min) / 15, 1e-8)``, ``zero = clamp(round(-min / scale), 0, 15)``,
  ``q = clamp(round(w / scale + zero), 0, 15)``, all in fp32 with the fp32 scale
  (the stored scale is its fp16 rounding); symmetric: ``scale = absmax / 7``, ``zero = 8``;
* ``w = fp16(fp32(scale) * (q - zero))``.

These functions are device agnostic torch code (offline / load-time work).
"""

from __future__ import annotations

import torch

_SHIFTS = torch.arange(0, 32, 4, dtype=torch.int32)


def _pack_int4(tensor: torch.Tensor) -> torch.Tensor:
    """Pack the last dimension by groups of 8 nibbles into int32 words."""
    *lead, n = tensor.shape
    assert n % 8 == 0
    nib = (tensor.to(torch.int32) & 0xF).reshape(*lead, n // 8, 8)
    shifts = _SHIFTS.to(tensor.device)
    # nibbles occupy disjoint bits, so the OR is a sum; the top nibble may set
    # the sign bit, which int32 wraps exactly like the bitwise form.
    words = (nib.to(torch.int64) << shifts.to(torch.int64)).sum(dim=-1)
    return torch.where(words >= (1 << 31), words - (1 << 32), words).to(torch.int32)


def _unpack_int4(packed: torch.Tensor, N: int) -> torch.Tensor:
    """Unpack int32 words into N nibble values along the last dimension."""
    *lead, pn = packed.shape
    assert pn == N // 8
    shifts = _SHIFTS.to(packed.device)
    nib = (packed.unsqueeze(-1) >> shifts) & 0xF
    return nib.reshape(*lead, N).to(torch.int32)


def quantize_tensor(weight: torch.Tensor, group_size: int = 128,
                    scheme: str = "asymmetric") -> tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    """Quantize a (K, N) weight matrix to the packed INT4 format.

    Returns ``(qweight (K, N/8) int32, scales (K/g, N) fp16, zeros (K/g, N/8) int32)``.
    """
    K, N = weight.shape
    assert K % group_size == 0, f"K={K} must be divisible by group_size={group_size}"
    assert N % 8 == 0, f"N={N} must be divisible by 8 for INT4 packing"
    G = K // group_size
    w = weight.float().reshape(G, group_size, N)
    if scheme == "asymmetric":
        lo = w.amin(dim=1)
        hi = w.amax(dim=1)
        scale = ((hi - lo) / 15.0).clamp(min=1e-8)
        zero = torch.round(-lo / scale).clamp(0, 15)
    else:
        scale = (w.abs().amax(dim=1) / 7.0).clamp(min=1e-8)
        zero = torch.full_like(scale, 8.0)
    q = torch.round(w / scale[:, None, :] + zero[:, None, :]).clamp(0, 15).to(torch.int32)
    return _pack_int4(q.reshape(K, N)), scale.half(), _pack_int4(zero.to(torch.int32))


def dequantize_tensor(qweight: torch.Tensor, scales: torch.Tensor, zeros: torch.Tensor,
                      group_size: int, N: int) -> torch.Tensor:
    """Packed INT4 -> fp16 (K, N): ``fp16(fp32(scale) * (q - zero))``."""
    K = qweight.shape[0]
    G = scales.shape[0]
    q = _unpack_int4(qweight, N).float().reshape(G, group_size, N)
    z = _unpack_int4(zeros, N).float()
    w = scales.float()[:, None, :] * (q - z[:, None, :])
    return w.reshape(K, N).half()
