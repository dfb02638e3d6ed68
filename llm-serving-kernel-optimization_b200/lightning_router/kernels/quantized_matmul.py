"""W4A16 GEMMs on the B200 tensor cores (tcgen05).

Drop-in for the reference's ``lightning_router/kernels/quantized_matmul.py:122-173``
(:func:`quantized_matmul`) plus the grouped expert GEMM used by ``ExpertGroup``
and ``MoELayer`` (:func:`grouped_w4a16`).

Weights stay in the reference's packed format (``qweight`` (K, N/8) int32,
``scales`` (K/g, N) fp16, ``zeros`` (K/g, N/8) int32).  A small per-expert
"weight table" (TMA descriptors + pointers, ~900 B per expert) is encoded once
per weight set and kept on the device together with references to the weight
tensors it points to (it holds only addresses and strides, so it stays valid
when a buffer is updated in place).  Modules keep their own tables; the
functional :func:`quantized_matmul` uses a small bounded cache.  Limits of the tcgen05 kernel: ``K % 64 == 0``,
``group_size % 64 == 0``, ``N % 32 == 0`` (``N % 64 == 0`` for the fused SwiGLU
mode), at most 256 experts per launch.
"""

from __future__ import annotations

from collections import OrderedDict
from typing import NamedTuple

import torch

from lightning_router import _ext

FFN_MODE_PLAIN = _ext.FFN_MODE_PLAIN
FFN_MODE_SILU = _ext.FFN_MODE_SILU
FFN_MODE_SWIGLU = _ext.FFN_MODE_SWIGLU

class WeightTable(NamedTuple):
    """Device table plus the weight tensors it points to.

    The table holds raw addresses; keeping ``refs`` alive keeps those addresses
    valid for as long as the table is in use.
    """
    table: torch.Tensor
    refs: tuple


_TABLE_CACHE: "OrderedDict[tuple, WeightTable]" = OrderedDict()
_TABLE_CACHE_MAX = 16


def _key(t: torch.Tensor | None):
    if t is None:
        return None
    return (t.data_ptr(), tuple(t.shape), t.device.index)


def weight_table(qweights, scales, zeros, num_experts: int, d_model: int, d_ff: int,
                 group_size: int, gated: bool, cache: bool = True) -> WeightTable:
    """Device-resident weight table for ``num_experts`` experts.

    ``qweights[e*3 + m]`` (m = 0 gate, 1 up, 2 down; ``None`` when absent) with
    gate/up of shape (d_model, d_ff/8) and down of shape (d_ff, d_model/8).
    Cached entries keep their weight tensors alive (at most 16 entries).
    """
    key = table_key(qweights, scales, zeros, num_experts, d_model, d_ff, group_size, gated)
    hit = _TABLE_CACHE.get(key) if cache else None
    if hit is not None:
        _TABLE_CACHE.move_to_end(key)
        return hit
    dev = next(t.device for t in qweights if t is not None)
    if group_size % 64 != 0:
        raise NotImplementedError(
            f"W4A16 tcgen05 kernel needs group_size % 64 == 0 (got {group_size})")
    host = _ext.ops().encode_weight_table(list(qweights), list(scales), list(zeros),
                                          int(num_experts), int(d_model), int(d_ff),
                                          int(group_size), bool(gated))
    table = torch.empty(host.numel(), dtype=torch.uint8, device=dev)
    assert table.data_ptr() % 128 == 0
    table.copy_(host)
    refs = tuple(t for t in (*qweights, *scales, *zeros) if t is not None)
    wt = WeightTable(table, refs)
    if cache:
        _TABLE_CACHE[key] = wt
        while len(_TABLE_CACHE) > _TABLE_CACHE_MAX:
            _TABLE_CACHE.popitem(last=False)
    return wt


def table_key(qweights, scales, zeros, *extra) -> tuple:
    return (tuple(_key(t) for t in qweights), tuple(_key(t) for t in scales),
            tuple(_key(t) for t in zeros), *extra)


def clear_weight_tables() -> None:
    _TABLE_CACHE.clear()


def grouped_w4a16(table: WeightTable, num_experts: int, mode: int, mat: int, A: torch.Tensor,
                  N: int, seg_start: torch.Tensor | None, seg_len: torch.Tensor | None,
                  max_rows: int, out: torch.Tensor | None = None) -> torch.Tensor:
    """Grouped GEMM over expert row segments; see ``lr_grouped_w4a16_gemm``."""
    _ext.require_cuda(A)
    err = _ext.error_word(A.device.index)
    return _ext.ops().grouped_w4a16_gemm(table.table, int(num_experts), int(mode), int(mat),
                                         A.contiguous(), int(N), seg_start, seg_len,
                                         int(max_rows), out, err)


def quantized_matmul(
    A: torch.Tensor,
    B_packed: torch.Tensor,
    scales: torch.Tensor,
    zeros: torch.Tensor,
    N: int,
    group_size: int = 128,
    block_m: int = 128,
    block_n: int = 64,
    block_k: int = 32,
) -> torch.Tensor:
    """``C = A @ dequant(B)`` with A (M, K) fp16 and B packed INT4; returns (M, N) fp16.

    ``block_*`` are accepted for signature compatibility and ignored: the tile
    shape is chosen by the kernel (128 weight columns x up to 256 rows of A).
    """
    M, K = A.shape
    assert A.dtype == torch.float16
    assert B_packed.dtype == torch.int32
    _ext.require_cuda(A, B_packed, scales, zeros)
    if B_packed.shape != (K, N // 8):
        raise ValueError(f"B_packed shape {tuple(B_packed.shape)} != ({K}, {N // 8})")
    if K % 64 != 0 or N % 32 != 0:
        raise NotImplementedError(f"W4A16 kernel needs K % 64 == 0 and N % 32 == 0 (K={K}, N={N})")
    if M == 0:
        return torch.empty(0, N, dtype=torch.float16, device=A.device)
    # cache only tables over the caller's own tensors, never over temporaries
    persistent = B_packed.is_contiguous() and scales.is_contiguous() and zeros.is_contiguous()
    table = weight_table([None, None, B_packed.contiguous()], [None, None, scales.contiguous()],
                         [None, None, zeros.contiguous()], 1, N, K, group_size, False,
                         cache=persistent)
    return grouped_w4a16(table, 1, FFN_MODE_PLAIN, 2, A, N, None, None, M)
