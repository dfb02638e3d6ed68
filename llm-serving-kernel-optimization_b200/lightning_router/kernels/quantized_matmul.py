"""W4A16 GEMMs on the B200: tcgen05 tensor cores for the model shapes.

Drop-in for the reference's ``lightning_router/kernels/quantized_matmul.py:122-173``
(:func:`quantized_matmul`) plus the grouped expert GEMM used by ``ExpertGroup``
and ``MoELayer`` (:func:`grouped_w4a16`).

Weights stay in the reference's packed format (``qweight`` (K, N/8) int32,
``scales`` (K/g, N) fp16, ``zeros`` (K/g, N/8) int32).  A small per-expert
"weight table" (TMA descriptors + pointers, ~1.3 KB per expert) is encoded once
per weight set and kept on the device together with references to the weight
tensors it points to (it holds only addresses and strides, so it stays valid
when a buffer is updated in place).  Modules keep their own tables; the
functional :func:`quantized_matmul` uses a small bounded cache.

Every shape of the packed format is accepted (``K % group_size == 0``,
``N % 8 == 0``, any M), as the reference's masked kernel does.  The kernel
follows the shape: the tcgen05 kernel when ``K % 64 == 0``,
``group_size % 64 == 0`` and ``N % 32 == 0``; an mma.sync kernel for
``K % 8 == 0``, ``N % 32 == 0`` and a power-of-two group of at least 16 (e.g.
group 32); CUDA cores otherwise (e.g. N = 48).  At most 256 experts per launch.
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
    group_size: int


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
    host = _ext.ops().encode_weight_table(list(qweights), list(scales), list(zeros),
                                          int(num_experts), int(d_model), int(d_ff),
                                          int(group_size), bool(gated))
    table = torch.empty(host.numel(), dtype=torch.uint8, device=dev)
    assert table.data_ptr() % 128 == 0
    table.copy_(host)
    refs = tuple(t for t in (*qweights, *scales, *zeros) if t is not None)
    wt = WeightTable(table, refs, int(group_size))
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


# Segments of at most 32 rows (decode) run on 8-bit tensor-core operands when
# the shape allows it (K and group size multiples of 128, N % 32 == 0): token
# rows as two 8-bit terms per 128-k block, INT4 codes as bytes (see
# ``lr_grouped_w4a16_workspace_bytes``).  False keeps every call on the
# fp16-operand kernels.
INT8_OPERANDS = True


def grouped_w4a16(table: WeightTable, num_experts: int, mode: int, mat: int, A: torch.Tensor,
                  N: int, seg_start: torch.Tensor | None, seg_len: torch.Tensor | None,
                  max_rows: int, out: torch.Tensor | None = None,
                  int8_operands: bool | None = None) -> torch.Tensor:
    """Grouped GEMM over expert row segments; see ``lr_grouped_w4a16_gemm``.

    ``int8_operands`` (default :data:`INT8_OPERANDS`) lets short segments take
    the 8-bit operand kernel."""
    _ext.require_cuda(A)
    err = _ext.error_word(A.device.index)
    i8 = INT8_OPERANDS if int8_operands is None else bool(int8_operands)
    return _ext.ops().grouped_w4a16_gemm(table.table, int(num_experts), int(mode), int(mat),
                                         A.contiguous(), int(N), table.group_size, seg_start,
                                         seg_len, int(max_rows), out, err, i8)


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

    ``block_*`` are accepted for signature compatibility and ignored: the kernel
    and its tile shape are chosen from the shape.  Any M; N % 8 == 0 and
    K % group_size == 0 (the packed format's limits).
    """
    M, K = A.shape
    assert A.dtype == torch.float16
    assert B_packed.dtype == torch.int32
    _ext.require_cuda(A, B_packed, scales, zeros)
    if B_packed.shape != (K, N // 8):
        raise ValueError(f"B_packed shape {tuple(B_packed.shape)} != ({K}, {N // 8})")
    if N % 8 != 0 or group_size < 1 or K % group_size != 0:
        raise ValueError(f"packed INT4 needs N % 8 == 0 and K % group_size == 0 "
                         f"(K={K}, N={N}, group_size={group_size})")
    if scales.shape != (K // group_size, N) or zeros.shape != (K // group_size, N // 8):
        raise ValueError("scales / zeros shapes do not match (K / group_size, N) / (K / group_size, N / 8)")
    if M == 0:
        return torch.empty(0, N, dtype=torch.float16, device=A.device)
    # cache only tables over the caller's own tensors, never over temporaries
    persistent = B_packed.is_contiguous() and scales.is_contiguous() and zeros.is_contiguous()
    table = weight_table([None, None, B_packed.contiguous()], [None, None, scales.contiguous()],
                         [None, None, zeros.contiguous()], 1, N, K, group_size, False,
                         cache=persistent)
    return grouped_w4a16(table, 1, FFN_MODE_PLAIN, 2, A, N, None, None, M)
