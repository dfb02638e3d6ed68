"""Expert FFNs, reference ``lightning_router/models/experts.py:21-121``.

``ExpertFFN`` keeps the reference's checkpoint contract: quantized experts own
buffers ``{gate,up,down}_{qweight,scales,zeros}`` with shapes
``(K, N/8)`` int32, ``(K/g, N)`` fp16, ``(K/g, N/8)`` int32 and attributes
``{name}_N`` (``experts.py:50-56``).  Gated experts compute
``down(silu(gate x) * up x)``; ``activation="silu"`` experts (no gate) compute
``down(silu(up x))``.

``ExpertGroup`` runs every expert in ONE grouped tcgen05 launch per matrix
(gate and up fused into one launch with a SwiGLU epilogue) over device-side row
segments, without the reference's per-expert ``.item()`` synchronisations.
"""

from __future__ import annotations

import torch
import torch.nn as nn
import torch.nn.functional as F

from lightning_router.kernels.quantized_matmul import (
    FFN_MODE_PLAIN, FFN_MODE_SILU, FFN_MODE_SWIGLU, WeightTable, grouped_w4a16, table_key,
    weight_table)


def _first_ptr(objs) -> int:
    return next((t.data_ptr() for t in objs if t is not None), 0)


def _module_table(cache: dict, q, s, z, n, d, f, g, gated) -> WeightTable:
    """Per-module table cache keyed by the buffers' addresses and shapes."""
    key = table_key(q, s, z, n, d, f, g, gated)
    wt = cache.get(key)
    if wt is None:
        cache.clear()
        wt = cache[key] = weight_table(q, s, z, n, d, f, g, gated, cache=False)
    return wt

_MATS = ("gate", "up", "down")


class ExpertFFN(nn.Module):
    """Single expert (SwiGLU by default), optionally 4-bit quantized."""

    def __init__(self, hidden_size: int, intermediate_size: int, quantized: bool = False,
                 group_size: int = 128, activation: str = "swiglu"):
        super().__init__()
        if activation not in ("swiglu", "silu"):
            raise ValueError(f"activation must be 'swiglu' or 'silu', got {activation!r}")
        self.hidden_size = hidden_size
        self.intermediate_size = intermediate_size
        self.quantized = quantized
        self.group_size = group_size
        self.activation = activation
        self._tables: dict = {}
        gated = activation == "swiglu"
        if not quantized:
            if gated:
                self.gate_proj = nn.Linear(hidden_size, intermediate_size, bias=False)
            self.up_proj = nn.Linear(hidden_size, intermediate_size, bias=False)
            self.down_proj = nn.Linear(intermediate_size, hidden_size, bias=False)
        else:
            if gated:
                self._register_quant_buffers("gate", hidden_size, intermediate_size)
            self._register_quant_buffers("up", hidden_size, intermediate_size)
            self._register_quant_buffers("down", intermediate_size, hidden_size)

    @property
    def gated(self) -> bool:
        return self.activation == "swiglu"

    def _register_quant_buffers(self, name: str, K: int, N: int) -> None:
        G = K // self.group_size
        self.register_buffer(f"{name}_qweight", torch.zeros(K, N // 8, dtype=torch.int32))
        self.register_buffer(f"{name}_scales", torch.zeros(G, N, dtype=torch.float16))
        self.register_buffer(f"{name}_zeros", torch.zeros(G, N // 8, dtype=torch.int32))
        setattr(self, f"{name}_N", N)

    def quant_tensors(self):
        """``(qweights[3], scales[3], zeros[3])`` in gate/up/down order (None if absent)."""
        q, s, z = [], [], []
        for m in _MATS:
            if m == "gate" and not self.gated:
                q.append(None), s.append(None), z.append(None)
                continue
            q.append(getattr(self, f"{m}_qweight"))
            s.append(getattr(self, f"{m}_scales"))
            z.append(getattr(self, f"{m}_zeros"))
        return q, s, z

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        """(num_tokens, hidden) -> (num_tokens, hidden)."""
        if not self.quantized:
            if self.gated:
                return self.down_proj(F.silu(self.gate_proj(x)) * self.up_proj(x))
            return self.down_proj(F.silu(self.up_proj(x)))
        q, s, z = self.quant_tensors()
        table = _module_table(self._tables, q, s, z, 1, self.hidden_size,
                              self.intermediate_size, self.group_size, self.gated)
        x = x.half().contiguous()
        M = x.shape[0]
        if M == 0:
            return torch.empty(0, self.hidden_size, dtype=torch.float16, device=x.device)
        if self.gated:
            h = grouped_w4a16(table, 1, FFN_MODE_SWIGLU, 0, x, self.intermediate_size,
                              None, None, M)
        else:
            h = grouped_w4a16(table, 1, FFN_MODE_SILU, 1, x, self.intermediate_size,
                              None, None, M)
        return grouped_w4a16(table, 1, FFN_MODE_PLAIN, 2, h, self.hidden_size, None, None, M)


class ExpertGroup(nn.Module):
    """``num_experts`` independent expert FFNs evaluated as grouped GEMMs."""

    def __init__(self, num_experts: int, hidden_size: int, intermediate_size: int,
                 quantized: bool = False, group_size: int = 128, activation: str = "swiglu"):
        super().__init__()
        self.num_experts = num_experts
        self.hidden_size = hidden_size
        self.intermediate_size = intermediate_size
        self.quantized = quantized
        self.group_size = group_size
        self.activation = activation
        self._tables: dict = {}
        self.experts = nn.ModuleList([
            ExpertFFN(hidden_size, intermediate_size, quantized, group_size, activation)
            for _ in range(num_experts)
        ])

    def _buffer_objects(self, first: int, count: int) -> tuple:
        # the experts' registered buffers, read from the modules' buffer dicts
        # (plain dict iteration: this runs on every forward)
        mods = self.experts._modules
        return tuple(b for e in range(first, first + count)
                     for b in mods[str(e)]._buffers.values())

    def table(self, first: int = 0, count: int | None = None) -> WeightTable:
        count = self.num_experts - first if count is None else count
        hit = self._tables.get((first, count))
        objs = self._buffer_objects(first, count)
        # The table holds the buffers' addresses.  ``.to()`` / ``.cuda()`` or
        # reassigning a buffer creates new tensor objects; loading a state dict
        # copies in place and keeps the addresses.  So the table is reused while
        # the buffer objects (and the first one's address) are unchanged.
        if hit is not None and len(hit[0]) == len(objs) and \
                all(a is b for a, b in zip(hit[0], objs)) and hit[1] == _first_ptr(objs):
            return hit[2]
        q, s, z = [], [], []
        for e in range(first, first + count):
            qe, se, ze = self.experts[e].quant_tensors()
            q += qe
            s += se
            z += ze
        wt = weight_table(q, s, z, count, self.hidden_size, self.intermediate_size,
                          self.group_size, self.activation == "swiglu", cache=False)
        self._tables[(first, count)] = (objs, _first_ptr(objs), wt)
        return wt

    def forward_segments(self, x: torch.Tensor, seg_start: torch.Tensor, seg_len: torch.Tensor,
                         max_rows: int, first_expert: int = 0,
                         num_local: int | None = None, mark=None,
                         out: torch.Tensor | None = None) -> torch.Tensor:
        """Rows ``[seg_start[e], seg_start[e] + seg_len[e])`` of ``x`` through expert
        ``first_expert + e``; other rows of the result (``out`` if given, with as many
        rows as ``x``) are left unwritten."""
        if not self.quantized:
            raise RuntimeError("forward_segments requires quantized experts")
        n = self.num_experts - first_expert if num_local is None else num_local
        table = self.table(first_expert, n)
        x = x.half().contiguous()
        R = x.shape[0]
        h = torch.empty(R, self.intermediate_size, dtype=torch.float16, device=x.device)
        if self.activation == "swiglu":
            grouped_w4a16(table, n, FFN_MODE_SWIGLU, 0, x, self.intermediate_size, seg_start,
                          seg_len, max_rows, out=h)
        else:
            grouped_w4a16(table, n, FFN_MODE_SILU, 1, x, self.intermediate_size, seg_start,
                          seg_len, max_rows, out=h)
        if mark is not None:
            mark("ffn_in")
        y = torch.empty(R, self.hidden_size, dtype=torch.float16, device=x.device) \
            if out is None else out
        grouped_w4a16(table, n, FFN_MODE_PLAIN, 2, h, self.hidden_size, seg_start, seg_len,
                      max_rows, out=y)
        if mark is not None:
            mark("ffn_out")
        return y

    def forward(self, permuted_tokens: torch.Tensor, expert_offsets: torch.Tensor) -> torch.Tensor:
        """Run each expert on its contiguous slice ``[offsets[e], offsets[e+1])``."""
        R = permuted_tokens.shape[0]
        if not self.quantized:
            out = torch.empty_like(permuted_tokens)
            offs = expert_offsets.tolist()
            for e, ex in enumerate(self.experts):
                if offs[e + 1] > offs[e]:
                    out[offs[e]:offs[e + 1]] = ex(permuted_tokens[offs[e]:offs[e + 1]])
            return out
        offs = expert_offsets.to(torch.int32)
        seg_start = offs[:-1].contiguous()
        seg_len = (offs[1:] - offs[:-1]).contiguous()
        return self.forward_segments(permuted_tokens, seg_start, seg_len, max(R, 1))
