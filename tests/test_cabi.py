"""CPU checks of the C ABI boundary: the library loads, exports every symbol the
header declares, and its host-only entry points behave (no device calls)."""

from __future__ import annotations

import ctypes
import re
from pathlib import Path

import pytest

from lightning_router import _ext

HEADER = Path(__file__).resolve().parents[1] / "include" / "lightning_router.h"


def declared_symbols() -> set[str]:
    text = HEADER.read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return set(re.findall(r"\b(lr_[a-z0-9_]+)\s*\(", text))


def test_header_and_loader_agree():
    assert declared_symbols() == set(_ext.C_ABI_SYMBOLS)


def test_library_exports_every_declared_symbol():
    lib = _ext.clib()
    for name in sorted(declared_symbols()):
        assert hasattr(lib, name), name


def test_torch_op_library_loads_and_registers_every_op():
    """The torch-op shim loads without a GPU (its op schemas parse at load time)."""
    ops = _ext.ops()
    for name in ("gate_logits", "topk_gating_dispatch", "gate_topk_gating_dispatch",
                 "expert_routing_forward", "combine", "topk_route", "permute_tokens",
                 "expert_routing_gather", "encode_weight_table", "grouped_w4a16_gemm",
                 "route_rows", "ep_plan", "ep_plan_tokens", "ep_gather", "ep_combine",
                 "ep_publish", "ep_plan_wait", "ep_signal"):
        assert hasattr(ops, name), name


def test_status_strings_and_version():
    lib = _ext.clib()
    assert lib.lr_abi_version() == 3
    assert lib.lr_status_string(0) == b"ok"
    assert b"invalid" in lib.lr_status_string(-1)
    assert b"workspace" in lib.lr_status_string(-4)


def test_workspace_queries_are_host_only():
    lib = _ext.clib()
    assert lib.lr_route_workspace_bytes(16384, 2, 8) >= 256 + 2 * 64 * 8 * 4
    assert lib.lr_dispatch_workspace_bytes(1 << 20, 64) > 0
    assert lib.lr_gather_workspace_bytes(1000, 500) >= 4 * (1000 * 2 + 500 * 3)
    assert lib.lr_weight_table_bytes(8) == 8 * lib.lr_weight_table_bytes(1)
    assert lib.lr_weight_table_bytes(1) % 128 == 0
    # gate + dispatch: covers both the one-launch path (T <= 256: ticket, 8 chunk
    # partials of T x E fp32, T x k rows) and the two-kernel path
    small = lib.lr_gate_dispatch_workspace_bytes(64, 2, 8)
    assert small >= 256 + 8 * 64 * 8 * 4 + 64 * 2 * 4
    assert small >= lib.lr_route_workspace_bytes(64, 2, 8)
    assert lib.lr_gate_dispatch_workspace_bytes(4096, 2, 8) == lib.lr_route_workspace_bytes(4096, 2, 8)


def test_int8_operand_workspace_query():
    """The 8-bit GEMM path's workspace: two 8-bit terms per token element plus a
    (sigma, block sum) pair per row and 128-k block; zero for shapes it does not take."""
    lib = _ext.clib()
    f = lib.lr_grouped_w4a16_workspace_bytes
    f.restype = ctypes.c_size_t

    def a128(b):
        return (b + 127) // 128 * 128

    # decode Mixtral-shaped gate/up: R = 128 rows, K = 4096, N = 14336, capacity 20
    assert f(8, 128, 4096, 14336, 128, 20) == a128(2 * 128 * 4096) + 2 * a128(4 * 128 * 32)
    assert f(8, 128, 14336, 4096, 128, 20) == a128(2 * 128 * 14336) + 2 * a128(4 * 128 * 112)
    assert f(1, 5, 256, 64, 256, 5) == a128(2 * 5 * 256) + 2 * a128(4 * 5 * 2)
    for args in [(8, 128, 4096, 14336, 128, 33),   # segments longer than 32 rows
                 (8, 128, 4096, 14336, 64, 20),    # group size not a multiple of 128
                 (8, 128, 4160, 14336, 64, 20),    # K not a multiple of 128
                 (8, 128, 4096, 14344, 128, 20),   # N not a multiple of 32
                 (8, 128, 4096, 14336, 128, 0), (0, 128, 4096, 14336, 128, 20),
                 (8, 0, 4096, 14336, 128, 20), (8, 128, 4096, 14336, 100, 20)]:
        assert f(*args) == 0, args


def test_argument_validation_without_device():
    """Invalid shapes are rejected before any CUDA call."""
    lib = _ext.clib()
    # d not a multiple of 16
    assert lib.lr_gate_logits(None, None, None, 4, 10, 8, None, None) == -1
    # E > 64 for the gating kernel
    assert lib.lr_topk_gating_dispatch(None, None, 4, 64, 65, 2, 8, ctypes.c_float(0.01), 0,
                                       None, None, None, None, None, None, None, None, None,
                                       None, None, ctypes.c_size_t(0), None, None) == -1
    # gate + dispatch: d not a multiple of 16, E > 64, k > E, T = 0
    nulls = [None] * 10  # the ten outputs after the logits
    for T, d, E, k in [(4, 24, 8, 2), (4, 64, 65, 2), (4, 64, 4, 5), (0, 64, 8, 2)]:
        assert lib.lr_gate_topk_gating_dispatch(
            None, None, None, T, d, E, k, 8, ctypes.c_float(0.01), 0, None, *nulls,
            None, ctypes.c_size_t(0), None, None) == -1
    # group size not dividing K, N not a multiple of 8, no operands
    for K, N, g in [(100, 64, 64), (128, 60, 64), (128, 64, 0)]:
        assert lib.lr_grouped_w4a16_gemm(ctypes.c_void_p(128), 1, 0, 2, None, 4, K, N, g, None,
                                         None, 4, None, None, ctypes.c_size_t(0), None,
                                         None) in (-1, -2)
    assert lib.lr_grouped_w4a16_gemm(ctypes.c_void_p(128), 1, 0, 2, None, 4, 96, 48, 32, None,
                                     None, 4, None, None, ctypes.c_size_t(0), None, None) == -1


def test_torch_ops_register():
    ops = _ext.ops()
    for name in ("gate_logits", "topk_gating_dispatch", "gate_topk_gating_dispatch",
                 "expert_routing_forward", "combine", "expert_routing_gather",
                 "encode_weight_table", "grouped_w4a16_gemm"):
        assert hasattr(ops, name), name


def test_cpu_tensors_fail_loudly():
    import torch
    from lightning_router.models.gating import TopKGating
    gate = TopKGating(64, 4, 2)
    with pytest.raises(RuntimeError, match="CUDA"):
        gate(torch.randn(3, 64))



@pytest.mark.gpu
def test_error_word_created_in_inference_mode_resets_outside():
    """The cached device error word stays resettable outside inference mode even
    when the first kernel call that needed it ran inside inference mode."""
    import torch
    _ext.error_word.cache_clear()
    with torch.inference_mode():
        w = _ext.error_word(0)
    assert not w.is_inference()
    w.fill_(0x8)
    with pytest.raises(RuntimeError, match="segment"):
        _ext.check_device_errors(0)
    assert int(w.item()) == 0
