"""Loader for the compiled sm_100a library and its torch custom ops.

``ops()`` returns ``torch.ops.lightning_router`` after loading
``_lib/_lr_torch_ops.so``; ``clib()`` returns a ``ctypes`` handle on the C ABI
library ``_lib/liblr_kernels.so`` (the functions declared in
``include/lightning_router.h``).  There is no fallback: a missing library or a
missing CUDA device raises.
"""

from __future__ import annotations

import ctypes
import functools
from pathlib import Path

import torch

LIB_DIR = Path(__file__).resolve().parent / "_lib"
KERNEL_LIB = LIB_DIR / "liblr_kernels.so"
OPS_LIB = LIB_DIR / "_lr_torch_ops.so"

# every symbol the C ABI header declares (checked by the CPU test-suite)
C_ABI_SYMBOLS = (
    "lr_status_string", "lr_abi_version", "lr_last_cuda_error",
    "lr_gate_logits",
    "lr_route_workspace_bytes", "lr_topk_gating_dispatch", "lr_topk_gating_dispatch_noalloc",
    "lr_gate_dispatch_workspace_bytes", "lr_gate_topk_gating_dispatch",
    "lr_topk_route", "lr_permute_tokens",
    "lr_dispatch_workspace_bytes", "lr_expert_routing_forward",
    "lr_combine", "lr_gather_workspace_bytes", "lr_expert_routing_gather",
    "lr_weight_table_bytes", "lr_encode_weight_table",
    "lr_grouped_gemm_workspace_bytes", "lr_grouped_w4a16_workspace_bytes",
    "lr_grouped_w4a16_gemm", "lr_quantized_matmul",
    "lr_ep_plan_size", "lr_ep_plan", "lr_ep_plan_tokens", "lr_ep_publish", "lr_ep_plan_wait",
    "lr_ep_signal", "lr_ep_gather", "lr_ep_combine",
    "lr_ipc_export", "lr_ipc_import", "lr_ipc_close",
)

FFN_MODE_PLAIN = 0
FFN_MODE_SILU = 1
FFN_MODE_SWIGLU = 2


class ExtensionMissing(RuntimeError):
    pass


@functools.lru_cache(maxsize=None)
def clib() -> ctypes.CDLL:
    if not KERNEL_LIB.exists():
        raise ExtensionMissing(
            f"{KERNEL_LIB} is missing: build it with "
            "`python llm-serving-kernel-optimization_b200/build.py`")
    lib = ctypes.CDLL(str(KERNEL_LIB))
    lib.lr_status_string.restype = ctypes.c_char_p
    lib.lr_status_string.argtypes = [ctypes.c_int]
    for name in ("lr_route_workspace_bytes", "lr_dispatch_workspace_bytes",
                 "lr_gate_dispatch_workspace_bytes",
                 "lr_gather_workspace_bytes", "lr_weight_table_bytes",
                 "lr_grouped_gemm_workspace_bytes"):
        getattr(lib, name).restype = ctypes.c_size_t
    return lib


@functools.lru_cache(maxsize=None)
def ops():
    if not OPS_LIB.exists():
        raise ExtensionMissing(
            f"{OPS_LIB} is missing: build it with "
            "`python llm-serving-kernel-optimization_b200/build.py`")
    clib()
    torch.ops.load_library(str(OPS_LIB))
    return torch.ops.lightning_router


def require_cuda(*tensors: torch.Tensor) -> None:
    """Raise unless every tensor lives on a CUDA device (there is no CPU path)."""
    for t in tensors:
        if t is not None and not t.is_cuda:
            raise RuntimeError(
                "lightning_router runs on CUDA (sm_100a) tensors only; got a tensor on "
                f"{t.device}")


@functools.lru_cache(maxsize=None)
def error_word(device_index: int) -> torch.Tensor:
    """Per-device int32 word the kernels OR contract violations into.

    Created as a normal tensor even when the first call comes from inside
    ``torch.inference_mode`` (an inference tensor could not be reset in place
    outside it later)."""
    with torch.inference_mode(False):
        return torch.zeros(1, dtype=torch.int32, device=f"cuda:{device_index}")


DEVERR_BITS = {
    0x1: "expert id outside [0, E)",
    0x2: "source token outside [0, T)",
    0x4: "GEMM pipeline wait timed out",
    0x8: "GEMM row segment outside the row range",
    0x10: "another rank's expert-parallel exchange flag did not arrive in time",
}


def check_device_errors(device: torch.device | int | None = None, reset: bool = True) -> None:
    """Synchronise and raise if a kernel flagged a contract violation on `device`."""
    idx = torch.cuda.current_device() if device is None else torch.device(device, ).index \
        if isinstance(device, torch.device) else int(device)
    w = error_word(idx)
    v = int(w.item())
    if reset and v:
        w.zero_()
    if v:
        msgs = [m for b, m in DEVERR_BITS.items() if v & b]
        raise RuntimeError(f"lightning_router device error 0x{v:x}: " + "; ".join(msgs))
