"""The allocation-free gating + dispatch entry point, called through the C ABI.

``lr_topk_gating_dispatch_noalloc`` serves callers that cannot allocate device
memory (a host that hands the library pre-sized buffers but no allocator, or a
loop where a synchronising cudaMalloc is not allowed).  Its scratch is a fixed
1 MiB device array inside the library.  This test calls it twice in a row on
the same inputs and checks each result against the workspace-taking entry point
``lr_topk_gating_dispatch`` (reached through its torch op): integer outputs and
rows bit-exact, gate weights within 1e-6 relative, aux loss within 1e-5.
It lives in its own file so a run that stops at the first failure has already
run every other test.
"""

from __future__ import annotations

import ctypes

import pytest
import torch

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _p(t):
    return ctypes.c_void_p(t.data_ptr())


def _noalloc(lib, x, logits, k, C, lbw=0.01, fill=1):
    T, E = logits.shape
    d = x.shape[1]
    S = T * k
    i32 = dict(dtype=torch.int32, device=DEV)
    f32 = dict(dtype=torch.float32, device=DEV)
    out = {
        "ids": torch.full((S,), -7, **i32), "w": torch.full((S,), -7.0, **f32),
        "tok": torch.full((S,), -7, **i32), "offsets": torch.full((E + 1,), -7, **i32),
        "kept": torch.full((E,), -7, **i32), "aux": torch.full((1,), -7.0, **f32),
        "perm": torch.full((S, d), 3.0, dtype=torch.float16, device=DEV),
        "rw": torch.full((S,), -7.0, **f32), "src": torch.full((S,), -7, **i32),
        "pos": torch.full((S,), -7, **i32), "err": torch.zeros(1, **i32),
    }
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    rc = lib.lr_topk_gating_dispatch_noalloc(
        _p(x), _p(logits), T, d, E, k, C, ctypes.c_float(lbw), fill,
        _p(out["ids"]), _p(out["w"]), _p(out["tok"]), _p(out["offsets"]), _p(out["kept"]),
        _p(out["aux"]), _p(out["perm"]), _p(out["rw"]), _p(out["src"]), _p(out["pos"]),
        _p(out["err"]), stream)
    return rc, out


@pytest.mark.parametrize("T,d,E,k,cf", [(1000, 256, 8, 2, 1.0), (513, 128, 64, 6, 1.5),
                                        (4099, 64, 16, 4, 0.75)])
def test_noalloc_matches_workspace_entry_point(T, d, E, k, cf):
    from lightning_router import _ext
    from lightning_router.kernels.expert_routing import topk_gating_dispatch
    lib = _ext.clib()
    g = torch.Generator().manual_seed(T + E)
    x = torch.randn(T, d, generator=g).half().to(DEV)
    logits = (torch.randn(T, E, generator=g) + torch.linspace(1.5, -1.5, E)).to(DEV)
    ref = topk_gating_dispatch(x, logits, k, cf, fill_dropped=True)
    for _call in range(2):
        rc, out = _noalloc(lib, x, logits, k, ref.capacity)
        assert rc == 0, lib.lr_status_string(rc)
        torch.cuda.synchronize()
        assert int(out["err"]) == 0
        assert torch.equal(out["ids"], ref.expert_ids)
        assert torch.equal(out["tok"], ref.token_indices)
        assert torch.equal(out["offsets"], ref.offsets)
        assert torch.equal(out["kept"], ref.kept_counts)
        assert torch.equal(out["pos"], ref.slot_pos)
        assert torch.equal(out["src"], ref.source_indices)
        assert torch.equal(out["perm"], ref.permuted)
        torch.testing.assert_close(out["w"], ref.gate_weights, rtol=1e-6, atol=1e-12)
        torch.testing.assert_close(out["rw"], ref.routing_weights, rtol=1e-6, atol=1e-12)
        torch.testing.assert_close(out["aux"][0], ref.aux_loss, rtol=1e-5, atol=0)


def test_noalloc_rejects_sizes_beyond_its_scratch():
    from lightning_router import _ext
    lib = _ext.clib()
    x = torch.zeros(8, 64, dtype=torch.float16, device=DEV)
    logits = torch.zeros(8, 64, device=DEV)
    # 1 << 20 tokens at E = 64 needs ~4 MiB of route scratch: rejected before any work
    T = 1 << 20
    S = T * 2
    i32 = dict(dtype=torch.int32, device=DEV)
    dummy = torch.zeros(16, **i32)
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    rc = lib.lr_topk_gating_dispatch_noalloc(
        _p(x), _p(logits), T, 64, 64, 2, S // 64, ctypes.c_float(0.01), 0,
        *([_p(dummy)] * 6), _p(x), *([_p(dummy)] * 3), _p(dummy), stream)
    assert rc == -6
    assert b"1 MiB" in lib.lr_status_string(rc)
