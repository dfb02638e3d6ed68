"""GPU numerics of the tcgen05 W4A16 GEMM against a plain fp32 reference of the
same op: ``A.float() @ dequantize(B).float()`` (the dequantized weights are
bit-exact fp16, so the only differences are accumulation order and the final
fp16 rounding).  Tolerance: relative L2 <= 1e-3 and max-abs <= 2e-2 * max|ref|.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from conftest import golden

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _quant(K, N, g, seed, scale=0.02):
    from lightning_router.quantization.pack_weights import dequantize_tensor, quantize_tensor
    gen = torch.Generator().manual_seed(seed)
    W = (torch.randn(K, N, generator=gen) * scale).half()
    qw, s, z = quantize_tensor(W, g)
    return qw.to(DEV), s.to(DEV), z.to(DEV), dequantize_tensor(qw, s, z, g, N).to(DEV)


def _check(out, ref, rel=1e-3, absf=2e-2):
    out, ref = out.float(), ref.float()
    err = (out - ref).norm() / ref.norm().clamp_min(1e-30)
    mx = (out - ref).abs().max()
    assert torch.isfinite(out).all()
    assert err <= rel, f"rel-L2 {err:.3e}"
    assert mx <= absf * ref.abs().max().clamp_min(1e-30), f"max-abs {mx:.3e}"


def test_reference_output_shape_and_error():
    """Mirrors the reference's tests/test_quantization.py:61-93."""
    from lightning_router.kernels.quantized_matmul import quantized_matmul
    M, K, N = 32, 256, 64
    qw, s, z, Wd = _quant(K, N, 128, 0)
    A = torch.randn(M, K, device=DEV).half()
    C = quantized_matmul(A, qw, s, z, N=N, group_size=128)
    assert C.shape == (M, N)
    ref = A @ Wd
    rel_err = (C - ref).float().norm() / ref.float().norm()
    assert rel_err < 0.2
    _check(C, A.float() @ Wd.float())


@pytest.mark.parametrize("M,K,N,g", [
    (1, 64, 64, 64), (7, 256, 128, 128), (16, 1024, 256, 64), (33, 512, 96, 128),
    (100, 1024, 384, 128), (128, 256, 128, 64), (255, 1024, 4096, 128), (256, 2048, 1408, 64),
    (300, 4096, 512, 128), (1000, 1024, 1024, 128), (4096, 1024, 256, 128),
])
def test_quantized_matmul_shapes(M, K, N, g):
    from lightning_router.kernels.quantized_matmul import quantized_matmul
    qw, s, z, Wd = _quant(K, N, g, M + K + N)
    A = torch.randn(M, K, device=DEV).half()
    C = quantized_matmul(A, qw, s, z, N=N, group_size=g)
    _check(C, A.float() @ Wd.float())


@pytest.mark.parametrize("M,K,N,g", [
    # the reference's own shapes (tests/test_quantization.py:61-93)
    (32, 256, 64, 128), (64, 256, 64, 128),
    # group 32 / K % 64 != 0: the mma.sync kernel (one and several 32-row token tiles)
    (32, 256, 64, 32), (7, 96, 64, 32), (300, 128, 256, 32), (17, 1024, 1408, 32),
    (64, 200, 96, 8 * 5),
    # N % 32 != 0, groups of 8 or 24, K % 8 != 0: CUDA cores
    (7, 96, 48, 32), (100, 256, 48, 128), (64, 40, 64, 8), (5, 72, 32, 24), (9, 36, 24, 12),
])
def test_quantized_matmul_any_packed_shape(M, K, N, g):
    """Every shape the packed format admits (K % g == 0, N % 8 == 0, any M), as the
    reference's masked Triton kernel accepts, against dequantize + fp32 matmul."""
    from lightning_router.kernels.quantized_matmul import quantized_matmul
    qw, s, z, Wd = _quant(K, N, g, 7 * M + K + N + g)
    A = torch.randn(M, K, device=DEV).half()
    C = quantized_matmul(A, qw, s, z, N=N, group_size=g)
    assert C.shape == (M, N)
    _check(C, A.float() @ Wd.float())


@pytest.mark.parametrize("mode", [0, 1, 2])
@pytest.mark.parametrize("d,f,g", [(96, 48, 16), (256, 96, 32), (128, 64, 64)])
def test_grouped_modes_off_tcgen05_shapes(mode, d, f, g):
    """Grouped modes where gate/up and down take different kernels (CUDA cores for
    N = 48, mma.sync for group 16/32), with ragged and empty segments."""
    from lightning_router.kernels.quantized_matmul import grouped_w4a16
    E = 4
    lens = [5, 0, 40, 17]
    table, A, ss, sl, deq, R = _grouped_case(E, d, f, g, lens, mode, seed=300 + d + f + g + mode)
    for mat, (K, N) in ((1, (d, f)), (2, (f, d))):
        if mat == 2 and mode == 2:
            continue  # SwiGLU is a gate/up launch
        X = A if K == d else torch.randn(R, K, device=DEV).half()
        sentinel = torch.full((R, N), 3.0, dtype=torch.float16, device=DEV)
        out = grouped_w4a16(table, E, mode, mat, X, N, ss, sl, max(lens), out=sentinel.clone())
        covered = torch.zeros(R, dtype=torch.bool, device=DEV)
        for e, L in enumerate(lens):
            st = int(ss[e])
            if L == 0:
                continue
            x = X[st:st + L].float()
            if mode == 0:
                ref = x @ deq[e][mat].float()
            elif mode == 1:
                ref = torch.nn.functional.silu(x @ deq[e][mat].float())
            else:
                ref = torch.nn.functional.silu(x @ deq[e][0].float()) * (x @ deq[e][1].float())
            _check(out[st:st + L], ref)
            covered[st:st + L] = True
        assert torch.equal(out[~covered], sentinel[~covered])


@pytest.mark.parametrize("name", ["m1", "m2"])
def test_matches_reference_triton_fixture(name):
    from lightning_router.kernels.quantized_matmul import quantized_matmul
    zz = golden("qmm_interp")
    A = torch.from_numpy(zz[f"{name}_a"]).to(DEV)
    C = quantized_matmul(A, torch.from_numpy(zz[f"{name}_qweight"]).to(DEV),
                         torch.from_numpy(zz[f"{name}_scales"]).to(DEV),
                         torch.from_numpy(zz[f"{name}_zeros"]).to(DEV),
                         N=int(zz[f"{name}_N"]), group_size=int(zz[f"{name}_gs"]))
    ref = zz[f"{name}_c"].astype(np.float32)
    c = C.float().cpu().numpy()
    assert np.linalg.norm(c - ref) / np.linalg.norm(ref) < 2e-3


def _grouped_case(E, d, f, g, lens, mode, seed):
    """Build E experts and row segments; returns (table, A, seg_start, seg_len, deq, R).

    The returned table holds references to the packed weights it points to."""
    from lightning_router.kernels.quantized_matmul import weight_table
    gen = torch.Generator().manual_seed(seed)
    starts, pos = [], 0
    for L in lens:
        starts.append(pos)
        pos += L + int(torch.randint(0, 5, (1,), generator=gen))  # gaps between segments
    R = pos + 3
    A = torch.randn(R, d, generator=gen).half().to(DEV)
    q, s, z, deq = [], [], [], []
    for e in range(E):
        de = {}
        for m, (K, N) in enumerate([(d, f), (d, f), (f, d)]):
            qw, sc, zr, Wd = _quant(K, N, g, seed * 100 + e * 3 + m)
            q.append(qw), s.append(sc), z.append(zr)
            de[m] = Wd
        deq.append(de)
    table = weight_table(q, s, z, E, d, f, g, True)
    ss = torch.tensor(starts, dtype=torch.int32, device=DEV)
    sl = torch.tensor(lens, dtype=torch.int32, device=DEV)
    return table, A, ss, sl, deq, R


@pytest.mark.parametrize("mode", [0, 1, 2])
@pytest.mark.parametrize("lens,maxr", [([0, 1, 100, 300], 300), ([16, 16, 3, 0], 16),
                                       ([20, 7, 31, 12], 32), ([600, 260, 5, 129], 600),
                                       ([64, 0, 33, 50], 64), ([128, 77, 1, 100], 128),
                                       ([128, 256, 385, 0], 385)])
def test_grouped_modes(mode, lens, maxr):
    from lightning_router.kernels.quantized_matmul import grouped_w4a16
    E, d, f, g = 4, 256, 384, 64
    table, A, ss, sl, deq, R = _grouped_case(E, d, f, g, lens, mode, seed=len(lens) + maxr + mode)
    N = f
    sentinel = torch.full((R, N), 7.0, dtype=torch.float16, device=DEV)
    out = grouped_w4a16(table, E, mode, 1, A, N, ss, sl, maxr, out=sentinel.clone())
    covered = torch.zeros(R, dtype=torch.bool, device=DEV)
    for e, L in enumerate(lens):
        st = int(ss[e])
        if L == 0:
            continue
        x = A[st:st + L].float()
        if mode == 0:
            ref = x @ deq[e][1].float()
        elif mode == 1:
            ref = torch.nn.functional.silu(x @ deq[e][1].float())
        else:
            ref = torch.nn.functional.silu(x @ deq[e][0].float()) * (x @ deq[e][1].float())
        _check(out[st:st + L], ref)
        covered[st:st + L] = True
    # rows outside the segments are not written
    assert torch.equal(out[~covered], sentinel[~covered])


@pytest.mark.parametrize("mode", [0, 1, 2])
def test_grouped_wide_tile_long_k(mode):
    """K >= 4096 with segments over 128 rows: the 256x256 tile with one accumulator
    (epilogue and next main loop take turns), ragged rows and a feature tail."""
    from lightning_router.kernels.quantized_matmul import grouped_w4a16
    E, d, f, g = 3, 4096, 320, 64   # every matrix needs K % g == 0 (d_ff = 320 for the down)
    lens = [300, 0, 129]
    table, A, ss, sl, deq, R = _grouped_case(E, d, f, g, lens, mode, seed=41 + mode)
    sentinel = torch.full((R, f), 5.0, dtype=torch.float16, device=DEV)
    out = grouped_w4a16(table, E, mode, 1, A, f, ss, sl, 300, out=sentinel.clone())
    covered = torch.zeros(R, dtype=torch.bool, device=DEV)
    for e, L in enumerate(lens):
        st = int(ss[e])
        if L == 0:
            continue
        x = A[st:st + L].float()
        if mode == 0:
            ref = x @ deq[e][1].float()
        elif mode == 1:
            ref = torch.nn.functional.silu(x @ deq[e][1].float())
        else:
            ref = torch.nn.functional.silu(x @ deq[e][0].float()) * (x @ deq[e][1].float())
        _check(out[st:st + L], ref)
        covered[st:st + L] = True
    assert torch.equal(out[~covered], sentinel[~covered])


def test_grouped_down_projection_long_k():
    """K = d_ff = 14336 (the Mixtral down projection), a few rows per expert."""
    from lightning_router.kernels.quantized_matmul import grouped_w4a16, weight_table
    E, d, f, g = 2, 256, 14336, 128
    q, s, z, deq = [], [], [], []
    for e in range(E):
        for m, (K, N) in enumerate([(d, f), (d, f), (f, d)]):
            if m < 2:
                q.append(None), s.append(None), z.append(None)
                continue
            qw, sc, zr, Wd = _quant(K, N, g, 900 + e)
            q.append(qw), s.append(sc), z.append(zr)
            deq.append(Wd)
    table = weight_table(q, s, z, E, d, f, g, False)
    A = torch.randn(40, f, device=DEV).half()
    ss = torch.tensor([0, 20], dtype=torch.int32, device=DEV)
    sl = torch.tensor([20, 17], dtype=torch.int32, device=DEV)
    out = grouped_w4a16(table, E, 0, 2, A, d, ss, sl, 20)
    _check(out[0:20], A[0:20].float() @ deq[0].float())
    _check(out[20:37], A[20:37].float() @ deq[1].float())


def test_segment_overflow_is_flagged_and_clamped():
    from lightning_router import _ext
    from lightning_router.kernels.quantized_matmul import grouped_w4a16
    E, d, f, g = 2, 128, 128, 64
    table, A, ss, sl, deq, R = _grouped_case(E, d, f, g, [10, 10], 0, seed=1)
    _ext.check_device_errors()
    bad = torch.tensor([0, R - 2], dtype=torch.int32, device=DEV)   # second segment runs past R
    grouped_w4a16(table, E, 0, 1, A, f, bad, sl, 10)
    with pytest.raises(RuntimeError, match="segment"):
        _ext.check_device_errors()


@pytest.mark.parametrize("mode", [0, 2])
@pytest.mark.parametrize("lens,maxr", [([20, 7, 31, 12], 32), ([600, 260, 5, 129], 600)])
def test_grouped_repeat_is_bit_identical(mode, lens, maxr):
    """Back-to-back launches on identical inputs give identical bits (no pipeline races)."""
    from lightning_router.kernels.quantized_matmul import grouped_w4a16
    E, d, f, g = 4, 256, 384, 64
    table, A, ss, sl, deq, R = _grouped_case(E, d, f, g, lens, mode, seed=77 + mode)
    outs = [grouped_w4a16(table, E, mode, 1, A, f, ss, sl, maxr,
                          out=torch.zeros(R, f, dtype=torch.float16, device=DEV))
            for _ in range(8)]
    for o in outs[1:]:
        assert torch.equal(o, outs[0])
    st, L = int(ss[0]), lens[0]
    x = A[st:st + L].float()
    ref = x @ deq[0][1].float() if mode == 0 else \
        torch.nn.functional.silu(x @ deq[0][0].float()) * (x @ deq[0][1].float())
    _check(outs[0][st:st + L], ref)


@pytest.mark.parametrize("mode", [0, 2])
@pytest.mark.parametrize("d,lens", [(256, [20, 7, 31, 12, 1, 30, 0, 25]),
                                    (256, [50, 7, 64, 12, 1, 30, 0, 25]),
                                    (4096, [20, 7, 31, 12, 1, 30, 0, 25]),
                                    (4096, [50, 7, 32, 12, 1, 30, 0, 25])])
def test_expert_rows_independent_of_other_experts(mode, d, lens):
    """An expert's output rows are bit-identical whether it runs alone or among 8
    experts (other tile counts, tile order and SM assignment): every output
    element keeps the same k-ordered UMMA accumulation.  Expert-parallel ranks
    rely on this to match one GPU bit for bit."""
    from lightning_router.kernels.quantized_matmul import grouped_w4a16, weight_table
    E, f, g = 8, 4096 if d == 256 else 512, 64
    q, s, z, deq = [], [], [], []
    for e in range(E):
        for m, (K, N) in enumerate([(d, f), (d, f), (f, d)]):
            qw, sc, zr, Wd = _quant(K, N, g, 500 + e * 3 + m)
            q.append(qw), s.append(sc), z.append(zr)
            if e == 0:
                deq.append(Wd)
    starts = [0]
    for L in lens[:-1]:
        starts.append(starts[-1] + L)
    R = starts[-1] + lens[-1]
    A = torch.randn(R, d, generator=torch.Generator().manual_seed(3)).half().to(DEV)
    ss = torch.tensor(starts, dtype=torch.int32, device=DEV)
    sl = torch.tensor(lens, dtype=torch.int32, device=DEV)
    table8 = weight_table(q, s, z, E, d, f, g, True)
    table1 = weight_table(q[:3], s[:3], z[:3], 1, d, f, g, True)
    L0 = lens[0]
    out8 = grouped_w4a16(table8, E, mode, 1, A, f, ss, sl, max(lens))
    out1 = grouped_w4a16(table1, 1, mode, 1, A, f, ss[:1], sl[:1], L0)
    assert torch.equal(out8[:L0], out1[:L0])
    x = A[:L0].float()
    ref = x @ deq[1].float() if mode == 0 else \
        torch.nn.functional.silu(x @ deq[0].float()) * (x @ deq[1].float())
    _check(out1[:L0], ref)



def _ref_mode(x, de, mode):
    if mode == 0:
        return x @ de[1].float()
    if mode == 1:
        return torch.nn.functional.silu(x @ de[1].float())
    return torch.nn.functional.silu(x @ de[0].float()) * (x @ de[1].float())


@pytest.mark.parametrize("mode", [0, 1, 2])
@pytest.mark.parametrize("d,f,g,lens", [
    (1024, 2048, 128, [20, 0, 32, 7, 1]),
    (4096, 1024, 128, [16, 16, 3, 0]),
    (1024, 1152, 128, [32, 5]),          # 1152 output rows: a partial 256-row weight tile
    (2048, 1024, 256, [31, 1, 12]),      # one group spans two 128-k blocks
])
def test_int8_operand_path(mode, d, f, g, lens):
    """Segments of at most 32 rows with K and the group size multiples of 128 run on
    8-bit operands (token rows as two 8-bit terms per 128-k block, INT4 codes as
    bytes, scale and zero folded per block).  Checked against the fp32 reference
    at the same bar as every GEMM, against the fp16-operand kernel on the same
    inputs, for repeat determinism, and rows outside the segments stay unwritten."""
    from lightning_router.kernels.quantized_matmul import grouped_w4a16
    E = len(lens)
    table, A, ss, sl, deq, R = _grouped_case(E, d, f, g, lens, mode, seed=d + f + g + mode)
    maxr = max(lens)
    sentinel = torch.full((R, f), 3.0, dtype=torch.float16, device=DEV)
    out = grouped_w4a16(table, E, mode, 1, A, f, ss, sl, maxr, out=sentinel.clone())
    again = grouped_w4a16(table, E, mode, 1, A, f, ss, sl, maxr, out=sentinel.clone())
    f16 = grouped_w4a16(table, E, mode, 1, A, f, ss, sl, maxr, int8_operands=False)
    assert torch.equal(out, again)
    covered = torch.zeros(R, dtype=torch.bool, device=DEV)
    for e, L in enumerate(lens):
        st = int(ss[e])
        if L == 0:
            continue
        ref = _ref_mode(A[st:st + L].float(), deq[e], mode)
        _check(out[st:st + L], ref)
        _check(f16[st:st + L], ref)
        _check(out[st:st + L], f16[st:st + L].float())
        covered[st:st + L] = True
    assert torch.equal(out[~covered], sentinel[~covered])


def test_int8_operand_path_rows_independent_of_other_experts():
    """On the 8-bit path an expert's rows are bit-identical alone or among 8 experts:
    each row's terms and its block sums depend on that row only."""
    from lightning_router.kernels.quantized_matmul import grouped_w4a16, weight_table
    E, d, f, g = 8, 1024, 2048, 128
    lens = [20, 7, 31, 12, 1, 30, 0, 25]
    q, s, z, deq = [], [], [], []
    for e in range(E):
        for m, (K, N) in enumerate([(d, f), (d, f), (f, d)]):
            qw, sc, zr, Wd = _quant(K, N, g, 700 + e * 3 + m)
            q.append(qw), s.append(sc), z.append(zr)
            if e == 0:
                deq.append(Wd)
    starts = [0]
    for L in lens[:-1]:
        starts.append(starts[-1] + L)
    R = starts[-1] + lens[-1]
    A = torch.randn(R, d, generator=torch.Generator().manual_seed(5)).half().to(DEV)
    ss = torch.tensor(starts, dtype=torch.int32, device=DEV)
    sl = torch.tensor(lens, dtype=torch.int32, device=DEV)
    table8 = weight_table(q, s, z, E, d, f, g, True)
    table1 = weight_table(q[:3], s[:3], z[:3], 1, d, f, g, True)
    L0 = lens[0]
    for mode in (0, 2):
        out8 = grouped_w4a16(table8, E, mode, 1, A, f, ss, sl, max(lens))
        out1 = grouped_w4a16(table1, 1, mode, 1, A[:L0].contiguous(), f, ss[:1], sl[:1], L0)
        assert torch.equal(out8[:L0], out1[:L0])
        _check(out1[:L0], _ref_mode(A[:L0].float(), deq, mode))


def test_int8_operand_path_large_rows_and_zero_rows():
    """Rows of large magnitude, all-zero rows and rows with a single non-zero entry
    per block keep the bar (the terms scale with each block's maximum)."""
    from lightning_router.kernels.quantized_matmul import grouped_w4a16
    E, d, f, g = 2, 1024, 1024, 128
    lens = [24, 9]
    table, A, ss, sl, deq, R = _grouped_case(E, d, f, g, lens, 0, seed=11)
    A[0:4] *= 200.0
    A[4:6] = 0
    A[6:8] = 0
    A[6:8, ::128] = 1.5
    out = grouped_w4a16(table, E, 0, 1, A, f, ss, sl, max(lens))
    for e, L in enumerate(lens):
        st = int(ss[e])
        _check(out[st:st + L], A[st:st + L].float() @ deq[e][1].float())
    assert torch.equal(out[4:6], torch.zeros_like(out[4:6]))


@pytest.mark.parametrize("mode", [0, 2])
def test_int8_operand_path_one_block_and_many_experts(mode):
    """K = 128 (one 128-deep block per tile for gate/up) with 64 experts of 0-32 rows:
    many tiles per CTA, empty experts between full ones, and a 64-entry tile table."""
    from lightning_router.kernels.quantized_matmul import grouped_w4a16
    E, d, f, g = 64, 128, 256, 128
    gen = torch.Generator().manual_seed(21)
    lens = [int(x) for x in torch.randint(0, 33, (E,), generator=gen)]
    lens[0], lens[5], lens[63] = 32, 0, 1
    table, A, ss, sl, deq, R = _grouped_case(E, d, f, g, lens, mode, seed=31 + mode)
    sentinel = torch.full((R, f), 9.0, dtype=torch.float16, device=DEV)
    out = grouped_w4a16(table, E, mode, 1, A, f, ss, sl, 32, out=sentinel.clone())
    covered = torch.zeros(R, dtype=torch.bool, device=DEV)
    for e, L in enumerate(lens):
        if L == 0:
            continue
        st = int(ss[e])
        _check(out[st:st + L], _ref_mode(A[st:st + L].float(), deq[e], mode))
        covered[st:st + L] = True
    assert torch.equal(out[~covered], sentinel[~covered])
