"""The arithmetic contract of the 8-bit decode GEMM, checked on CPU in numpy.

Token rows enter as two signed 8-bit terms per 128-k block,
x ~ sigma * (a1 + a2 / 256) with sigma = max|x| / 127, and the packed INT4 codes
as unsigned bytes; each block's int32 accumulators are folded as
y += (sigma / 256) * s * (256 * A1 + A2 - z * X) with X = sum(256 * a1 + a2).
These tests restate that arithmetic (fp32 where the kernel uses fp32) and check:
the reconstruction bound (sigma / 512, or sigma / 256 where the second term
saturates at +-127 because the residual sits at +-sigma / 2), that the fold
equals sum x~ * s * (q - z) exactly, and that the result stays within the layer tolerance of the reference's
dequant-then-matmul (pack_weights.py: w = fp16(scale * (q - zero)))."""

from __future__ import annotations

import numpy as np
import pytest

QK = 128


def terms(x: np.ndarray):
    """(a1, a2, sig_over_256, X) per row and 128-k block, as the token-term pass computes."""
    R, K = x.shape
    xb = x.astype(np.float32).reshape(R, K // QK, QK)
    m = np.abs(xb).max(axis=2).astype(np.float32)
    sigma = (m / np.float32(127)).astype(np.float32)
    with np.errstate(divide="ignore"):
        inv = np.where(m > 0, np.float32(127) / m, np.float32(0)).astype(np.float32)
    q1 = np.clip(np.rint(xb * inv[..., None]), -127, 127).astype(np.float32)
    # fmaf(-q1, sigma, x): one rounding of the exact value, which float64 holds
    rr = (xb.astype(np.float64) - q1.astype(np.float64) * sigma[..., None].astype(np.float64)
          ).astype(np.float32)
    q2 = np.clip(np.rint(rr * inv[..., None] * np.float32(256)), -127, 127).astype(np.float32)
    a1, a2 = q1.astype(np.int64), q2.astype(np.int64)
    X = (256 * a1 + a2).sum(axis=2)
    return a1, a2, (sigma * np.float32(1 / 256)).astype(np.float32), X, sigma, rr


@pytest.mark.parametrize("seed,scale", [(0, 1.0), (1, 300.0), (2, 1e-3)])
def test_reconstruction_bound(seed, scale):
    rng = np.random.default_rng(seed)
    x = (rng.standard_normal((16, 512)) * scale).astype(np.float16)
    x[3] = 0
    x[5, ::7] = 0
    a1, a2, sig256, X, sigma, rr = terms(x)
    assert np.abs(a1).max() <= 127 and np.abs(a2).max() <= 127
    rec = sigma[..., None].astype(np.float64) * (a1 + a2 / 256.0)
    err = np.abs(rec - x.astype(np.float64).reshape(rec.shape))
    sg = sigma[..., None].astype(np.float64)
    # sigma / 256 plus the fp32 rounding of x / sigma at a residual of exactly +-sigma / 2
    assert (err <= sg / 256 * (1 + 1e-3) + 1e-30).all()
    saturated = np.abs(256 * rr.astype(np.float64)) > 127.5 * sg * (1 - 1e-5)
    assert saturated.mean() < 0.01
    ok = ~saturated
    assert (err[ok] <= sg.repeat(err.shape[-1], -1)[ok] / 512 * (1 + 1e-5) + 1e-30).all()
    assert (X == (256 * a1 + a2).sum(axis=2)).all()
    assert np.array_equal(a1[3], np.zeros_like(a1[3])) and np.array_equal(a2[3], a1[3])


@pytest.mark.parametrize("K,N,g", [(512, 256, 128), (1024, 384, 256)])
def test_fold_equals_terms_times_dequant_and_meets_tolerance(K, N, g):
    rng = np.random.default_rng(K + N)
    R = 20
    x = rng.standard_normal((R, K)).astype(np.float16)
    q = rng.integers(0, 16, (K, N))
    z = rng.integers(0, 16, (K // g, N))
    s = (rng.random((K // g, N)) * 0.01 + 1e-3).astype(np.float16)
    a1, a2, sig256, X, sigma, _ = terms(x)
    y = np.zeros((R, N))
    for j in range(K // QK):
        grp = j * QK // g
        qb = q[j * QK:(j + 1) * QK]
        A1 = a1[:, j] @ qb            # exact int
        A2 = a2[:, j] @ qb
        v = 256 * A1 + A2 - z[grp][None, :] * X[:, j][:, None]
        assert np.abs(v).max() < 2**31   # fits the int32 the kernel uses
        y += sig256[:, j][:, None].astype(np.float64) * s[grp].astype(np.float64)[None, :] * v
    # the fold is sum_k x~ * s * (q - z) with x~ the two-term value
    xt = (sigma[..., None].astype(np.float64) * (a1 + a2 / 256.0)).reshape(R, K)
    w_exact = s.astype(np.float64).repeat(g, 0) * (q - z.repeat(g, 0))
    assert np.allclose(y, xt @ w_exact, rtol=1e-12, atol=1e-12)
    # and within the layer bar of the reference's fp16-rounded dequant-then-matmul
    w_ref = (s.astype(np.float32).repeat(g, 0) * (q - z.repeat(g, 0)).astype(np.float32)) \
        .astype(np.float16).astype(np.float64)
    ref = x.astype(np.float64) @ w_ref
    rel = np.linalg.norm(y - ref) / np.linalg.norm(ref)
    assert rel <= 1e-3, rel
    assert np.abs(y - ref).max() <= 2e-2 * np.abs(ref).max()


def test_unpacked_byte_order_and_its_inverse():
    """Two packed words (16 features of one k) unpacked as the weight-operand
    warps do -- low nibbles of word 0, its high nibbles, then word 1 -- put
    feature chunk_feature(b) at byte b; the epilogue maps TMEM lane b back
    with that function (pack_weights.py: nibble i of word j is column 8j+i)."""
    import torch
    import lightning_router.quantization.pack_weights as pw

    rng = np.random.default_rng(7)
    q = torch.from_numpy(rng.integers(0, 16, (3, 64)).astype(np.int32))
    words = pw._pack_int4(q).numpy().view(np.uint32)          # [3, 8]

    def unpack(w):
        out = []
        for v in (w & 0x0F0F0F0F, (w >> 4) & 0x0F0F0F0F):
            out += [(int(v) >> (8 * i)) & 0xFF for i in range(4)]
        return out

    def chunk_feature(b):
        return (b & 8) | ((b & 3) << 1) | ((b >> 2) & 1)

    assert sorted(chunk_feature(b) for b in range(16)) == list(range(16))
    assert [chunk_feature(b) for b in range(16)] == [0, 2, 4, 6, 1, 3, 5, 7,
                                                     8, 10, 12, 14, 9, 11, 13, 15]
    for k in range(3):
        for c in range(4):                                     # 16-feature chunks
            got = unpack(words[k, 2 * c]) + unpack(words[k, 2 * c + 1])
            for b in range(16):
                assert got[b] == int(q[k, 16 * c + chunk_feature(b)])
