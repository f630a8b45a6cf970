"""Tensor-core (tcgen05) Q8_0 GEMM on a B200, through the C ABI.

The reference runs prompt tokens one at a time through its Q8_0 mat-vec; the
batched paths here use a GEMM whose rows are those same mat-vecs, so every
output row is held to the north-star bound (atol 1e-3, rtol 1e-3) against an
fp64 dequantised product, and — because the hi/lo operand split is meant to be
near-exact — to a 1e-4 bound relative to the row RMS (a single fp16 product
would reach ~1e-3 there; the split measures ~1e-5, set by the tensor core's
fp32 accumulation).  Replays are
bit-identical.
"""

import numpy as np
import pytest

import oracle as O
import synth_gguf as sg
import vrt

pytestmark = pytest.mark.gpu
ATOL, RTOL = 1e-3, 1e-3


def dequant(raw: np.ndarray, rows: int, cols: int) -> np.ndarray:
    """Q8_0 rows (34-byte blocks: fp16 scale + 32 int8) -> fp64 [rows][cols]."""
    b = raw.reshape(rows, cols // 32, 34)
    scale = b[:, :, :2].copy().view(np.float16).astype(np.float64)
    q = b[:, :, 2:].view(np.int8).astype(np.float64)
    return (q * scale).reshape(rows, cols)


def check(y, ref):
    err = np.abs(y.astype(np.float64) - ref)
    bound = ATOL + RTOL * np.abs(ref)
    assert np.all(err <= bound), f"max err {err.max():.3g}, worst ratio {(err / bound).max():.3g}"
    scale = np.sqrt(np.mean(ref ** 2, axis=-1, keepdims=True)) + 1e-30
    assert (err / scale).max() < 1e-4, f"hi/lo split error {(err / scale).max():.3g}"


def packed(ctx, raw, rows, cols):
    w = ctx.upload(raw)
    pk = ctx.alloc(vrt.lib().vrt_q8t_bytes(rows, cols))
    vrt.check(vrt.lib().vrt_q8t_pack(ctx.h, w, raw.nbytes, 0, rows, cols, pk, None))
    return pk


@pytest.mark.parametrize("rows,cols,m", [(1536, 640, 1), (1536, 640, 77), (640, 1024, 128), (640, 2048, 300),
                                         (2048, 640, 129), (8192, 5376, 40), (5376, 21504, 24)])
def test_gemm_vs_fp64(ctx, rows, cols, m):
    raw = sg.q8_matrix_bytes(7, f"gemm.{rows}x{cols}", rows, cols)
    x = np.random.default_rng(rows + m).standard_normal((m, cols)).astype(np.float32)
    ref = x.astype(np.float64) @ dequant(raw, rows, cols).T
    pk = packed(ctx, raw, rows, cols)
    dx, dy = ctx.upload(x), ctx.alloc(4 * m * rows)
    vrt.check(vrt.lib().vrt_q8t_gemm(ctx.h, pk, rows, cols, dx, m, dy, None))
    y = ctx.download(dy, m * rows).reshape(m, rows)
    check(y, ref)
    vrt.check(vrt.lib().vrt_q8t_gemm(ctx.h, pk, rows, cols, dx, m, dy, None))
    assert np.array_equal(ctx.download(dy, m * rows).reshape(m, rows), y)


def test_gemm_rows_match_gemv(ctx):
    rows, cols, m = 2048, 640, 5
    raw = sg.q8_matrix_bytes(7, "gemm.gemv", rows, cols)
    x = np.random.default_rng(5).standard_normal((m, cols)).astype(np.float32)
    pk = packed(ctx, raw, rows, cols)
    dx, dy = ctx.upload(x), ctx.alloc(4 * m * rows)
    vrt.check(vrt.lib().vrt_q8t_gemm(ctx.h, pk, rows, cols, dx, m, dy, None))
    y = ctx.download(dy, m * rows).reshape(m, rows)
    for i in range(m):
        ref = O.q8_matvec(raw, x[i], rows, lanes=0)   # the oracle's fp64 mat-vec
        err = np.abs(y[i].astype(np.float64) - ref)
        assert np.all(err <= ATOL + RTOL * np.abs(ref))


@pytest.mark.parametrize("ff,d,m", [(2048, 640, 100), (768, 128, 3)])
def test_gemm_gate_up_gelu(ctx, ff, d, m):
    g = sg.q8_matrix_bytes(9, "gemm.gate", ff, d)
    u = sg.q8_matrix_bytes(9, "gemm.up", ff, d)
    raw = np.concatenate([g, u])
    x = np.random.default_rng(ff).standard_normal((m, d)).astype(np.float32)
    xg = x.astype(np.float64) @ dequant(g, ff, d).T
    xu = x.astype(np.float64) @ dequant(u, ff, d).T
    c = np.sqrt(2.0 / np.pi)
    ref = 0.5 * xg * (1.0 + np.tanh(c * (xg + 0.044715 * xg ** 3))) * xu
    w = ctx.upload(raw)
    pair = ctx.alloc(vrt.lib().vrt_q8t_bytes(2 * ff, d))
    vrt.check(vrt.lib().vrt_q8t_pack_pair(ctx.h, w, raw.nbytes, 0, g.nbytes, ff, d, pair, None))
    dx, da = ctx.upload(x), ctx.alloc(4 * m * ff)
    vrt.check(vrt.lib().vrt_q8t_gemm_gelu(ctx.h, pair, ff, d, dx, m, da, None))
    act = ctx.download(da, m * ff).reshape(m, ff)
    err = np.abs(act.astype(np.float64) - ref)
    assert np.all(err <= ATOL + RTOL * np.abs(ref)), f"max err {err.max():.3g}"


def test_gemm_rejects_bad_shapes(ctx):
    L = vrt.lib()
    dx, dy, w = ctx.alloc(4 * 640), ctx.alloc(4 * 1000), ctx.alloc(1 << 20)
    assert L.vrt_q8t_gemm(ctx.h, w, 100, 640, dx, 1, dy, None) == vrt.VRT_E_INVALID   # rows % 128
    assert L.vrt_q8t_gemm(ctx.h, w, 128, 96, dx, 1, dy, None) == vrt.VRT_E_INVALID    # cols % 128
    assert L.vrt_q8t_gemm(ctx.h, w, 128, 640, dx, 0, dy, None) == vrt.VRT_E_INVALID   # m == 0
