"""Few-row Q8_0 GEMM on the integer tensor cores (tcgen05 kind::i8) on a
B200, through the C ABI (vrt_q8t_to_q8m, vrt_q8m_gemm, vrt_q8m_gemm_gelu).

The activation rows are quantised per 32-block to int16 (the mat-vec's
activation format) and every Q8_0 block is an exact int32 MMA, so each output
row is held to the north-star bound (atol 1e-3, rtol 1e-3) against an fp64
dequantised product and to 2e-4 of the row RMS; replays are bit-identical,
and rows agree with the oracle's mat-vec."""

import numpy as np
import pytest

import oracle as O
import synth_gguf as sg
import vrt

pytestmark = pytest.mark.gpu
ATOL, RTOL = 1e-3, 1e-3


def dequant(raw: np.ndarray, rows: int, cols: int) -> np.ndarray:
    b = raw.reshape(rows, cols // 32, 34)
    scale = b[:, :, :2].copy().view(np.float16).astype(np.float64)
    q = b[:, :, 2:].view(np.int8).astype(np.float64)
    return (q * scale).reshape(rows, cols)


def check(y, ref):
    err = np.abs(y.astype(np.float64) - ref)
    bound = ATOL + RTOL * np.abs(ref)
    assert np.all(err <= bound), f"max err {err.max():.3g}, worst ratio {(err / bound).max():.3g}"
    # int16 activations: rounding error ~ amax / 32512 / sqrt(12) ~ 2e-5 of the
    # block's spread per element, ~9e-5 of the row RMS at the maximum over
    # ~10^5 outputs (the mat-vec's activation format has the same bound)
    scale = np.sqrt(np.mean(ref ** 2, axis=-1, keepdims=True)) + 1e-30
    assert (err / scale).max() < 2e-4, f"relative to row RMS {(err / scale).max():.3g}"


def q8m(ctx, raw, rows, cols, pair_split=None):
    w = ctx.upload(raw)
    n = vrt.lib().vrt_q8t_bytes(rows, cols)
    pk = ctx.alloc(n)
    if pair_split is None:
        vrt.check(vrt.lib().vrt_q8t_pack(ctx.h, w, raw.nbytes, 0, rows, cols, pk, None))
    else:
        vrt.check(vrt.lib().vrt_q8t_pack_pair(ctx.h, w, raw.nbytes, 0, pair_split, rows // 2, cols, pk, None))
    out = ctx.alloc(n)
    vrt.check(vrt.lib().vrt_q8t_to_q8m(ctx.h, pk, rows, cols, out, None))
    return out


@pytest.mark.parametrize("rows,cols,m", [(1536, 640, 1), (1536, 640, 16), (640, 1024, 17), (640, 2048, 32),
                                         (8192, 5376, 32), (5376, 21504, 24), (43008, 5376, 7)])
def test_q8m_gemm_vs_fp64(ctx, rows, cols, m):
    raw = sg.q8_matrix_bytes(7, f"gemm.{rows}x{cols}", rows, cols)
    x = np.random.default_rng(rows + m).standard_normal((m, cols)).astype(np.float32)
    ref = x.astype(np.float64) @ dequant(raw, rows, cols).T
    w = q8m(ctx, raw, rows, cols)
    dx, dy = ctx.upload(x), ctx.alloc(4 * m * rows)
    vrt.check(vrt.lib().vrt_q8m_gemm(ctx.h, w, rows, cols, dx, m, dy, None))
    y = ctx.download(dy, m * rows).reshape(m, rows)
    check(y, ref)
    vrt.check(vrt.lib().vrt_q8m_gemm(ctx.h, w, rows, cols, dx, m, dy, None))
    assert np.array_equal(ctx.download(dy, m * rows).reshape(m, rows), y)


def test_q8m_gemm_rows_match_gemv(ctx):
    rows, cols, m = 2048, 640, 5
    raw = sg.q8_matrix_bytes(7, "gemm.gemv", rows, cols)
    x = np.random.default_rng(5).standard_normal((m, cols)).astype(np.float32)
    w = q8m(ctx, raw, rows, cols)
    dx, dy = ctx.upload(x), ctx.alloc(4 * m * rows)
    vrt.check(vrt.lib().vrt_q8m_gemm(ctx.h, w, rows, cols, dx, m, dy, None))
    y = ctx.download(dy, m * rows).reshape(m, rows)
    for i in range(m):
        ref = O.q8_matvec(raw, x[i], rows, lanes=0)
        assert np.all(np.abs(y[i].astype(np.float64) - ref) <= ATOL + RTOL * np.abs(ref))


@pytest.mark.parametrize("ff,d,m", [(2048, 640, 32), (768, 128, 3)])
def test_q8m_gate_up_gelu(ctx, ff, d, m):
    g = sg.q8_matrix_bytes(9, "gemm.gate", ff, d)
    u = sg.q8_matrix_bytes(9, "gemm.up", ff, d)
    raw = np.concatenate([g, u])
    x = np.random.default_rng(ff).standard_normal((m, d)).astype(np.float32)
    xg = x.astype(np.float64) @ dequant(g, ff, d).T
    xu = x.astype(np.float64) @ dequant(u, ff, d).T
    c = np.sqrt(2.0 / np.pi)
    ref = 0.5 * xg * (1.0 + np.tanh(c * (xg + 0.044715 * xg ** 3))) * xu
    w = q8m(ctx, raw, 2 * ff, d, pair_split=g.nbytes)
    dx, da = ctx.upload(x), ctx.alloc(4 * m * ff)
    vrt.check(vrt.lib().vrt_q8m_gemm_gelu(ctx.h, w, ff, d, dx, m, da, None))
    act = ctx.download(da, m * ff).reshape(m, ff)
    err = np.abs(act.astype(np.float64) - ref)
    assert np.all(err <= ATOL + RTOL * np.abs(ref)), f"max err {err.max():.3g}"


def test_q8m_rejects_bad_shapes(ctx):
    with pytest.raises(vrt.VrtError):
        vrt.check(vrt.lib().vrt_q8m_gemm(ctx.h, None, 128, 128, None, 1, None, None))
    raw = sg.q8_matrix_bytes(7, "gemm.bad", 256, 256)
    w = q8m(ctx, raw, 256, 256)
    dx, dy = ctx.upload(np.zeros((40, 256), np.float32)), ctx.alloc(4 * 40 * 256)
    with pytest.raises(vrt.VrtError, match="m <= 32"):
        vrt.check(vrt.lib().vrt_q8m_gemm(ctx.h, w, 256, 256, dx, 40, dy, None))
