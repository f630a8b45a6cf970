"""Kernel parity on a B200, through the C ABI of libvortexrt_b200.so.

Tolerances: the reference tests' own (2e-3 for the Q8 mat-vec KAT, 5e-3 for
the FFN KAT, 5e-5 for gelu), and the north-star bound atol 1e-3 / rtol 1e-3
against the CPU oracle for the benchmark shapes.  Replays must be bit-equal.
"""

import ctypes as C

import numpy as np
import pytest

import kat
import oracle as O
import synth_gguf as sg
import vrt

pytestmark = pytest.mark.gpu
ATOL, RTOL = 1e-3, 1e-3


def _close(y, ref, atol=ATOL, rtol=RTOL):
    err = np.abs(y.astype(np.float64) - ref.astype(np.float64))
    bound = atol + rtol * np.abs(ref.astype(np.float64))
    assert np.all(err <= bound), f"max err {err.max():.3g}, worst ratio {(err / bound).max():.3g}"


def _argmax_dev(ctx, res_ptr):
    r = ctx.download(res_ptr, 2, np.uint32)
    return int(r[0]), float(r[1:2].view(np.float32)[0])


def test_context_and_device(ctx):
    info = ctx.info()
    assert info.cc_major >= 10
    assert info.sm_count >= 100
    assert info.warp_size == 32


def test_q8_gemv_known_answer(ctx):
    raw, x, ref, n_in, n_out = kat.q8_test_case()
    w = ctx.upload(raw)
    dx = ctx.upload(x)
    dy = ctx.alloc(4 * n_out)
    vrt.check(vrt.lib().vrt_q8_gemv(ctx.h, w, raw.nbytes, 0, dx, dy, n_in, n_out, None))
    y1 = ctx.download(dy, n_out)
    assert np.abs(y1 - ref).max() <= 2e-3
    vrt.check(vrt.lib().vrt_q8_gemv(ctx.h, w, raw.nbytes, 0, dx, dy, n_in, n_out, None))
    assert np.array_equal(y1, ctx.download(dy, n_out))  # replay identical (reference: <= 1e-6)
    # pair / triplet: three copies of the matrix, packed output (q8_test_main.cpp:324-581)
    multi = np.concatenate([raw, raw, raw])
    wm = ctx.upload(multi)
    offs = (C.c_uint64 * 3)(0, raw.nbytes, 2 * raw.nbytes)
    dims = (C.c_uint32 * 3)(n_out, n_out, n_out)
    dy3 = ctx.alloc(12 * n_out)
    for count in (2, 3):
        vrt.check(vrt.lib().vrt_q8_gemv_multi(ctx.h, wm, multi.nbytes, offs, dims, count, dx, dy3, n_in, None))
        y3 = ctx.download(dy3, count * n_out)
        for c in range(count):
            assert np.array_equal(y3[c * n_out:(c + 1) * n_out], y1)
    # packed (Q8T) path: 257 rows exercises the zero-padded last row group
    pk = ctx.alloc(vrt.lib().vrt_q8t_bytes(n_out, n_in))
    vrt.check(vrt.lib().vrt_q8t_pack(ctx.h, w, raw.nbytes, 0, n_out, n_in, pk, None))
    vrt.check(vrt.lib().vrt_q8t_gemv(ctx.h, pk, n_out, n_in, dx, dy, None))
    yp = ctx.download(dy, n_out)
    assert np.abs(yp - ref).max() <= 2e-3
    vrt.check(vrt.lib().vrt_q8t_gemv(ctx.h, pk, n_out, n_in, dx, dy, None))
    assert np.array_equal(yp, ctx.download(dy, n_out))


def test_q8_ffn_known_answer(ctx):
    raw, offs, x, ref, (n_in, n_ffn, n_out) = kat.ffn_test_case()
    w = ctx.upload(raw)
    dx = ctx.upload(x)
    ws = ctx.alloc(4 * 2 * n_ffn)
    dy = ctx.alloc(4 * n_out)
    args = (ctx.h, w, raw.nbytes, offs[0], offs[1], offs[2], dx, ws, dy, n_in, n_ffn, n_out, None)
    vrt.check(vrt.lib().vrt_q8_ffn(*args))
    y1 = ctx.download(dy, n_out)
    assert np.abs(y1 - ref).max() <= 5e-3
    vrt.check(vrt.lib().vrt_q8_ffn(*args))
    assert np.abs(ctx.download(dy, n_out) - y1).max() <= 1e-6


def test_gelu_known_answer(ctx):
    gate, up, ref = kat.gelu_test_case()
    dg, du = ctx.upload(gate), ctx.upload(up)
    vrt.check(vrt.lib().vrt_gelu_mul(ctx.h, dg, du, gate.size, None))
    assert np.abs(ctx.download(dg, gate.size) - ref).max() <= 5e-5


@pytest.mark.parametrize("case", ["ties", "nan", "allnan", "neginf", "single", "large", "last"])
def test_argmax_edge_cases(ctx, case):
    rng = np.random.default_rng(5)
    if case == "ties":
        v = np.zeros(1000, np.float32); v[[10, 500, 999]] = 7.0
    elif case == "nan":
        v = rng.standard_normal(5000).astype(np.float32); v[::7] = np.nan; v[3000] = 9.0
    elif case == "allnan":
        v = np.full(300, np.nan, np.float32)
    elif case == "neginf":
        v = np.full(300, -np.inf, np.float32)
    elif case == "single":
        v = np.array([-3.5], np.float32)
    elif case == "large":
        v = rng.standard_normal(262144 * 4 + 13).astype(np.float32)
    else:
        v = np.zeros(4097, np.float32); v[-1] = 1.0
    dv = ctx.upload(v)
    res = ctx.alloc(8)
    vrt.check(vrt.lib().vrt_argmax(ctx.h, dv, v.size, res, None))
    got = _argmax_dev(ctx, res)
    want = O.argmax(v)
    assert got[0] == want[0]
    assert (got[1] == want[1]) or (np.isinf(got[1]) and np.isinf(want[1]))


def _synthetic(rows, cols, name, seed=1234):
    return sg.q8_matrix_bytes(seed, name, rows, cols)


# The isolated-sweep shapes of the benchmark plan (rows x cols).
SWEEP = [(1920, 640), (640, 1024), (2048, 640), (640, 2048), (21504, 5376)]


@pytest.mark.parametrize("rows,cols", SWEEP)
def test_gemv_vs_oracle(ctx, rows, cols):
    raw = _synthetic(rows, cols, f"sweep.{rows}x{cols}")
    x = np.random.default_rng(rows).standard_normal(cols).astype(np.float32)
    ref = O.q8_matvec(raw, x, rows, lanes=0, threads=8)   # fp64 reference mat-vec
    w, dx, dy = ctx.upload(raw), ctx.upload(x), ctx.alloc(4 * rows)
    vrt.check(vrt.lib().vrt_q8_gemv(ctx.h, w, raw.nbytes, 0, dx, dy, cols, rows, None))
    _close(ctx.download(dy, rows), ref)
    pk = ctx.alloc(vrt.lib().vrt_q8t_bytes(rows, cols))
    vrt.check(vrt.lib().vrt_q8t_pack(ctx.h, w, raw.nbytes, 0, rows, cols, pk, None))
    vrt.check(vrt.lib().vrt_q8t_gemv(ctx.h, pk, rows, cols, dx, dy, None))
    _close(ctx.download(dy, rows), ref)


def test_fused_ffn_270m_shape_vs_oracle(ctx):
    d, ff = 640, 2048
    g = _synthetic(ff, d, "sweep.gate")
    u = _synthetic(ff, d, "sweep.up")
    dn = _synthetic(d, ff, "sweep.down")
    raw = np.concatenate([g, u, dn])
    x = np.random.default_rng(3).standard_normal(d).astype(np.float32)
    rg = O.q8_matvec(g, x, ff, lanes=0)
    ru = O.q8_matvec(u, x, ff, lanes=0)
    act = O.gelu_mul(rg, ru)
    ref = O.q8_matvec(dn, act, d, lanes=0)
    w, dx = ctx.upload(raw), ctx.upload(x)
    ws, dy = ctx.alloc(8 * ff), ctx.alloc(4 * d)
    vrt.check(vrt.lib().vrt_q8_ffn(ctx.h, w, raw.nbytes, 0, g.nbytes, g.nbytes + u.nbytes, dx, ws, dy, d, ff, d,
                                   None))
    _close(ctx.download(dy, d), ref)
    # packed: gate/up pair (gelu fused in the epilogue) + down
    pair = ctx.alloc(vrt.lib().vrt_q8t_bytes(2 * ff, d))
    down = ctx.alloc(vrt.lib().vrt_q8t_bytes(d, ff))
    vrt.check(vrt.lib().vrt_q8t_pack_pair(ctx.h, w, raw.nbytes, 0, g.nbytes, ff, d, pair, None))
    vrt.check(vrt.lib().vrt_q8t_pack(ctx.h, w, raw.nbytes, g.nbytes + u.nbytes, d, ff, down, None))
    act_d = ctx.alloc(4 * ff)
    vrt.check(vrt.lib().vrt_q8t_gate_up(ctx.h, pair, ff, d, dx, act_d, None))
    _close(ctx.download(act_d, ff), act)
    vrt.check(vrt.lib().vrt_q8t_ffn(ctx.h, pair, down, d, ff, d, dx, act_d, dy, None))
    _close(ctx.download(dy, d), ref)


def test_lm_head_argmax_270m_vs_oracle(ctx):
    V, d = 262144, 640
    raw = _synthetic(V, d, "token_embd.weight", seed=42)
    x = np.random.default_rng(9).standard_normal(d).astype(np.float32)
    ref = O.q8_matvec(raw, x, V, lanes=0, threads=8)
    w, dx = ctx.upload(raw), ctx.upload(x)
    logits, res = ctx.alloc(4 * V), ctx.alloc(8)
    vrt.check(vrt.lib().vrt_lm_head_argmax(ctx.h, w, raw.nbytes, 0, dx, d, V, logits, res, None))
    got = ctx.download(logits, V)
    _close(got, ref)
    idx, val = _argmax_dev(ctx, res)
    assert (idx, val) == O.argmax(got)  # fused argmax == argmax of the kernel's own logits
    top2 = np.sort(ref)[-2:]
    if top2[1] - top2[0] > 1e-3:
        assert idx == int(np.argmax(ref))
    pk = ctx.alloc(vrt.lib().vrt_q8t_bytes(V, d))
    vrt.check(vrt.lib().vrt_q8t_pack(ctx.h, w, raw.nbytes, 0, V, d, pk, None))
    vrt.check(vrt.lib().vrt_q8t_lm_head_argmax(ctx.h, pk, V, d, dx, logits, res, None))
    got2 = ctx.download(logits, V)
    _close(got2, ref)
    assert _argmax_dev(ctx, res) == O.argmax(got2)


def test_invalid_arguments_rejected(ctx):
    raw, x, ref, n_in, n_out = kat.q8_test_case()
    w, dx, dy = ctx.upload(raw), ctx.upload(x), ctx.alloc(4 * n_out)
    L = vrt.lib()
    assert L.vrt_q8_gemv(ctx.h, w, raw.nbytes, 2, dx, dy, n_in, n_out, None) == vrt.VRT_E_INVALID
    assert b"4-byte aligned" in L.vrt_last_error()
    assert L.vrt_q8_gemv(ctx.h, w, raw.nbytes, 0, dx, dy, 33, n_out, None) == vrt.VRT_E_INVALID
    assert L.vrt_q8_gemv(ctx.h, w, raw.nbytes, 0, dx, dy, n_in, n_out + 1, None) == vrt.VRT_E_INVALID
    assert b"too small" in L.vrt_last_error()
    assert L.vrt_q8_gemv(ctx.h, w, raw.nbytes, 0, dx, dy, 0, n_out, None) == vrt.VRT_E_INVALID
    assert L.vrt_argmax(ctx.h, dx, 0, dy, None) == vrt.VRT_E_INVALID
    assert L.vrt_q8t_gemv(ctx.h, w, n_out, 96, dx, dy, None) == vrt.VRT_E_INVALID
