"""vrt_q8_ffn_static: the fused FFN for callers that cannot allocate device
memory (no context, no workspace; its gate/up intermediate lives in a
library-owned device array).  Checked through the C ABI against the existing
entry point, vrt_q8_ffn, on two calls in a row, within the tolerance the
other kernel tests use (atol 1e-3, rtol 1e-3; the same kernels run, so the
results are expected to be identical), and against an independent CPU
result: the reference FFN test's own expected output for its case (its
tolerance, 5e-3) and the oracle's fp64 FFN for the 27B-shaped case and for
ffn_dim at the array's limit of 32768.  This file sorts last so that a run
stopping at the first failure has run every other test first; it also passes
on its own in a fresh process."""

import ctypes as C
import os

import numpy as np
import pytest

import kat
import oracle as O
import synth_gguf as sg
import vrt

pytestmark = pytest.mark.gpu


def _close(a, b):
    err = np.abs(a.astype(np.float64) - b.astype(np.float64))
    assert np.all(err <= 1e-3 + 1e-3 * np.abs(b.astype(np.float64))), err.max()


def _fp64_ffn(g, u, dn, x, ff, d_out):
    """The oracle's FFN: fp64 mat-vecs (ffn_test's matvec) and gelu_tanh * up."""
    threads = os.cpu_count() or 1
    a = O.gelu_mul(O.q8_matvec(g, x, ff, lanes=0, threads=threads), O.q8_matvec(u, x, ff, lanes=0, threads=threads))
    return O.q8_matvec(dn, a, d_out, lanes=0, threads=threads)


def _synthetic(seed, d_in, ff, d_out):
    g = sg.q8_matrix_bytes(seed, "static.gate", ff, d_in)
    u = sg.q8_matrix_bytes(seed, "static.up", ff, d_in)
    dn = sg.q8_matrix_bytes(seed, "static.down", d_out, ff)
    x = np.random.default_rng(seed).standard_normal(d_in).astype(np.float32)
    return (np.concatenate([g, u, dn]), (0, g.nbytes, g.nbytes + u.nbytes), x, d_in, ff, d_out,
            _fp64_ffn(g, u, dn, x, ff, d_out), 1e-3)


def _cases():
    # (weights, offsets, x, input_dim, ffn_dim, output_dim, independent reference, its tolerance)
    raw, offs, x, ref, (n_in, n_ffn, n_out) = kat.ffn_test_case()
    yield raw, offs, x, n_in, n_ffn, n_out, ref, 5e-3  # src/ffn_test_main.cpp's case and tolerance
    yield _synthetic(9, 5376, 21504, 5376)  # the 27B-shaped FFN
    yield _synthetic(10, 64, 32768, 64)     # ffn_dim at the static array's limit


def test_static_ffn_matches_workspace_ffn():
    L = vrt.lib()
    with vrt.Context(0) as ctx:
        for raw, offs, x, n_in, n_ffn, n_out, ref, tol in _cases():
            w, dx = ctx.upload(raw), ctx.upload(x)
            ws, y_ref, y = ctx.alloc(8 * n_ffn), ctx.alloc(4 * n_out), ctx.alloc(4 * n_out)
            vrt.check(L.vrt_q8_ffn(ctx.h, w, raw.nbytes, offs[0], offs[1], offs[2], dx, ws, y_ref, n_in, n_ffn,
                                   n_out, None))
            want = ctx.download(y_ref, n_out)
            for _ in range(2):  # the scratch keeps the previous call's contents
                # on the caller's stream (the context's), so the read-back below is ordered after it
                vrt.check(L.vrt_q8_ffn_static(w, raw.nbytes, offs[0], offs[1], offs[2], dx, y, n_in, n_ffn,
                                              n_out, ctx.stream))
                vrt.check(L.vrt_ctx_synchronize(ctx.h))
                got = ctx.download(y, n_out)
                _close(got, want)
                err = np.abs(got.astype(np.float64) - np.asarray(ref, np.float64))
                assert np.all(err <= tol + tol * np.abs(np.asarray(ref, np.float64))), (n_ffn, err.max())


def test_static_ffn_rejects_oversized():
    L = vrt.lib()
    with vrt.Context(0) as ctx:
        big = 32768 + 32
        dummy = ctx.alloc(64)
        rc = L.vrt_q8_ffn_static(dummy, 1 << 40, 0, 0, 0, dummy, dummy, 64, big, 64, None)
        assert rc == vrt.VRT_E_INVALID
        assert b"static scratch limit" in L.vrt_last_error()
