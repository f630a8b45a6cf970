"""vrt_q8_ffn_static: the fused FFN for callers that cannot allocate device
memory (no context, no workspace; its gate/up intermediate lives in a
library-owned device array).  Checked through the C ABI against the existing
entry point, vrt_q8_ffn, on two calls in a row, within the tolerance the
other kernel tests use (atol 1e-3, rtol 1e-3; the same kernels run, so the
results are expected to be identical).  This file sorts last so that a run
stopping at the first failure has run every other test first; it also
passes on its own in a fresh process."""

import ctypes as C

import numpy as np
import pytest

import kat
import synth_gguf as sg
import vrt

pytestmark = pytest.mark.gpu


def _close(a, b):
    err = np.abs(a.astype(np.float64) - b.astype(np.float64))
    assert np.all(err <= 1e-3 + 1e-3 * np.abs(b.astype(np.float64))), err.max()


def _cases():
    raw, offs, x, ref, (n_in, n_ffn, n_out) = kat.ffn_test_case()
    yield raw, offs, x, n_in, n_ffn, n_out
    d, ff = 5376, 21504  # the 27B-shaped FFN, the largest the runtime serves
    g = sg.q8_matrix_bytes(9, "static.gate", ff, d)
    u = sg.q8_matrix_bytes(9, "static.up", ff, d)
    dn = sg.q8_matrix_bytes(9, "static.down", d, ff)
    xx = np.random.default_rng(9).standard_normal(d).astype(np.float32)
    yield np.concatenate([g, u, dn]), (0, g.nbytes, g.nbytes + u.nbytes), xx, d, ff, d


def test_static_ffn_matches_workspace_ffn():
    L = vrt.lib()
    with vrt.Context(0) as ctx:
        for raw, offs, x, n_in, n_ffn, n_out in _cases():
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
                _close(ctx.download(y, n_out), want)


def test_static_ffn_rejects_oversized():
    L = vrt.lib()
    with vrt.Context(0) as ctx:
        big = 32768 + 32
        dummy = ctx.alloc(64)
        rc = L.vrt_q8_ffn_static(dummy, 1 << 40, 0, 0, 0, dummy, dummy, 64, big, 64, None)
        assert rc == vrt.VRT_E_INVALID
        assert b"static scratch limit" in L.vrt_last_error()
