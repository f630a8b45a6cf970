"""The raw-row pipeline mat-vec (`vrt_q8_gemv`, `vrt_q8_gemv_multi`,
`vrt_lm_head_argmax`: the Q8MatVecPipeline replacement over GGUF-layout
Q8_0 rows) on shapes and offsets that reach every form of the kernels:

* the staged kernel at every lanes-per-row width (8 .. 512, and two blocks
  per thread above 512 blocks per row), with matrices at 4-byte offsets that
  are not 16-byte aligned (the blocks touching a partial 16-byte chunk at
  either end of the matrix are read from global memory), odd block counts
  (rows starting 2 bytes off a word), rows fewer than one iteration, several
  matrices in one call, x at an address that is not 16-byte aligned;
* the row-wise kernel: rows wider than 1024 blocks, and every case again
  under VRT_RAW_ROWWISE=1 in a child process.

Each output is checked against the oracle's fp64 mat-vec within atol/rtol
1e-3 and must replay bit for bit.
"""

import ctypes as C
import json
import os
import subprocess
import sys

import numpy as np
import pytest

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path[:0] = [os.path.join(HERE, "..", "vortex-rt_b200"), os.path.join(HERE, "..", "oracle")]

import oracle as O  # noqa: E402
import synth_gguf as sg  # noqa: E402
import vrt  # noqa: E402

pytestmark = pytest.mark.gpu
ATOL, RTOL = 1e-3, 1e-3

# rows, cols, byte offset of the matrix in its buffer
CASES = [
    (1, 32, 0),        # one block, one row
    (7, 96, 4),        # 3 blocks (odd): LPR 8
    (300, 160, 12),    # 5 blocks: LPR 8, offset 12
    (5000, 256, 20),   # 8 blocks, many iterations
    (2049, 640, 4),    # 20 blocks: LPR 32 (the 270M width)
    (513, 1056, 8),    # 33 blocks: LPR 64
    (100, 5376, 4),    # 168 blocks: LPR 256 (the 27B width)
    (37, 16416, 12),   # 513 blocks: two blocks per thread
    (64, 21504, 4),    # 672 blocks: two blocks per thread
    (40, 32768, 0),    # 1024 blocks: the widest staged row
    (9, 32800, 4),     # 1025 blocks: the row-wise kernel
]


def _case_data(rows, cols, off, seed):
    raw = sg.q8_matrix_bytes(seed, f"raw.{rows}x{cols}", rows, cols)
    buf = np.zeros(off + raw.nbytes + 20, np.uint8)
    buf[off:off + raw.nbytes] = raw
    buf[off + raw.nbytes:] = 0xA5  # bytes past the matrix: never part of a result
    if off:
        buf[:off] = 0x5A
    x = np.random.default_rng(seed + cols).standard_normal(cols).astype(np.float32)
    return raw, buf, x


def _run_gemv(ctx, rows, cols, off, seed=7):
    raw, buf, x = _case_data(rows, cols, off, seed)
    w, dx, dy = ctx.upload(buf), ctx.upload(x), ctx.alloc(4 * rows)
    vrt.check(vrt.lib().vrt_q8_gemv(ctx.h, w, buf.nbytes, off, dx, dy, cols, rows, None))
    y1 = ctx.download(dy, rows)
    vrt.check(vrt.lib().vrt_q8_gemv(ctx.h, w, buf.nbytes, off, dx, dy, cols, rows, None))
    y2 = ctx.download(dy, rows)
    return raw, x, y1, y2


def _close(y, ref):
    err = np.abs(y.astype(np.float64) - ref.astype(np.float64))
    bound = ATOL + RTOL * np.abs(ref.astype(np.float64))
    assert np.all(err <= bound), f"max err {err.max():.3g}, worst ratio {(err / bound).max():.3g}"


@pytest.mark.parametrize("rows,cols,off", CASES)
def test_raw_gemv_vs_oracle(ctx, rows, cols, off):
    raw, x, y1, y2 = _run_gemv(ctx, rows, cols, off)
    ref = O.q8_matvec(raw, x, rows, lanes=0, threads=8)
    _close(y1, ref)
    assert np.array_equal(y1, y2)


@pytest.mark.parametrize("rows,cols", [(300, 640), (64, 21504)])
def test_raw_gemv_x_not_16_byte_aligned(ctx, rows, cols):
    """x at a 4-byte (not 16-byte) aligned address: the scalar activation loads."""
    raw, buf, x = _case_data(rows, cols, 4, 21)
    xs = np.concatenate([np.zeros(1, np.float32), x])
    w, dxs, dy = ctx.upload(buf), ctx.upload(xs), ctx.alloc(4 * rows)
    vrt.check(vrt.lib().vrt_q8_gemv(ctx.h, w, buf.nbytes, 4, dxs + 4, dy, cols, rows, None))
    _close(ctx.download(dy, rows), O.q8_matvec(raw, x, rows, lanes=0, threads=8))


def test_raw_gemv_multi_unaligned(ctx):
    cols = 640
    dims = [300, 64, 1000, 17]
    seed = 11
    mats = [sg.q8_matrix_bytes(seed, f"multi.{i}", r, cols) for i, r in enumerate(dims)]
    offs, pos, parts = [], 4, [np.full(4, 0x5A, np.uint8)]
    for i, m in enumerate(mats):
        offs.append(pos)
        gap = (4, 12, 8, 0)[i]
        parts += [m, np.full(gap, 0xA5, np.uint8)]
        pos += m.nbytes + gap
    buf = np.concatenate(parts)
    x = np.random.default_rng(5).standard_normal(cols).astype(np.float32)
    w, dx, dy = ctx.upload(buf), ctx.upload(x), ctx.alloc(4 * sum(dims))
    c_offs = (C.c_uint64 * len(dims))(*offs)
    c_dims = (C.c_uint32 * len(dims))(*dims)
    vrt.check(vrt.lib().vrt_q8_gemv_multi(ctx.h, w, buf.nbytes, c_offs, c_dims, len(dims), dx, dy, cols, None))
    y = ctx.download(dy, sum(dims))
    at = 0
    for m, r in zip(mats, dims):
        _close(y[at:at + r], O.q8_matvec(m, x, r, lanes=0, threads=8))
        at += r


def test_raw_lm_head_argmax_unaligned(ctx):
    V, d, off = 70001, 640, 4
    raw, buf, x = _case_data(V, d, off, 3)
    w, dx = ctx.upload(buf), ctx.upload(x)
    logits, res = ctx.alloc(4 * V), ctx.alloc(8)
    vrt.check(vrt.lib().vrt_lm_head_argmax(ctx.h, w, buf.nbytes, off, dx, d, V, logits, res, None))
    got = ctx.download(logits, V)
    _close(got, O.q8_matvec(raw, x, V, lanes=0, threads=8))
    r = ctx.download(res, 2, np.uint32)
    assert (int(r[0]), float(r[1:2].view(np.float32)[0])) == O.argmax(got)


def test_pipeline_status_clear(ctx):
    """No wait of the staged kernel expired in this process's calls (context
    and static entry points); the word reads back cleared."""
    _run_gemv(ctx, 2049, 640, 4)
    for h in (ctx.h, None):
        st = C.c_uint32(0xFFFFFFFF)
        vrt.check(vrt.lib().vrt_pipeline_status(h, C.byref(st)))
        assert st.value == 0


def _child_outputs(out_path):
    """Child process body: every case through vrt_q8_gemv, outputs saved."""
    ctx = vrt.Context(0)
    res = {}
    for rows, cols, off in CASES:
        _, _, y1, y2 = _run_gemv(ctx, rows, cols, off)
        res[f"{rows}x{cols}+{off}"] = [y1.tolist(), bool(np.array_equal(y1, y2))]
    ctx.close()
    with open(out_path, "w") as f:
        json.dump(res, f)


def test_rowwise_kernel_vs_oracle(tmp_path):
    out = tmp_path / "rowwise.json"
    env = dict(os.environ, VRT_RAW_ROWWISE="1")
    p = subprocess.run([sys.executable, os.path.abspath(__file__), str(out)], env=env, capture_output=True,
                       text=True, timeout=600)
    assert p.returncode == 0, p.stdout + p.stderr
    res = json.loads(out.read_text())
    for rows, cols, off in CASES:
        y, replay_equal = res[f"{rows}x{cols}+{off}"]
        raw, _, x = _case_data(rows, cols, off, 7)
        _close(np.asarray(y, np.float32), O.q8_matvec(raw, x, rows, lanes=0, threads=8))
        assert replay_equal


if __name__ == "__main__":
    _child_outputs(sys.argv[1])
