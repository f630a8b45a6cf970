"""Streaming GGUF upload (model.cu `Loader`): a 270M-shaped file (291 MB of
Q8_0 + norms, written by synth_gguf) loaded through the pipelined loader
(memory-mapped file, host copies on worker threads, three pinned staging
buffers recycled through CUDA events, repack on the device) decodes bit for
bit like the device-side generator of the same seed.  The load rate of a
cold and a warm (page-cached) load is printed."""

import os
import time

import numpy as np
import pytest

import synth_gguf as sg
import vrt

pytestmark = pytest.mark.gpu


def test_loader_270m_equals_device_generator(ctx, model_dir):
    shape = sg.SHAPES["270m"]
    path = sg.cached_model(shape, 555, model_dir)
    size = os.path.getsize(path)
    models = []
    for what in ("cold", "warm"):
        t0 = time.perf_counter()
        models.append(vrt.Model(ctx, path, max_positions=32))
        dt = time.perf_counter() - t0
        print(f"{what} load of {size / 1e6:.0f} MB in {dt:.2f} s ({size / dt / 1e9:.2f} GB/s)")
    models[1].close()
    a = models[0]
    b = vrt.Model(ctx, None, config=vrt.Gemma3Config.from_shape(shape), seed=555, max_positions=32)
    for pos, t in enumerate([2, 7, 300, 262143]):
        ha, ia, la = a.decode(t, pos, 1)
        hb, ib, lb = b.decode(t, pos, 1)
        assert np.array_equal(ha, hb) and np.array_equal(ia, ib) and np.array_equal(la, lb)
    assert np.array_equal(a.logits(), b.logits())
