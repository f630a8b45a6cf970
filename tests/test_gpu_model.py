"""Decode-step parity of the GPU-resident token loop against the CPU oracle
and the reference's own token loop, through the C ABI.

* hidden states, logits and per-layer residuals within atol 1e-3 / rtol 1e-3;
* greedy token streams identical, except that from the first step whose
  oracle top-2 logit margin is below 1e-3 on, the streams may diverge;
* KV indexing: the sliding window is crossed (tiny window 8) and global
  layers grow linearly;
* the device-side generator is bit-identical to loading the GGUF it writes.
"""

import numpy as np
import pytest

import oracle as O
import synth_gguf as sg
import vrt

pytestmark = pytest.mark.gpu
ATOL, RTOL = 1e-3, 1e-3


def _close(a, b, atol=ATOL, rtol=RTOL):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    err = np.abs(a - b)
    bound = atol + rtol * np.abs(b)
    assert np.all(err <= bound), f"max err {err.max():.3g} (worst ratio {(err / bound).max():.3g})"


def _streams_agree(gpu, ref, margins, tol=1e-3):
    for i, (a, b) in enumerate(zip(gpu, ref)):
        if a != b:
            assert margins[i] < tol, f"step {i}: gpu {a} vs ref {b} with margin {margins[i]}"
            return i
    assert len(gpu) == len(ref) or (len(gpu) < len(ref) and gpu[-1] == 1) or (len(ref) < len(gpu) and ref[-1] == 1)
    return None


@pytest.fixture(scope="module")
def tiny_path(model_dir):
    return sg.cached_model(sg.SHAPES["tiny"], 1234, model_dir)


@pytest.fixture(scope="module")
def gqa_path(model_dir):
    return sg.cached_model(sg.SHAPES["tiny-gqa"], 4321, model_dir)


@pytest.mark.parametrize("which", ["tiny", "gqa"])
def test_decode_steps_vs_oracle(ctx, which, tiny_path, gqa_path):
    path = tiny_path if which == "tiny" else gqa_path
    m = vrt.Model(ctx, path, max_positions=64)
    o = O.Oracle(path)
    m.set_trace(True)
    rng = np.random.default_rng(1)
    toks = [2] + rng.integers(3, o.vocab, 39).tolist()   # 40 positions: crosses the window of 8
    for pos, t in enumerate(toks):
        trace = np.zeros((o.L, o.d), np.float32)
        h_ref, ids_ref, lg_ref, full_ref = o.decode(t, pos, 1, full_logits=True, trace=trace)
        h, ids, lg = m.decode(t, pos, 1)
        _close(h, h_ref)
        _close(m.trace(), trace)
        _close(m.logits(), full_ref)
        top2 = np.sort(full_ref)[-2:]
        if top2[1] - top2[0] > 1e-3:
            assert int(ids[0]) == int(ids_ref[0]), pos
        _close(lg, lg_ref)


def test_generate_vs_reference_tiny(ctx, tiny_path):
    m = vrt.Model(ctx, tiny_path, max_positions=128)
    o = O.Oracle(tiny_path)
    prompt = [2, 300, 301, 302]
    ref, margins = o.generate(prompt, 40, margins=True)
    gpu = m.generate(prompt, 40)
    _streams_agree(gpu, ref, margins)
    if O.reference_available():
        assert O.Reference(tiny_path).generate(prompt, 40)[0] == ref


def test_top_k_and_zero(ctx, tiny_path):
    m = vrt.Model(ctx, tiny_path, max_positions=16)
    o = O.Oracle(tiny_path)
    h0, ids0, lg0 = m.decode(2, 0, 0)
    h0r, _, _ = o.decode(2, 0, 0)
    _close(h0, h0r)
    assert ids0.size == 0
    h1, ids, lg = m.decode(300, 1, 8)
    h1r, idsr, lgr = o.decode(300, 1, 8)
    _close(h1, h1r)
    _close(lg, lgr)
    full = m.logits()
    assert list(ids) == sorted(range(full.size), key=lambda i: (-full[i], i))[:8]


def test_graph_pdl_variants_identical(ctx, tiny_path):
    """Graph replay, PDL and plain stream launches give bit-identical results."""
    outs = []
    for g, p in ((True, True), (True, False), (False, False), (False, True)):
        m = vrt.Model(ctx, tiny_path, max_positions=64, use_graph=g, use_pdl=p)
        ids = m.generate([2, 5, 6, 7], 20)
        m.reset()
        h = np.stack([m.decode(t, i, 1)[0] for i, t in enumerate([2, 5, 6, 7, 8])])
        outs.append((ids, h))
        m.close()
    for ids, h in outs[1:]:
        assert ids == outs[0][0]
        assert np.array_equal(h, outs[0][1])


def test_device_generator_equals_file(ctx, model_dir):
    for name in ("tiny", "tiny-gqa"):
        shape = sg.SHAPES[name]
        path = sg.cached_model(shape, 555, model_dir)
        a = vrt.Model(ctx, path, max_positions=32)
        b = vrt.Model(ctx, None, config=vrt.Gemma3Config.from_shape(shape), seed=555, max_positions=32)
        for pos, t in enumerate([2, 7, 300, 11]):
            ha, ia, la = a.decode(t, pos, 1)
            hb, ib, lb = b.decode(t, pos, 1)
            assert np.array_equal(ha, hb) and np.array_equal(ia, ib) and np.array_equal(la, lb)
            assert np.array_equal(a.logits(), b.logits())


def test_errors_and_reset(ctx, tiny_path):
    m = vrt.Model(ctx, tiny_path, max_positions=8)
    with pytest.raises(vrt.VrtError, match="contiguous"):
        m.decode(2, 1, 1)
    with pytest.raises(vrt.VrtError, match="vocabulary"):
        m.decode(10 ** 6, 0, 1)
    for p in range(8):
        m.decode(2, p, 1)
    with pytest.raises(vrt.VrtError, match="capacity|context"):
        m.decode(2, 8, 1)
    m.reset()
    m.decode(2, 0, 1)
    assert m.device_status() == 0
    with pytest.raises(vrt.VrtError):
        vrt.Model(ctx, "/nonexistent.gguf")
    assert m.generate([2], 0) == []
    with pytest.raises(vrt.VrtError, match="no input tokens"):
        m.generate([], 3)


def test_270m_config0_vs_reference(ctx, model_dir):
    """Config 0: BOS + 8 seeded ids, 16 greedy tokens, on the 270M shape."""
    shape = sg.SHAPES["270m"]
    path = sg.cached_model(shape, 2024, model_dir)
    prompt = [2] + np.random.default_rng(2024).integers(3, shape.vocab_size, 8).tolist()
    o = O.Oracle(path, threads=16)
    ref, margins = o.generate(prompt, 16, margins=True)
    m = vrt.Model(ctx, path, max_positions=64)
    gpu = m.generate(prompt, 16)
    _streams_agree(gpu, ref, margins)
    if O.reference_available():
        r = O.Reference(path, threads=16)
        assert r.generate(prompt, 16)[0] == ref
    m.reset()
    o.reset()
    for pos, t in enumerate(prompt[:3]):
        _close(m.decode(t, pos, 1)[0], o.decode(t, pos, 1)[0])
    b = vrt.Model(ctx, None, config=vrt.Gemma3Config.from_shape(shape), seed=2024, max_positions=64)
    assert b.generate(prompt, 16) == gpu


def test_27b_shape_slice_vs_oracle(ctx):
    """27B widths (d 5376, 32 q heads / 16 KV heads of 128, ffn 21504) on a
    6-layer, 16384-vocab slice: GQA, a global layer, the GQA restatement."""
    shape = sg.SHAPES["27b"].with_(block_count=6, vocab_size=16384, name="27b-slice")
    o = O.Oracle(shape=shape, seed=27, threads=16, max_positions=16)
    m = vrt.Model(ctx, None, config=vrt.Gemma3Config.from_shape(shape), seed=27, max_positions=16)
    for pos, t in enumerate([2, 1000, 2000, 3000]):
        h_ref, ids_ref, lg_ref, full = o.decode(t, pos, 1, full_logits=True)
        h, ids, lg = m.decode(t, pos, 1)
        _close(h, h_ref)
        _close(m.logits(), full)
        top2 = np.sort(full)[-2:]
        if top2[1] - top2[0] > 1e-3:
            assert int(ids[0]) == int(ids_ref[0])
