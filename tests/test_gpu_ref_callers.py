"""The reference's own callers on this backend (tests/ref_callers/Makefile).

src/q8_test_main.cpp, src/ffn_test_main.cpp and src/gemma_main.cpp are
compiled unmodified from the reference tree against include/vortexrt/*.hpp
and libvortexrt_b200.so, so the C++ drop-in surface (VulkanContext, Buffer,
Q8MatVecPipeline, ArgmaxPipeline, Gemma3Model, GgufFile) is driven by the
code it replaces:

* the Q8 test: every lane variant (8/16/32/64), the staged path, the fused
  pair and triplet, replay identity (q8_test_main.cpp:185-617, its own
  tolerances 2e-3 and 1e-6), "Validation: OK";
* the FFN test: the fused gate/up -> gelu -> down path against its fp64
  matvec (ffn_test_main.cpp:254-441);
* the reference CLI on synthetic GGUFs: generated ids equal the reference's
  own token loop (oracle/_ref) unless its top-2 margin is below 1e-3, and the
  top-k logits match within atol/rtol 1e-3.

The binaries are built where the reference tree exists (in build()); a box
without them skips these tests.
"""

import os
import re
import subprocess

import numpy as np
import pytest

import oracle as O
import synth_gguf as sg

pytestmark = pytest.mark.gpu
BIN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "ref_callers", "_bin")


def _run(name, *args, expect_ok=True):
    exe = os.path.join(BIN, name)
    if not os.path.exists(exe):
        pytest.skip(f"{name} not built (the reference tree was absent when the repository was built)")
    p = subprocess.run([exe, *args], capture_output=True, text=True, errors="replace", timeout=600)
    if expect_ok:
        assert p.returncode == 0, p.stdout + p.stderr
    return p


def test_reference_q8_test_program():
    out = _run("vortexrt-q8-test").stdout
    assert "Validation: OK" in out
    for what in ("max abs error", "32-lane max abs error", "16-lane max abs error", "8-lane max abs error",
                 "staged max abs error", "fused pair max abs error", "fused triplet max abs error"):
        v = float(re.search(rf"  {what}: ([-\d.e+]+)", out).group(1))
        assert v <= 2e-3, (what, v)
    for what in ("staged cached replay error", "fused pair cached replay error", "fused triplet cached replay error"):
        assert float(re.search(rf"  {what}: ([-\d.e+]+)", out).group(1)) <= 1e-6


def test_reference_ffn_test_program():
    p = _run("vortexrt-ffn-test")
    assert "Validation: OK" in p.stdout, p.stdout


@pytest.mark.parametrize("name,seed,gen", [("tiny", 1234, 16), ("270m", 1234, 8)])
def test_reference_cli_generate_vs_reference_loop(model_dir, name, seed, gen):
    if not O.reference_available():
        pytest.skip("oracle/_ref not built")
    path = sg.cached_model(sg.SHAPES[name], seed, model_dir)
    out = _run("vortexrt-gemma", path, "--token-id", "2", "--generate", str(gen)).stdout
    got = [int(x) for x in re.search(r"Generated token ids:(.*)", out).group(1).split()]
    r = O.Reference(path, threads=os.cpu_count() or 1)
    ref, _ = r.generate([2], gen)
    # the reference's margins along its own stream
    r.reset()
    margins = []
    tok = 2
    for pos in range(gen):
        _, ids, lg = r.decode(tok, pos, 2)
        margins.append(float(lg[0] - lg[1]))
        tok = int(ids[0])
    for i, (a, b) in enumerate(zip(got, ref)):
        if a != b:
            assert margins[i] < 1e-3, (got, ref, margins[i])
            break
    else:
        assert got == ref


def test_reference_cli_top_logits_vs_reference_loop(model_dir):
    if not O.reference_available():
        pytest.skip("oracle/_ref not built")
    path = sg.cached_model(sg.SHAPES["tiny"], 1234, model_dir)
    out = _run("vortexrt-gemma", path, "--token-id", "2", "--top-k", "8").stdout
    rows = re.findall(r"id=(\d+) logit=([-\d.e+]+)", out)
    assert len(rows) == 8
    r = O.Reference(path)
    _, ids, lg = r.decode(2, 0, 8, single=True)
    got = np.array([float(v) for _, v in rows], np.float64)
    assert np.all(np.abs(got - lg) <= 1e-3 + 1e-3 * np.abs(lg))
    assert [int(i) for i, _ in rows][:1] == [int(ids[0])]


def test_reference_cli_rejects_bad_flags(model_dir):
    path = sg.cached_model(sg.SHAPES["tiny"], 1234, model_dir)
    p = _run("vortexrt-gemma", path, "--q8-lanes", "12", expect_ok=False)
    assert p.returncode != 0 and "q8-lanes" in p.stderr
