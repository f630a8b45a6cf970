"""The C++ drop-in surface on a B200: vortexrt-gemma (reference flags and
report lines) over Gemma3Model, compared with the reference's own token loop
(oracle/_ref) or the C restatement."""

import os
import re
import subprocess

import numpy as np
import pytest

import oracle as O
import synth_gguf as sg
import vrt

pytestmark = pytest.mark.gpu
CLI = os.path.join(os.path.dirname(vrt.LIB_PATH), "vortexrt-gemma")


def run(*args):
    p = subprocess.run([CLI, *args], capture_output=True, text=True, errors="replace", timeout=600)
    assert p.returncode == 0, p.stderr
    assert "Validation: OK" in p.stdout
    return p.stdout


@pytest.fixture(scope="module")
def tiny(model_dir):
    return sg.cached_model(sg.SHAPES["tiny"], 1234, model_dir)


def test_cli_prompt_generation(tiny):
    out = run(tiny, "--prompt", "Hello world", "--generate", "12")
    assert "Layers: 6" in out and "TEXT_BEGIN" in out and "TEXT_END" in out
    prompt = [int(x) for x in re.search(r"Prompt token ids:(.*)", out).group(1).split()]
    gen = [int(x) for x in re.search(r"Generated token ids:(.*)", out).group(1).split()]
    o = O.Oracle(tiny)
    ref, margins = o.generate(prompt, 12, margins=True)
    if O.reference_available():
        r = O.Reference(tiny)
        assert r.tokenize("Hello world") == prompt
        assert r.generate(prompt, 12)[0] == ref
    for i, (a, b) in enumerate(zip(gen, ref)):
        if a != b:
            assert margins[i] < 1e-3
            break
    else:
        assert gen == ref


def test_cli_single_token_top_logits(tiny):
    out = run(tiny, "--token-id", "2", "--top-k", "8")
    assert "Top logits:" in out and "Final hidden checksum:" in out
    rows = re.findall(r"id=(\d+) logit=([-\d.e+]+)", out)
    o = O.Oracle(tiny)
    h, ids, lg = o.decode(2, 0, 8)
    got = np.array([float(v) for _, v in rows], np.float64)
    assert np.all(np.abs(got - lg) <= 1e-3 + 1e-3 * np.abs(lg))
    chk = float(re.search(r"Final hidden checksum: ([-\d.e+]+)", out).group(1))
    ref_chk = float(np.sum(h.astype(np.float64) * np.arange(1, h.size + 1)))
    assert abs(chk - ref_chk) <= 1e-3 * max(1.0, abs(ref_chk)) * h.size ** 0.5


def test_cli_prompt_ids_and_flags(tiny):
    out = run(tiny, "--prompt-ids", "2,300,301", "--generate", "4", "--q8-lanes", "8", "--projection-fusion", "off")
    assert "Prompt token ids: 2 300 301" in out
    assert "Narrow Q8 kernel: 8 lanes" in out and "Projection fusion: disabled" in out
    bad = subprocess.run([CLI, tiny, "--q8-lanes", "12"], capture_output=True, text=True)
    assert bad.returncode == 1 and "q8-lanes" in bad.stderr
