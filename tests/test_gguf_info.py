"""vortexrt-gguf-info parity: the reference's GGUF probe (src/gguf_main.cpp:84-170)
built unmodified against this repository's GgufFile (include/vortexrt/gguf.hpp,
vortex-rt_b200/csrc/gguf.cpp) prints exactly what the same source prints when
built against the reference's own parser (src/gguf.cpp) -- header fields,
every metadata entry, every tensor, the Q8_0 count -- and fails the same way
(exit code and message) on an architecture mismatch, a missing file and a
truncated file.  Host code only: no GPU.  The binaries come from
tests/ref_callers/Makefile (built where the reference tree exists)."""

import os
import subprocess

import pytest

import synth_gguf as sg

BIN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "ref_callers", "_bin")
OURS = os.path.join(BIN, "vortexrt-gguf-info")
REF = os.path.join(BIN, "vortexrt-gguf-info-ref")


def _both(*args):
    if not (os.path.exists(OURS) and os.path.exists(REF)):
        pytest.skip("GGUF probes not built (the reference tree was absent when the repository was built)")
    a = subprocess.run([OURS, *args], capture_output=True, text=True, timeout=120)
    b = subprocess.run([REF, *args], capture_output=True, text=True, timeout=120)
    return a, b


def _same(a, b):
    assert a.returncode == b.returncode, (a.returncode, b.returncode, a.stderr, b.stderr)
    assert a.stdout == b.stdout
    assert a.stderr == b.stderr


@pytest.mark.parametrize("shape,seed", [("tiny", 1234), ("tiny-gqa", 4321)])
def test_gguf_info_matches_reference(model_dir, shape, seed):
    path = sg.cached_model(sg.SHAPES[shape], seed, model_dir)
    a, b = _both(path)
    _same(a, b)
    assert a.returncode == 0 and "Architecture: gemma3" in a.stdout


def test_gguf_info_errors_match_reference(model_dir, tmp_path):
    path = sg.cached_model(sg.SHAPES["tiny"], 1234, model_dir)
    _same(*_both(path, "--expect-arch", "llama"))        # architecture mismatch
    _same(*_both(str(tmp_path / "missing.gguf")))        # no such file
    raw = open(path, "rb").read()
    for cut in (3, 20, 2000, len(raw) // 2):             # truncated: header, metadata, tensor infos, data
        bad = tmp_path / f"cut{cut}.gguf"
        bad.write_bytes(raw[:cut])
        a, b = _both(str(bad))
        _same(a, b)
        assert a.returncode != 0 or cut == len(raw) // 2
