"""The C-ABI library builds, loads and exports every function
include/vortexrt_b200.h declares; without a GPU, context creation fails with
an error code and a message instead of crashing.  No compute call here."""

import ctypes as C
import os
import subprocess

import pytest

import vrt


def test_library_exports_header():
    names = vrt.header_symbols()
    assert len(names) >= 40
    out = subprocess.run(["nm", "-D", "--defined-only", vrt.LIB_PATH], capture_output=True, text=True,
                         check=True).stdout
    exported = {line.split()[-1] for line in out.splitlines() if " T " in line}
    missing = [n for n in names if n not in exported]
    assert not missing, missing
    for n in names:
        assert n in vrt._SIGS, f"binding lacks {n}"


def test_version_and_error_without_device():
    L = vrt.lib()
    assert b"sm_100a" in L.vrt_version()
    try:
        import torch
        has_gpu = torch.cuda.is_available()
    except Exception:
        has_gpu = False
    if has_gpu:
        pytest.skip("a GPU is present")
    h = C.c_void_p()
    rc = L.vrt_ctx_create(0, C.byref(h))
    assert rc in (vrt.VRT_E_CUDA, vrt.VRT_E_INVALID)
    assert L.vrt_last_error()


def test_null_arguments_rejected_without_device():
    L = vrt.lib()
    assert L.vrt_q8_gemv(None, None, 0, 0, None, None, 32, 1, None) == vrt.VRT_E_INVALID
    assert L.vrt_model_reset(None) == vrt.VRT_E_INVALID
    assert L.vrt_decode_step(None, 0, 0, 1, None, None, None) == vrt.VRT_E_INVALID
    assert vrt.lib().vrt_q8t_bytes(257, 640) == 17 * 5 * 2176
