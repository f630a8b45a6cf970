"""TEST INFRASTRUCTURE -- ctypes front for the two CPU oracles.

* ``Oracle``: the C restatement of the Gemma 3 Q8_0 token loop
  (oracle/gemma3_oracle.c -> oracle/liboracle.so), generalised to grouped
  KV heads.
* ``Reference``: the reference's own src/gemma3.cpp + src/gguf.cpp compiled
  with the host shim (oracle/Makefile `ref` -> oracle/_ref/libvrt_ref.so).

Only tests/, ``__graft_entry__.smoke`` and bench.py's CPU-baseline leg use
this module, and only as the checker.  The product never imports it.
"""

from __future__ import annotations

import ctypes as C
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "liboracle.so")
REF_PATH = os.path.join(HERE, "_ref", "libvrt_ref.so")
# the reference tree: $VRT_REFERENCE_TREE, else the tree beside this repository
REF_SRC = os.environ.get("VRT_REFERENCE_TREE", os.path.join(os.path.dirname(HERE), "..", "reference"))

_f32p = np.ctypeslib.ndpointer(np.float32, flags="C_CONTIGUOUS")
_u32p = np.ctypeslib.ndpointer(np.uint32, flags="C_CONTIGUOUS")
_u8p = np.ctypeslib.ndpointer(np.uint8, flags="C_CONTIGUOUS")


def build(ref: bool = True) -> None:
    """Compile liboracle.so, and the reference build when its sources exist."""
    subprocess.run(["make", "-s", "-C", HERE], check=True)
    if ref and os.path.isdir(os.path.join(REF_SRC, "src")):
        subprocess.run(["make", "-s", "-C", HERE, "ref", "REF=" + REF_SRC], check=True)


def reference_available() -> bool:
    return os.path.exists(REF_PATH)


_lib = None


def lib() -> C.CDLL:
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            build(ref=False)
        L = C.CDLL(LIB_PATH)
        L.orc_stream_key.restype = C.c_uint64
        L.orc_stream_key.argtypes = [C.c_uint64, C.c_char_p]
        L.orc_synth_q8_rows.argtypes = [C.c_uint64, C.c_uint32, C.c_uint64, C.c_uint64, C.c_double, _u8p]
        L.orc_synth_norm.argtypes = [C.c_uint64, C.c_uint32, C.c_double, _f32p]
        L.orc_q8_matvec.argtypes = [_u8p, _f32p, _f32p, C.c_uint32, C.c_uint32, C.c_uint32, C.c_int]
        L.orc_gelu_mul.argtypes = [_f32p, _f32p, C.c_uint32]
        L.orc_argmax.argtypes = [_f32p, C.c_uint32, C.POINTER(C.c_uint32), C.POINTER(C.c_float)]
        L.orc_open.restype = C.c_void_p
        L.orc_open.argtypes = [C.c_char_p, C.c_uint32, C.c_uint32, C.c_int, C.c_int, C.c_uint32,
                               C.c_char_p, C.c_size_t]
        L.orc_open_synthetic.restype = C.c_void_p
        L.orc_open_synthetic.argtypes = [_u32p, C.c_float, C.c_float, C.c_uint64, C.c_uint32,
                                         C.c_uint32, C.c_int, C.c_int, C.c_uint32]
        L.orc_close.argtypes = [C.c_void_p]
        L.orc_error.restype = C.c_char_p
        L.orc_error.argtypes = [C.c_void_p]
        L.orc_set_threads.argtypes = [C.c_void_p, C.c_int]
        L.orc_set_trace.argtypes = [C.c_void_p, C.c_void_p]
        L.orc_config_get.argtypes = [C.c_void_p, _u32p, _f32p]
        L.orc_weight.restype = C.c_void_p
        L.orc_weight.argtypes = [C.c_void_p, C.c_char_p, C.c_uint32]
        L.orc_reset.argtypes = [C.c_void_p]
        L.orc_decode.argtypes = [C.c_void_p, C.c_uint32, C.c_uint32, C.c_uint32, C.c_void_p,
                                 C.c_void_p, C.c_void_p, C.POINTER(C.c_uint32), C.c_void_p]
        L.orc_generate.argtypes = [C.c_void_p, _u32p, C.c_uint32, C.c_uint32, _u32p,
                                   C.POINTER(C.c_uint32), C.c_void_p]
        _lib = L
    return _lib


def q8_matvec(raw: np.ndarray, x: np.ndarray, rows: int, lanes: int = 8, threads: int = 1) -> np.ndarray:
    """y = W x over raw Q8_0 rows.  lanes: shader lane count (8/16/32/64) or 0 = fp64 sequential."""
    x = np.ascontiguousarray(x, np.float32)
    y = np.zeros(rows, np.float32)
    lib().orc_q8_matvec(np.ascontiguousarray(raw, np.uint8), x, y, x.size, rows, lanes, threads)
    return y


def gelu_mul(gate: np.ndarray, up: np.ndarray) -> np.ndarray:
    g = np.array(gate, np.float32, copy=True)
    lib().orc_gelu_mul(g, np.ascontiguousarray(up, np.float32), g.size)
    return g


def argmax(v: np.ndarray) -> tuple[int, float]:
    i, val = C.c_uint32(), C.c_float()
    lib().orc_argmax(np.ascontiguousarray(v, np.float32), v.size, C.byref(i), C.byref(val))
    return i.value, val.value


def synth_q8(seed: int, name: str, rows: int, cols: int, r0: int = 0, nr: int | None = None) -> np.ndarray:
    nr = rows - r0 if nr is None else nr
    out = np.zeros(nr * (cols // 32) * 34, np.uint8)
    L = lib()
    L.orc_synth_q8_rows(L.orc_stream_key(seed, name.encode()), cols, r0, nr, 0.02, out)
    return out


def synth_norm(seed: int, name: str, n: int) -> np.ndarray:
    out = np.zeros(n, np.float32)
    L = lib()
    L.orc_synth_norm(L.orc_stream_key(seed, name.encode()), n, 0.1, out)
    return out


class Oracle:
    """The C restatement.  `subgroup`/`lanes`/`fusion` mirror the reference policy."""

    def __init__(self, path: str | None = None, *, shape=None, seed: int = 1234, subgroup: int = 8,
                 lanes: int = 0, fusion: int = -1, threads: int = 1, max_positions: int = 0):
        L = lib()
        if path is not None:
            err = C.create_string_buffer(512)
            self.h = L.orc_open(path.encode(), subgroup, lanes, fusion, threads, max_positions, err, 512)
            if not self.h:
                raise RuntimeError(err.value.decode())
        else:
            dims = np.array([shape.embedding_length, shape.block_count, shape.head_count,
                             shape.head_count_kv, shape.head_dim, shape.feed_forward_length,
                             shape.vocab_size, shape.sliding_window, shape.context_length], np.uint32)
            self.h = L.orc_open_synthetic(dims, shape.rms_epsilon, shape.rope_freq_base, seed, subgroup,
                                          lanes, fusion, threads, max_positions)
            if not self.h:
                raise RuntimeError("oracle synthetic model allocation failed")
        cfg, cf = np.zeros(10, np.uint32), np.zeros(3, np.float32)
        L.orc_config_get(self.h, cfg, cf)
        (self.context_length, self.d, self.L, self.ff, self.H, self.KV, self.hd, self.vd,
         self.vocab, self.window) = (int(v) for v in cfg)
        self.eps, self.theta_g, self.theta_l = (float(v) for v in cf)

    def close(self):
        if self.h:
            lib().orc_close(self.h)
            self.h = None

    __del__ = close

    def set_threads(self, n: int):
        lib().orc_set_threads(self.h, n)

    def reset(self):
        lib().orc_reset(self.h)

    def weight(self, what: str, layer: int = 0) -> int:
        return lib().orc_weight(self.h, what.encode(), layer)

    def decode(self, token: int, position: int, top_k: int = 1, full_logits: bool = False, trace=None):
        """Returns (hidden[d], ids, logits[, full_logits]) like Gemma3Model::decode_token."""
        hidden = np.zeros(self.d, np.float32)
        k = max(top_k, 1)
        ids = np.zeros(k, np.uint32)
        lg = np.zeros(k, np.float32)
        n = C.c_uint32()
        full = np.zeros(self.vocab, np.float32) if full_logits else None
        if trace is not None:
            lib().orc_set_trace(self.h, trace.ctypes.data)
        rc = lib().orc_decode(self.h, token, position, top_k, hidden.ctypes.data, ids.ctypes.data,
                              lg.ctypes.data, C.byref(n), full.ctypes.data if full is not None else None)
        if trace is not None:
            lib().orc_set_trace(self.h, None)
        if rc:
            raise RuntimeError(lib().orc_error(self.h).decode())
        out = (hidden, ids[:n.value].copy(), lg[:n.value].copy())
        return out + (full,) if full_logits else out

    def generate(self, prompt, max_new: int, margins: bool = False):
        p = np.ascontiguousarray(prompt, np.uint32)
        out = np.zeros(max(max_new, 1), np.uint32)
        n = C.c_uint32()
        mg = np.zeros(max(max_new, 1), np.float32) if margins else None
        rc = lib().orc_generate(self.h, p, p.size, max_new, out, C.byref(n),
                                mg.ctypes.data if mg is not None else None)
        if rc:
            raise RuntimeError(lib().orc_error(self.h).decode())
        ids = out[:n.value].tolist()
        return (ids, mg[:n.value].copy()) if margins else ids


_ref = None


def _reflib() -> C.CDLL:
    global _ref
    if _ref is None:
        L = C.CDLL(REF_PATH)
        L.vrt_ref_open.restype = C.c_void_p
        L.vrt_ref_open.argtypes = [C.c_char_p, C.c_uint, C.c_uint, C.c_int, C.c_uint, C.c_char_p, C.c_size_t]
        L.vrt_ref_close.argtypes = [C.c_void_p]
        L.vrt_ref_set_threads.argtypes = [C.c_void_p, C.c_uint]
        L.vrt_ref_config.argtypes = [C.c_void_p, _u32p, _f32p, _u32p]
        L.vrt_ref_reset.argtypes = [C.c_void_p]
        L.vrt_ref_decode.argtypes = [C.c_void_p, C.c_uint, C.c_uint, C.c_size_t, C.c_int, C.c_void_p,
                                     C.c_void_p, C.c_void_p, C.POINTER(C.c_size_t), C.c_char_p, C.c_size_t]
        L.vrt_ref_generate.argtypes = [C.c_void_p, _u32p, C.c_size_t, C.c_size_t, _u32p,
                                       C.POINTER(C.c_size_t), C.c_char_p, C.c_size_t, C.c_char_p, C.c_size_t]
        L.vrt_ref_tokenize.argtypes = [C.c_void_p, C.c_char_p, C.c_int, _u32p, C.c_size_t,
                                       C.POINTER(C.c_size_t), C.c_char_p, C.c_size_t]
        _ref = L
    return _ref


class Reference:
    """The reference's own Gemma3Model (src/gemma3.cpp) over the host shim."""

    def __init__(self, path: str, subgroup: int = 8, lanes: int = 0, fusion: int = -1, threads: int = 1):
        L = _reflib()
        err = C.create_string_buffer(1024)
        self.h = L.vrt_ref_open(path.encode(), subgroup, lanes, fusion, threads, err, 1024)
        if not self.h:
            raise RuntimeError(err.value.decode())
        cfg, cf, pol = np.zeros(10, np.uint32), np.zeros(3, np.float32), np.zeros(3, np.uint32)
        L.vrt_ref_config(self.h, cfg, cf, pol)
        (self.context_length, self.d, self.L, self.ff, self.H, self.KV, self.hd, self.vd,
         self.vocab, self.window) = (int(v) for v in cfg)
        self.eps, self.theta_g, self.theta_l = (float(v) for v in cf)
        self.narrow_lanes, self.fusion, self.fused_ffn = (int(v) for v in pol)

    def close(self):
        if self.h:
            _reflib().vrt_ref_close(self.h)
            self.h = None

    __del__ = close

    def set_threads(self, n: int):
        _reflib().vrt_ref_set_threads(self.h, n)

    def reset(self):
        _reflib().vrt_ref_reset(self.h)

    def decode(self, token: int, position: int, top_k: int = 1, single: bool = False):
        hidden = np.zeros(self.d, np.float32)
        k = max(top_k, 1)
        ids = np.zeros(k, np.uint32)
        lg = np.zeros(k, np.float32)
        n = C.c_size_t()
        err = C.create_string_buffer(1024)
        rc = _reflib().vrt_ref_decode(self.h, token, position, top_k, int(single), hidden.ctypes.data,
                                      ids.ctypes.data, lg.ctypes.data, C.byref(n), err, 1024)
        if rc:
            raise RuntimeError(err.value.decode())
        return hidden, ids[:n.value].copy(), lg[:n.value].copy()

    def generate(self, prompt, max_new: int):
        p = np.ascontiguousarray(prompt, np.uint32)
        out = np.zeros(max(max_new, 1), np.uint32)
        n = C.c_size_t()
        text = C.create_string_buffer(1 << 16)
        err = C.create_string_buffer(1024)
        rc = _reflib().vrt_ref_generate(self.h, p, p.size, max_new, out, C.byref(n), text, 1 << 16, err, 1024)
        if rc:
            raise RuntimeError(err.value.decode())
        return out[:n.value].tolist(), text.value

    def tokenize(self, text: str, add_bos: bool = True):
        out = np.zeros(4 * len(text.encode()) + 8, np.uint32)
        n = C.c_size_t()
        err = C.create_string_buffer(1024)
        rc = _reflib().vrt_ref_tokenize(self.h, text.encode(), int(add_bos), out, out.size, C.byref(n), err, 1024)
        if rc:
            raise RuntimeError(err.value.decode())
        return out[:n.value].tolist()
