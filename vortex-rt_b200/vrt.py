"""ctypes binding of libvortexrt_b200.so (C ABI in include/vortexrt_b200.h).

The binding is a thin host-side layer for tests and the benchmark; every
computation happens in the CUDA library.  Importing this module never falls
back to anything: if the shared library is missing it raises, and every C
error code becomes a ``VrtError`` carrying ``vrt_last_error()``.
"""

from __future__ import annotations

import ctypes as C
import os
import subprocess
import sys
import weakref

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
# VRT_LIB: another build of the library (e.g. the timing build of `make stamps`)
LIB_PATH = os.environ.get("VRT_LIB") or os.path.join(HERE, "libvortexrt_b200.so")
HEADER = os.path.join(ROOT, "include", "vortexrt_b200.h")

VRT_OK, VRT_E_INVALID, VRT_E_CUDA, VRT_E_NOMEM, VRT_E_IO, VRT_E_STATE, VRT_E_NUMERIC, VRT_E_TIMEOUT, \
    VRT_E_UNSUPPORTED = 0, -1, -2, -3, -4, -5, -6, -7, -8


class VrtError(RuntimeError):
    def __init__(self, code: int, msg: str):
        super().__init__(f"[{code}] {msg}")
        self.code = code


def build() -> None:
    subprocess.run(["make", "-s", "-C", HERE], check=True)


class Gemma3Config(C.Structure):
    _fields_ = [(n, C.c_uint32) for n in (
        "context_length", "embedding_length", "block_count", "feed_forward_length", "head_count",
        "head_count_kv", "head_dim", "value_dim", "vocab_size", "sliding_window")] + [
        ("rms_epsilon", C.c_float), ("global_rope_base", C.c_float), ("local_rope_base", C.c_float)]

    @classmethod
    def from_shape(cls, s) -> "Gemma3Config":
        return cls(s.context_length, s.embedding_length, s.block_count, s.feed_forward_length, s.head_count,
                   s.head_count_kv, s.head_dim, s.head_dim, s.vocab_size, s.sliding_window,
                   s.rms_epsilon, s.rope_freq_base, 1e4)


class ModelOptions(C.Structure):
    _fields_ = [("max_positions", C.c_uint32), ("tp_rank", C.c_int), ("tp_world", C.c_int),
                ("nccl_id", C.c_void_p), ("use_graph", C.c_int), ("use_pdl", C.c_int),
                ("tp_exchange", C.c_int), ("tp_wait_ms", C.c_uint32), ("prefill_chunk", C.c_uint32),
                ("step_mode", C.c_int)]


class DeviceInfo(C.Structure):
    _fields_ = [("name", C.c_char * 256), ("device", C.c_int), ("sm_count", C.c_int), ("cc_major", C.c_int),
                ("cc_minor", C.c_int), ("warp_size", C.c_uint32), ("global_mem_bytes", C.c_uint64),
                ("l2_bytes", C.c_uint64)]


class TpShard(C.Structure):
    _fields_ = [(n, C.c_uint32) for n in ("q_head0", "q_heads", "kv_head0", "kv_heads", "ffn0", "ffn", "vocab0",
                                          "vocab")]


class ArgmaxResult(C.Structure):
    _fields_ = [("index", C.c_uint32), ("value", C.c_float)]


_lib = None
_vp, _u32, _u64, _i = C.c_void_p, C.c_uint32, C.c_uint64, C.c_int

_SIGS = {
    "vrt_last_error": (C.c_char_p, []),
    "vrt_version": (C.c_char_p, []),
    "vrt_ctx_create": (_i, [_i, C.POINTER(_vp)]),
    "vrt_ctx_destroy": (_i, [_vp]),
    "vrt_ctx_info": (_i, [_vp, C.POINTER(DeviceInfo)]),
    "vrt_ctx_synchronize": (_i, [_vp]),
    "vrt_ctx_stream": (_vp, [_vp]),
    "vrt_alloc": (_i, [_vp, C.c_size_t, C.POINTER(_vp)]),
    "vrt_free": (_i, [_vp, _vp]),
    "vrt_upload": (_i, [_vp, _vp, _vp, C.c_size_t]),
    "vrt_download": (_i, [_vp, _vp, _vp, C.c_size_t]),
    "vrt_upload_async": (_i, [_vp, _vp, _vp, C.c_size_t, _vp]),
    "vrt_download_async": (_i, [_vp, _vp, _vp, C.c_size_t, _vp]),
    "vrt_host_alloc_pinned": (_i, [C.c_size_t, C.POINTER(_vp)]),
    "vrt_host_free_pinned": (_i, [_vp]),
    "vrt_q8_gemv": (_i, [_vp, _vp, _u64, _u64, _vp, _vp, _u32, _u32, _vp]),
    "vrt_q8_gemv_multi": (_i, [_vp, _vp, _u64, _vp, _vp, _u32, _vp, _vp, _u32, _vp]),
    "vrt_q8_ffn": (_i, [_vp, _vp, _u64, _u64, _u64, _u64, _vp, _vp, _vp, _u32, _u32, _u32, _vp]),
    "vrt_q8_ffn_static": (_i, [_vp, _u64, _u64, _u64, _u64, _vp, _vp, _u32, _u32, _u32, _vp]),
    "vrt_gelu_mul": (_i, [_vp, _vp, _vp, _u32, _vp]),
    "vrt_pipeline_status": (_i, [_vp, C.POINTER(_u32)]),
    "vrt_argmax": (_i, [_vp, _vp, _u32, _vp, _vp]),
    "vrt_lm_head_argmax": (_i, [_vp, _vp, _u64, _u64, _vp, _u32, _u32, _vp, _vp, _vp]),
    "vrt_q8t_bytes": (_u64, [_u32, _u32]),
    "vrt_q8t_pack": (_i, [_vp, _vp, _u64, _u64, _u32, _u32, _vp, _vp]),
    "vrt_q8t_pack_pair": (_i, [_vp, _vp, _u64, _u64, _u64, _u32, _u32, _vp, _vp]),
    "vrt_q8t_gemv": (_i, [_vp, _vp, _u32, _u32, _vp, _vp, _vp]),
    "vrt_q8t_gate_up": (_i, [_vp, _vp, _u32, _u32, _vp, _vp, _vp]),
    "vrt_q8t_ffn": (_i, [_vp, _vp, _vp, _u32, _u32, _u32, _vp, _vp, _vp, _vp]),
    "vrt_q8t_lm_head_argmax": (_i, [_vp, _vp, _u32, _u32, _vp, _vp, _vp, _vp]),
    "vrt_q8t_gemm": (_i, [_vp, _vp, _u32, _u32, _vp, _u32, _vp, _vp]),
    "vrt_batch_create": (_i, [_vp, _u32, _u32, _i, _vp]),
    "vrt_batch_destroy": (_i, [_vp]),
    "vrt_batch_prefill": (_i, [_vp, _u32, _vp, _u32]),
    "vrt_batch_decode_steps": (_i, [_vp, _u32, _u32]),
    "vrt_batch_read": (_i, [_vp, _u32, _vp, _u32, _vp, _vp]),
    "vrt_batch_logits": (_i, [_vp, _u32, _vp]),
    "vrt_batch_last_ids": (_i, [_vp, _u32, _vp]),
    "vrt_q8t_gemm_gelu": (_i, [_vp, _vp, _u32, _u32, _vp, _u32, _vp, _vp]),
    "vrt_q8t_to_q8m": (_i, [_vp, _vp, _u32, _u32, _vp, _vp]),
    "vrt_q8m_gemm": (_i, [_vp, _vp, _u32, _u32, _vp, _u32, _vp, _vp]),
    "vrt_q8m_gemm_gelu": (_i, [_vp, _vp, _u32, _u32, _vp, _u32, _vp, _vp]),
    "vrt_model_options_default": (None, [C.POINTER(ModelOptions)]),
    "vrt_model_load": (_i, [_vp, C.c_char_p, C.POINTER(ModelOptions), C.POINTER(_vp)]),
    "vrt_model_create_synthetic": (_i, [_vp, C.POINTER(Gemma3Config), _u64, C.POINTER(ModelOptions),
                                        C.POINTER(_vp)]),
    "vrt_model_destroy": (_i, [_vp]),
    "vrt_model_config": (_i, [_vp, C.POINTER(Gemma3Config)]),
    "vrt_model_reset": (_i, [_vp]),
    "vrt_decode_step": (_i, [_vp, _u32, _u32, _u32, _vp, _vp, _vp]),
    "vrt_model_logits": (_i, [_vp, _vp]),
    "vrt_generate_greedy": (_i, [_vp, _vp, _u32, _u32, _vp, C.POINTER(_u32)]),
    "vrt_decode_steps_async": (_i, [_vp, _u32, _vp, _vp]),
    "vrt_prefill": (_i, [_vp, _vp, _u32]),
    "vrt_model_next_token": (_i, [_vp, C.POINTER(_u32), C.POINTER(_u32)]),
    "vrt_model_step_kernels": (_i, [_vp, C.POINTER(_u32)]),
    "vrt_model_device_status": (_i, [_vp, C.POINTER(_u32)]),
    "vrt_model_set_trace": (_i, [_vp, _i]),
    "vrt_model_trace": (_i, [_vp, _vp]),
    "vrt_model_time_kernel": (_i, [_vp, _u32, _u32, _u32, C.POINTER(C.c_float), C.POINTER(_u64)]),
    "vrt_tp_unique_id": (_i, [_vp]),
    "vrt_tp_plan": (_i, [C.POINTER(Gemma3Config), _i, _i, C.POINTER(TpShard)]),
    "vrt_tokenizer_open": (_i, [C.c_char_p, C.POINTER(_vp)]),
    "vrt_tokenizer_close": (None, [_vp]),
    "vrt_tokenize": (_i, [_vp, C.c_char_p, _i, _vp, C.c_size_t, C.POINTER(C.c_size_t)]),
    "vrt_token_piece": (_i, [_vp, _u32, _i, C.c_char_p, C.c_size_t, C.POINTER(C.c_size_t)]),
}


def lib() -> C.CDLL:
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise FileNotFoundError(
                f"{LIB_PATH} is not built; run `make -C {HERE}` (or __graft_entry__.build()). "
                "There is no CPU fallback.")
        L = C.CDLL(LIB_PATH)
        for name, (res, args) in _SIGS.items():
            f = getattr(L, name)
            f.restype = res
            f.argtypes = args
        _lib = L
    return _lib


def check(rc: int) -> int:
    if rc != VRT_OK:
        raise VrtError(rc, lib().vrt_last_error().decode())
    return rc


def _ptr(a: np.ndarray | None):
    return None if a is None else a.ctypes.data_as(C.c_void_p)


class Context:
    """One device (vrt_ctx_create)."""

    def __init__(self, device: int = 0):
        self.h = _vp()
        check(lib().vrt_ctx_create(device, C.byref(self.h)))
        self._bufs: list[int] = []
        self._children = weakref.WeakSet()  # models / batches: closed before the context

    def _adopt(self, obj):
        self._children.add(obj)

    def info(self) -> DeviceInfo:
        i = DeviceInfo()
        check(lib().vrt_ctx_info(self.h, C.byref(i)))
        return i

    @property
    def stream(self):
        return lib().vrt_ctx_stream(self.h)

    def sync(self):
        check(lib().vrt_ctx_synchronize(self.h))

    def alloc(self, nbytes: int) -> int:
        p = _vp()
        check(lib().vrt_alloc(self.h, int(nbytes), C.byref(p)))
        return p.value

    def free(self, p: int):
        check(lib().vrt_free(self.h, p))

    def upload(self, arr: np.ndarray) -> int:
        arr = np.ascontiguousarray(arr)
        p = self.alloc(max(arr.nbytes, 1))
        check(lib().vrt_upload(self.h, p, _ptr(arr), arr.nbytes))
        return p

    def download(self, p: int, count: int, dtype=np.float32) -> np.ndarray:
        out = np.empty(count, dtype)
        check(lib().vrt_download(self.h, _ptr(out), p, out.nbytes))
        return out

    def close(self):
        if self.h and not sys.is_finalizing():  # at interpreter exit the CUDA runtime may already be gone
            kids = list(self._children)
            for k in kids:  # batches before the models they decode with
                if isinstance(k, Batch):
                    k.close()
            for k in kids:
                k.close()
            lib().vrt_ctx_destroy(self.h)
            self.h = _vp()

    def __enter__(self):
        return self

    def __exit__(self, *a):
        self.close()


class Model:
    """A Gemma 3 model resident on one device (vrt_model_*)."""

    def __init__(self, ctx: Context, path: str | None = None, *, config: Gemma3Config | None = None,
                 seed: int = 1234, max_positions: int = 0, use_graph: bool = True, use_pdl: bool = True,
                 tp_rank: int = 0, tp_world: int = 1, nccl_id: bytes | None = None,
                 tp_exchange: str = "peer", tp_wait_ms: int = 0, prefill_chunk: int = 0,
                 step_mode: str = "launches"):
        self.ctx = ctx
        self.h = _vp()
        self._batches = weakref.WeakSet()
        ctx._adopt(self)
        o = ModelOptions()
        lib().vrt_model_options_default(C.byref(o))
        o.max_positions = max_positions
        o.use_graph = int(use_graph)
        o.use_pdl = int(use_pdl)
        o.tp_rank, o.tp_world = tp_rank, tp_world
        o.tp_exchange = {"peer": 0, "nccl": 1}[tp_exchange]
        o.tp_wait_ms = tp_wait_ms
        o.prefill_chunk = prefill_chunk
        o.step_mode = {"persistent": 0, "launches": 1}[step_mode]
        self._id = C.create_string_buffer(nccl_id, 128) if nccl_id else None
        o.nccl_id = C.cast(self._id, C.c_void_p) if self._id is not None else None
        self.h = _vp()
        if path is not None:
            check(lib().vrt_model_load(ctx.h, path.encode(), C.byref(o), C.byref(self.h)))
        else:
            check(lib().vrt_model_create_synthetic(ctx.h, C.byref(config), seed, C.byref(o), C.byref(self.h)))
        self.config = Gemma3Config()
        check(lib().vrt_model_config(self.h, C.byref(self.config)))

    def close(self):
        if self.h and not sys.is_finalizing():  # at interpreter exit the CUDA runtime may already be gone
            for b in list(self._batches):
                b.close()
            lib().vrt_model_destroy(self.h)
            self.h = _vp()

    __del__ = close

    def reset(self):
        check(lib().vrt_model_reset(self.h))

    def decode(self, token: int, position: int, top_k: int = 1, want_hidden: bool = True):
        d = self.config.embedding_length
        hidden = np.zeros(d, np.float32) if want_hidden else None
        k = max(top_k, 1)
        ids = np.zeros(k, np.uint32)
        lg = np.zeros(k, np.float32)
        check(lib().vrt_decode_step(self.h, token, position, top_k, _ptr(hidden), _ptr(ids), _ptr(lg)))
        n = min(top_k, self.config.vocab_size)
        return hidden, ids[:n].copy(), lg[:n].copy()

    def logits(self) -> np.ndarray:
        out = np.zeros(self.config.vocab_size, np.float32)
        check(lib().vrt_model_logits(self.h, _ptr(out)))
        return out

    def generate(self, prompt, max_new: int) -> list[int]:
        p = np.ascontiguousarray(prompt, np.uint32)
        out = np.zeros(max(max_new, 1), np.uint32)
        n = _u32()
        check(lib().vrt_generate_greedy(self.h, _ptr(p), p.size, max_new, _ptr(out), C.byref(n)))
        return out[:n.value].tolist()

    def prefill(self, prompt):
        p = np.ascontiguousarray(prompt, np.uint32)
        check(lib().vrt_prefill(self.h, _ptr(p), p.size))

    def decode_steps_async(self, steps: int, d_out: int | None = None, stream=None):
        check(lib().vrt_decode_steps_async(self.h, steps, d_out, stream))

    def next_token(self) -> tuple[int, int]:
        t, p = _u32(), _u32()
        check(lib().vrt_model_next_token(self.h, C.byref(t), C.byref(p)))
        return t.value, p.value

    def step_kernels(self) -> int:
        n = _u32()
        check(lib().vrt_model_step_kernels(self.h, C.byref(n)))
        return n.value

    def device_status(self) -> int:
        n = _u32()
        check(lib().vrt_model_device_status(self.h, C.byref(n)))
        return n.value

    def time_kernel(self, layer: int, which: int, iters: int = 20) -> tuple[float, int]:
        ms, nb = C.c_float(), _u64()
        check(lib().vrt_model_time_kernel(self.h, layer, which, iters, C.byref(ms), C.byref(nb)))
        return ms.value, nb.value

    def set_trace(self, on: bool):
        check(lib().vrt_model_set_trace(self.h, int(on)))

    def trace(self) -> np.ndarray:
        c = self.config
        out = np.zeros(c.block_count * c.embedding_length, np.float32)
        check(lib().vrt_model_trace(self.h, _ptr(out)))
        return out.reshape(c.block_count, c.embedding_length)


class Batch:
    """Independent sequences decoded together on one model (vrt_batch_*)."""

    def __init__(self, model: "Model", max_seqs: int, max_positions: int, keep_logits: bool = False):
        self.model = model
        self.h = _vp()
        model.ctx._adopt(self)
        model._batches.add(self)
        check(lib().vrt_batch_create(model.h, max_seqs, max_positions, int(keep_logits), C.byref(self.h)))

    def close(self):
        if self.h and not sys.is_finalizing():  # at interpreter exit the CUDA runtime may already be gone
            lib().vrt_batch_destroy(self.h)
            self.h = _vp()

    __del__ = close

    def prefill(self, seq: int, prompt):
        p = np.ascontiguousarray(prompt, np.uint32)
        check(lib().vrt_batch_prefill(self.h, seq, _ptr(p), p.size))

    def decode_steps(self, count: int, steps: int):
        check(lib().vrt_batch_decode_steps(self.h, count, steps))

    def read(self, seq: int, cap: int = 1 << 16) -> tuple[list[int], int]:
        out = np.zeros(max(cap, 1), np.uint32)
        n, pos = _u32(), _u32()
        check(lib().vrt_batch_read(self.h, seq, _ptr(out), cap, C.byref(n), C.byref(pos)))
        return out[:min(n.value, cap)].tolist(), pos.value

    def logits(self, seq: int) -> np.ndarray:
        out = np.zeros(self.model.config.vocab_size, np.float32)
        check(lib().vrt_batch_logits(self.h, seq, _ptr(out)))
        return out

    def last_ids(self, count: int, out: np.ndarray | None = None) -> np.ndarray:
        out = np.zeros(count, np.uint32) if out is None else out
        check(lib().vrt_batch_last_ids(self.h, count, _ptr(out)))
        return out


class Tokenizer:
    """Host tokenizer of a GGUF vocabulary (vrt_tokenizer_*; no GPU)."""

    def __init__(self, path: str):
        self.h = _vp()
        check(lib().vrt_tokenizer_open(path.encode(), C.byref(self.h)))

    def close(self):
        if self.h and not sys.is_finalizing():  # at interpreter exit the CUDA runtime may already be gone
            lib().vrt_tokenizer_close(self.h)
            self.h = _vp()

    __del__ = close

    def tokenize(self, text: str, add_bos: bool = True) -> list[int]:
        data = text.encode()
        out = np.zeros(4 * len(data) + 8, np.uint32)
        n = C.c_size_t()
        check(lib().vrt_tokenize(self.h, data, int(add_bos), _ptr(out), out.size, C.byref(n)))
        return out[:n.value].tolist()

    def piece(self, token: int, decoded: bool = False) -> bytes:
        buf = C.create_string_buffer(256)
        n = C.c_size_t()
        check(lib().vrt_token_piece(self.h, token, int(decoded), buf, 256, C.byref(n)))
        return buf.raw[:n.value]


def tp_plan(config: Gemma3Config, world: int, rank: int) -> TpShard:
    s = TpShard()
    check(lib().vrt_tp_plan(C.byref(config), world, rank, C.byref(s)))
    return s


def tp_unique_id() -> bytes:
    buf = C.create_string_buffer(128)
    check(lib().vrt_tp_unique_id(buf))
    return buf.raw


def header_symbols() -> list[str]:
    """Names of every function the C header declares (VRT_API)."""
    import re
    text = open(HEADER).read()
    return re.findall(r"VRT_API\s+[^;(]*?\b(vrt_\w+)\s*\(", text)
