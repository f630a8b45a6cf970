"""Seeded synthetic Gemma 3 models written as GGUF v3 files.

The runtime loads Gemma 3 Q8_0 checkpoints the same way the Vortex-RT
reference does (`src/gemma3.cpp:72-654`: architecture check, config keys,
tokenizer arrays, per-layer tensor names, tied `token_embd.weight`).  No real
checkpoint is available offline, so every model used by the tests and the
benchmark is generated here from a counter-based hash:

* each tensor gets a 64-bit stream key from the seed and its name (FNV-1a),
* element ``i`` (row-major over the logical ``[rows][cols]`` matrix) draws
  ``h = splitmix64(key + i)``; the four 16-bit chunks of ``h`` are summed
  (Irwin-Hall of order 4, mean 131070, std 37837.2265) and scaled by one
  correctly-rounded fp32 multiply, so the value is bit-identical in numpy,
  C and CUDA;
* matrices are N(0, 0.02)-shaped and quantized to Q8_0 per 32-block:
  ``scale = absmax / 127`` (fp32), rounded to fp16 round-to-nearest-even,
  ``q = clamp(rint(v / fp16(scale)), -127, 127)``; an all-zero block uses
  scale 1 (the rule of the reference's FFN test, `src/ffn_test_main.cpp:183-200`);
* norm weights are ``1 + N(0, 0.1)`` in fp32: GGUF stores Gemma's folded
  ``(1 + w)`` RMSNorm weight, which the reference multiplies as stored
  (`src/gemma3.cpp:988-995`).

The same generator exists in CUDA (`vrt_model_create_synthetic`, which writes
the device arena directly, used for the 28.7 GB 27B-shaped benchmark model)
and in the C oracle; tests check all three agree bit for bit.
"""

from __future__ import annotations

import dataclasses
import os
import struct
from typing import Iterable

import numpy as np

M64 = (1 << 64) - 1
IH_MEAN = 131070
IH_STD = 37837.2265
GGML_F32 = 0
GGML_Q8_0 = 8

_GOLDEN = np.uint64(0x9E3779B97F4A7C15)
_MIX1 = np.uint64(0xBF58476D1CE4E5B9)
_MIX2 = np.uint64(0x94D049BB133111EB)
_KEYMUL = 0xD1B54A32D192ED03


@dataclasses.dataclass(frozen=True)
class Gemma3Shape:
    """Gemma 3 decoder dimensions (the fields of `Gemma3Config`, gemma3.hpp:19-33)."""

    name: str
    embedding_length: int
    block_count: int
    head_count: int
    head_count_kv: int
    head_dim: int
    feed_forward_length: int
    vocab_size: int
    sliding_window: int
    context_length: int
    rms_epsilon: float = 1e-6
    rope_freq_base: float = 1e6

    @property
    def q_width(self) -> int:
        return self.head_count * self.head_dim

    @property
    def kv_width(self) -> int:
        return self.head_count_kv * self.head_dim

    def with_(self, **kw) -> "Gemma3Shape":
        return dataclasses.replace(self, **kw)


# The synthetic configurations named by the benchmark plan.
SHAPES = {
    "tiny": Gemma3Shape("tiny", 128, 6, 4, 1, 64, 256, 768, 8, 256),
    "tiny-gqa": Gemma3Shape("tiny-gqa", 128, 6, 8, 2, 64, 256, 768, 8, 256),
    "270m": Gemma3Shape("270m", 640, 18, 4, 1, 256, 2048, 262144, 512, 32768),
    "27b": Gemma3Shape("27b", 5376, 62, 32, 16, 128, 21504, 262144, 1024, 131072),
}


def fnv1a64(text: str) -> int:
    h = 0xCBF29CE484222325
    for b in text.encode():
        h ^= b
        h = (h * 0x100000001B3) & M64
    return h


def _splitmix64_scalar(x: int) -> int:
    x = (x + 0x9E3779B97F4A7C15) & M64
    z = x
    z = ((z ^ (z >> 30)) * 0xBF58476D1CE4E5B9) & M64
    z = ((z ^ (z >> 27)) * 0x94D049BB133111EB) & M64
    return z ^ (z >> 31)


def stream_key(seed: int, tensor_name: str) -> int:
    return _splitmix64_scalar(
        (seed & M64) ^ (((fnv1a64(tensor_name) + 1) * _KEYMUL) & M64))


def _splitmix64(x: np.ndarray) -> np.ndarray:
    x = x + _GOLDEN
    z = (x ^ (x >> np.uint64(30))) * _MIX1
    z = (z ^ (z >> np.uint64(27))) * _MIX2
    return z ^ (z >> np.uint64(31))


def irwin_hall(key: int, start: int, count: int) -> np.ndarray:
    """Centred Irwin-Hall(4) integers for elements [start, start+count)."""
    idx = np.arange(count, dtype=np.uint64) + np.uint64((key + start) & M64)
    h = _splitmix64(idx)
    m = np.uint64(0xFFFF)
    s = (h & m) + ((h >> np.uint64(16)) & m) + ((h >> np.uint64(32)) & m) + (h >> np.uint64(48))
    return s.astype(np.int64) - IH_MEAN


def normal_values(key: int, start: int, count: int, std: float) -> np.ndarray:
    mult = np.float32(std / IH_STD)
    return irwin_hall(key, start, count).astype(np.float32) * mult


def norm_values(key: int, count: int, std: float = 0.1) -> np.ndarray:
    return np.float32(1.0) + normal_values(key, 0, count, std)


def quantize_q8_0(values: np.ndarray) -> np.ndarray:
    """Q8_0-encode a float32 array whose length is a multiple of 32 -> uint8 bytes."""
    v = values.reshape(-1, 32).astype(np.float32)
    amax = np.abs(v).max(axis=1)
    scale = np.where(amax == 0, np.float32(1.0), amax / np.float32(127.0)).astype(np.float32)
    half = scale.astype(np.float16)
    dq = half.astype(np.float32)
    q = np.clip(np.rint(v / dq[:, None]), -127, 127).astype(np.int8)
    out = np.empty((v.shape[0], 34), dtype=np.uint8)
    out[:, 0:2] = half.view(np.uint8).reshape(-1, 2)
    out[:, 2:] = q.view(np.uint8)
    return out.reshape(-1)


def q8_matrix_bytes(seed: int, name: str, rows: int, cols: int, std: float = 0.02,
                    row_start: int = 0, row_count: int | None = None) -> np.ndarray:
    """Q8_0 bytes of rows [row_start, row_start+row_count) of a synthetic matrix."""
    if cols % 32:
        raise ValueError("Q8_0 matrix columns must be a multiple of 32")
    if row_count is None:
        row_count = rows - row_start
    key = stream_key(seed, name)
    out = np.empty(row_count * (cols // 32) * 34, dtype=np.uint8)
    rows_per_chunk = max(1, (1 << 22) // cols)
    row_bytes = cols // 32 * 34
    for r0 in range(0, row_count, rows_per_chunk):
        nr = min(rows_per_chunk, row_count - r0)
        vals = normal_values(key, (row_start + r0) * cols, nr * cols, std)
        out[r0 * row_bytes:(r0 + nr) * row_bytes] = quantize_q8_0(vals)
    return out


def dequantize_q8_0(raw: np.ndarray, rows: int, cols: int) -> np.ndarray:
    blocks = raw.reshape(rows * (cols // 32), 34)
    d = blocks[:, 0:2].copy().view(np.float16).astype(np.float32).reshape(-1)
    q = blocks[:, 2:].copy().view(np.int8).astype(np.float32)
    return (q * d[:, None]).reshape(rows, cols)


# --------------------------------------------------------------------------
# Tokenizer vocabulary


def vocab_pieces(vocab_size: int) -> tuple[list[str], list[float], list[int]]:
    """Synthetic SentencePiece-style vocabulary.

    ids 0..3 are <pad>/<eos>/<bos>/<unk>, followed by the 256 byte pieces
    ``<0xHH>`` (type 6, used by the byte fallback of gemma3.cpp:354-379),
    some printable pieces (type 1), then ``<t%d>`` filler pieces (type 1).
    """
    if vocab_size < 260:
        raise ValueError("synthetic vocabulary needs at least 260 entries")
    toks = ["<pad>", "<eos>", "<bos>", "<unk>"]
    types = [3, 3, 3, 2]
    toks += ["<0x%02X>" % b for b in range(256)]
    types += [6] * 256
    marker = "▁"
    words = ["Hello", "world", "the", "and", "ing", "token", "Gemma", "B200", "is", "a"]
    extra = [marker] + [marker + w for w in words] + words
    extra += [chr(c) for c in range(33, 127)]
    extra += [marker + chr(c) for c in range(ord("a"), ord("z") + 1)]
    for p in extra:
        if len(toks) >= vocab_size:
            break
        toks.append(p)
        types.append(1)
    while len(toks) < vocab_size:
        toks.append("<t%d>" % len(toks))
        types.append(1)
    scores = [0.0] * 4 + [0.0] * 256 + [-0.01 * (i % 97) - 0.001 * len(toks[i])
                                        for i in range(260, vocab_size)]
    return toks, scores, types


# --------------------------------------------------------------------------
# GGUF v3 writer

_T_U32, _T_I32, _T_F32, _T_BOOL, _T_STRING, _T_ARRAY = 4, 5, 6, 7, 8, 9


def _gstr(s: str) -> bytes:
    b = s.encode()
    return struct.pack("<Q", len(b)) + b


def _kv(key: str, vtype: int, payload: bytes) -> bytes:
    return _gstr(key) + struct.pack("<I", vtype) + payload


def layer_tensors(shape: Gemma3Shape) -> list[tuple[str, int, list[int]]]:
    """(name, ggml_type, dims) of every tensor, in file order (gemma3.cpp:456-533)."""
    d, ff = shape.embedding_length, shape.feed_forward_length
    out: list[tuple[str, int, list[int]]] = [("token_embd.weight", GGML_Q8_0, [d, shape.vocab_size])]
    for layer in range(shape.block_count):
        p = "blk.%d." % layer
        out += [
            (p + "attn_norm.weight", GGML_F32, [d]),
            (p + "attn_q.weight", GGML_Q8_0, [d, shape.q_width]),
            (p + "attn_k.weight", GGML_Q8_0, [d, shape.kv_width]),
            (p + "attn_v.weight", GGML_Q8_0, [d, shape.kv_width]),
            (p + "attn_q_norm.weight", GGML_F32, [shape.head_dim]),
            (p + "attn_k_norm.weight", GGML_F32, [shape.head_dim]),
            (p + "attn_output.weight", GGML_Q8_0, [shape.q_width, d]),
            (p + "post_attention_norm.weight", GGML_F32, [d]),
            (p + "ffn_norm.weight", GGML_F32, [d]),
            (p + "ffn_gate.weight", GGML_Q8_0, [d, ff]),
            (p + "ffn_up.weight", GGML_Q8_0, [d, ff]),
            (p + "ffn_down.weight", GGML_Q8_0, [ff, d]),
            (p + "post_ffw_norm.weight", GGML_F32, [d]),
        ]
    out.append(("output_norm.weight", GGML_F32, [d]))
    return out


def tensor_nbytes(ggml_type: int, dims: Iterable[int]) -> int:
    n = 1
    for x in dims:
        n *= x
    return n * 4 if ggml_type == GGML_F32 else n // 32 * 34


def tensor_payload(seed: int, name: str, ggml_type: int, dims: list[int]) -> np.ndarray:
    if ggml_type == GGML_F32:
        return norm_values(stream_key(seed, name), dims[0]).view(np.uint8)
    return q8_matrix_bytes(seed, name, dims[1], dims[0])


def write_gguf(path: str | os.PathLike, shape: Gemma3Shape, seed: int = 1234,
               alignment: int = 32) -> dict:
    """Write a synthetic Gemma 3 Q8_0 GGUF; returns {name: (offset, nbytes)}."""
    toks, scores, types = vocab_pieces(shape.vocab_size)
    kvs = [
        _kv("general.architecture", _T_STRING, _gstr("gemma3")),
        _kv("general.alignment", _T_U32, struct.pack("<I", alignment)),
        _kv("gemma3.context_length", _T_U32, struct.pack("<I", shape.context_length)),
        _kv("gemma3.embedding_length", _T_U32, struct.pack("<I", shape.embedding_length)),
        _kv("gemma3.block_count", _T_U32, struct.pack("<I", shape.block_count)),
        _kv("gemma3.feed_forward_length", _T_U32, struct.pack("<I", shape.feed_forward_length)),
        _kv("gemma3.attention.head_count", _T_U32, struct.pack("<I", shape.head_count)),
        _kv("gemma3.attention.head_count_kv", _T_U32, struct.pack("<I", shape.head_count_kv)),
        _kv("gemma3.attention.key_length", _T_U32, struct.pack("<I", shape.head_dim)),
        _kv("gemma3.attention.value_length", _T_U32, struct.pack("<I", shape.head_dim)),
        _kv("gemma3.attention.layer_norm_rms_epsilon", _T_F32, struct.pack("<f", shape.rms_epsilon)),
        _kv("gemma3.attention.sliding_window", _T_U32, struct.pack("<I", shape.sliding_window)),
        _kv("gemma3.rope.freq_base", _T_F32, struct.pack("<f", shape.rope_freq_base)),
        _kv("tokenizer.ggml.model", _T_STRING, _gstr("llama")),
        _kv("tokenizer.ggml.tokens", _T_ARRAY,
            struct.pack("<IQ", _T_STRING, len(toks)) + b"".join(_gstr(t) for t in toks)),
        _kv("tokenizer.ggml.scores", _T_ARRAY,
            struct.pack("<IQ", _T_F32, len(scores)) + np.asarray(scores, np.float32).tobytes()),
        _kv("tokenizer.ggml.token_type", _T_ARRAY,
            struct.pack("<IQ", _T_I32, len(types)) + np.asarray(types, np.int32).tobytes()),
        _kv("tokenizer.ggml.bos_token_id", _T_U32, struct.pack("<I", 2)),
        _kv("tokenizer.ggml.eos_token_id", _T_U32, struct.pack("<I", 1)),
        _kv("tokenizer.ggml.unknown_token_id", _T_U32, struct.pack("<I", 3)),
        _kv("tokenizer.ggml.add_space_prefix", _T_BOOL, struct.pack("<B", 0)),
    ]
    tensors = layer_tensors(shape)
    layout = {}
    infos = []
    off = 0
    for name, t, dims in tensors:
        nb = tensor_nbytes(t, dims)
        layout[name] = (off, nb)
        infos.append(_gstr(name) + struct.pack("<I", len(dims)) +
                     b"".join(struct.pack("<Q", x) for x in dims) + struct.pack("<IQ", t, off))
        off += nb
        off = (off + alignment - 1) // alignment * alignment
    header = struct.pack("<IIQQ", 0x46554747, 3, len(tensors), len(kvs)) + b"".join(kvs) + b"".join(infos)
    pad = (-len(header)) % alignment
    with open(path, "wb") as f:
        f.write(header + b"\0" * pad)
        pos = 0
        for name, t, dims in tensors:
            o, nb = layout[name]
            if o > pos:
                f.write(b"\0" * (o - pos))
                pos = o
            payload = tensor_payload(seed, name, t, dims)
            assert payload.nbytes == nb
            f.write(payload.tobytes())
            pos += nb
        tail = (-pos) % alignment
        f.write(b"\0" * tail)
    return layout


def cached_model(shape: Gemma3Shape, seed: int = 1234, directory: str | None = None) -> str:
    """Path of a synthetic GGUF for (shape, seed), writing it once per directory."""
    directory = directory or os.environ.get("VRT_MODEL_CACHE", "/tmp/vrt_models")
    os.makedirs(directory, exist_ok=True)
    tag = "%s_d%d_l%d_h%d_kv%d_hd%d_ff%d_v%d_w%d_s%d" % (
        shape.name, shape.embedding_length, shape.block_count, shape.head_count,
        shape.head_count_kv, shape.head_dim, shape.feed_forward_length, shape.vocab_size,
        shape.sliding_window, seed)
    path = os.path.join(directory, tag + ".gguf")
    if not os.path.exists(path):
        tmp = path + ".%d.tmp" % os.getpid()
        write_gguf(tmp, shape, seed)
        os.replace(tmp, path)
    return path
