"""Known-answer inputs restated from the reference's own test programs.

* q8_test: src/q8_test_main.cpp:80-131 -- 640 x 257 Q8_0 matrix, weights
  0.5 cos(0.017 (13 row + 32 block + k)), input 0.75 sin(0.031 i), scale
  absmax/127 rounded to fp16 by the test's round-half-up converter,
  q = nearbyint(v / scale) (the unrounded scale), fp32 reference sum in
  row/block/k order.  Tolerance 2e-3 (q8_test_main.cpp:311-317).
* ffn_test: src/ffn_test_main.cpp:112-250 -- gate/up 64 -> 96, down 96 -> 64,
  values sin/cos of phase(seed, row, col), q = nearbyint(v / fp16 scale),
  fp64 reference mat-vec, gelu_tanh * up.  Tolerance 5e-3 (437-441).
* gelu_test: src/gelu_test_main.cpp:34-56 -- 4096 elements, gate 5 sin(0.0137 i),
  up 3 cos(0.0211 i).  Tolerance 5e-5 (135-138).
All arithmetic is fp32 numpy with one rounding per operation, as in C++.
"""

import math
import struct

import numpy as np

f32 = np.float32


def f32_to_f16_roundup(f: float) -> int:
    """The reference tests' float -> half converter (q8_test_main.cpp:18-41)."""
    x = struct.unpack("<I", struct.pack("<f", f))[0]
    sign = (x >> 16) & 0x8000
    mant = x & 0x7FFFFF
    exp = ((x >> 23) & 0xFF) - 127 + 15
    if exp <= 0:
        if exp < -10:
            return sign
        mant = (mant | 0x800000) >> (1 - exp)
        return (sign + ((mant + 0x1000) >> 13)) & 0xFFFF
    if exp >= 31:
        return sign | 0x7C00
    return (sign | (exp << 10) | ((mant + 0x1000) >> 13)) & 0xFFFF


def f16_bits_to_f32(h: int) -> float:
    return float(np.array([h], np.uint16).view(np.float16)[0])


def q8_test_case():
    n_in, n_out = 640, 257
    blocks = n_in // 32
    x = np.array([f32(math.sin(f32(i) * f32(0.031))) * f32(0.75) for i in range(n_in)], np.float32)
    raw = bytearray(n_out * blocks * 34)
    ref = np.zeros(n_out, np.float32)
    for row in range(n_out):
        acc = f32(0.0)
        for b in range(blocks):
            vals = [f32(math.cos(f32(row * 13 + b * 32 + k) * f32(0.017))) * f32(0.5) for k in range(32)]
            amax = max(abs(v) for v in vals)
            scale = f32(amax / f32(127.0))
            h = f32_to_f16_roundup(float(scale))
            dq = f32(f16_bits_to_f32(h))
            base = (row * blocks + b) * 34
            raw[base:base + 2] = struct.pack("<H", h)
            for k in range(32):
                q = int(np.clip(np.rint(f32(vals[k] / scale)), -127, 127))
                raw[base + 2 + k] = q & 0xFF
                acc = f32(acc + f32(f32(dq * f32(q)) * x[b * 32 + k]))
        ref[row] = acc
    return np.frombuffer(bytes(raw), np.uint8).copy(), x, ref, n_in, n_out


def _ffn_matrix(seed: int, n_in: int, n_out: int):
    blocks = n_in // 32
    raw = bytearray()
    deq = np.zeros((n_out, n_in), np.float32)
    for row in range(n_out):
        for b in range(blocks):
            vals = []
            for k in range(32):
                col = b * 32 + k
                ph = f32(seed * 97 + row * 131 + col * 17)
                vals.append(f32(f32(math.sin(f32(ph * f32(0.0031)))) * f32(0.45)) +
                            f32(f32(math.cos(f32(ph * f32(0.0017)))) * f32(0.15)))
            amax = max(abs(v) for v in vals)
            scale = f32(1.0) if amax == 0 else f32(amax / f32(127.0))
            h = f32_to_f16_roundup(float(scale))
            dq = f32(f16_bits_to_f32(h))
            raw += struct.pack("<H", h)
            for k in range(32):
                q = int(np.clip(np.rint(f32(vals[k] / dq)), -127, 127))
                raw.append(q & 0xFF)
                deq[row, b * 32 + k] = f32(dq * f32(q))
    return bytes(raw), deq


def ffn_test_case():
    """Returns (raw bytes, offsets (gate, up, down), x, reference) -- ffn_test_main.cpp:254-307."""
    n_in, n_ffn, n_out = 64, 96, 64
    enc = bytearray()
    offs = []
    mats = []
    for seed, (ni, no) in zip((1, 2, 3), ((n_in, n_ffn), (n_in, n_ffn), (n_ffn, n_out))):
        while len(enc) % 4:
            enc.append(0)
        offs.append(len(enc))
        r, dq = _ffn_matrix(seed, ni, no)
        enc += r
        mats.append(dq)
    while len(enc) % 4:
        enc.append(0)
    x = np.array([f32(f32(math.sin(f32(i) * f32(0.071))) * f32(0.8)) for i in range(n_in)], np.float32)

    def matvec(dq, v):
        return (dq.astype(np.float64) @ v.astype(np.float64)).astype(np.float32)

    g = matvec(mats[0], x)
    u = matvec(mats[1], x)
    act = np.array([gelu_tanh_f32(a) * b for a, b in zip(g, u)], np.float32)
    ref = matvec(mats[2], act)
    return np.frombuffer(bytes(enc), np.uint8).copy(), offs, x, ref, (n_in, n_ffn, n_out)


def gelu_tanh_f32(x) -> np.float32:
    x = f32(x)
    x3 = f32(f32(x * x) * x)
    inner = f32(f32(0.7978845608028654) * f32(x + f32(f32(0.044715) * x3)))
    return f32(f32(f32(0.5) * x) * f32(f32(1.0) + f32(math.tanh(inner))))


def gelu_test_case():
    n = 4096
    gate = np.array([f32(f32(math.sin(f32(i) * f32(0.0137))) * f32(5.0)) for i in range(n)], np.float32)
    up = np.array([f32(f32(math.cos(f32(i) * f32(0.0211))) * f32(3.0)) for i in range(n)], np.float32)
    ref = np.array([f32(gelu_tanh_f32(g) * u) for g, u in zip(gate, up)], np.float32)
    return gate, up, ref
