"""Regenerates the golden fixtures in tests/golden/ (run from the repo root:
``python tests/golden/make_golden.py``).

Fixtures and where their expected values come from:

q2k_gguf.npz
    Q2_K blocks (from the oracle's quantizer on seeded N(0, 0.02) weights,
    plus hand-made edge blocks) and their fp32 decoding by the third-party
    gguf-py 0.19.0 ``Q2_K.dequantize_blocks`` -- an implementation independent
    of this repository that pins the block layout (scales/mins nibbles, 2-bit
    packing order, fp16 d/dmin).

q3k_gguf.npz
    Q3_K blocks (random hmask/qs/scales bits with seeded positive fp16 d,
    plus an all-zero block and a block with every field at its extremes) and
    their fp32 decoding by gguf-py 0.19.0 ``Q3_K.dequantize_blocks`` -- pins
    the 6-bit scale packing, the high-bit mask order and the -4 offset.

q6k_gguf.npz
    Q6_K blocks (random ql/qh/scales bits with seeded positive fp16 d, plus an
    all-zero block and a block at the extremes) and their fp32 decoding by
    gguf-py 0.19.0 ``Q6_K.dequantize_blocks`` -- pins the nibble / 2-bit
    placement, the -32 offset and the signed 8-bit scales.

demo_linear.npz
    The reference example examples/demo_linear.c:16-34 (batch 2, 16 -> 16,
    inputs k%7-3 times 1/8, weights k%11-5 times 1/16, bias k%5-2 times 1/32).
    Every product and partial sum is an exact dyadic rational well inside
    fp32's precision, so the expected output is computed exactly with Python
    fractions and holds for any summation order.

lcg.npz
    The reference benches' LCG data (bench_sme_full_timing.c:33-51) for the
    Linear case seeds 1001/1002/1003, generated here by a pure-Python
    restatement of the generator (fp16 rounding by numpy).
"""
from __future__ import annotations

import os
import sys
from fractions import Fraction

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.abspath(os.path.join(HERE, "..", "..")))

from oracle import oracle as O  # noqa: E402


def lcg_py(count: int, seed: int) -> np.ndarray:
    s = seed
    out = np.empty(count, np.float32)
    for i in range(count):
        s = (s * 1664525 + 1013904223) & 0xFFFFFFFF
        out[i] = np.float32(np.float32(s % 2001) / np.float32(2000.0)) - np.float32(0.5)
    return out


def make_q2k():
    from gguf.quants import Q2_K
    rng = np.random.default_rng(20240601)
    w = (rng.standard_normal(4 * 4096) * 0.02).astype(np.float32)
    blocks = O.quantize_q2_K(w).view(np.uint8).reshape(-1, 84).copy()
    # edge blocks: all-zero; all 2-bit codes 3 with max scales/mins; random bytes
    zero = np.zeros((1, 84), np.uint8)
    full = np.zeros((1, 84), np.uint8)
    full[0, :16] = 0xFF
    full[0, 16:80] = 0xFF
    full[0, 80:82] = np.frombuffer(np.float16(0.5).tobytes(), np.uint8)
    full[0, 82:84] = np.frombuffer(np.float16(0.25).tobytes(), np.uint8)
    rnd = rng.integers(0, 256, size=(6, 84), dtype=np.uint8)
    for r in rnd:  # keep d/dmin finite and moderate
        r[80:82] = np.frombuffer(np.float16(rng.uniform(1e-3, 1e-1)).tobytes(), np.uint8)
        r[82:84] = np.frombuffer(np.float16(rng.uniform(1e-3, 1e-1)).tobytes(), np.uint8)
    blocks = np.concatenate([blocks, zero, full, rnd], axis=0)
    deq = Q2_K.dequantize_blocks(blocks).astype(np.float32).reshape(-1)
    np.savez_compressed(os.path.join(HERE, "q2k_gguf.npz"), blocks=blocks, dequant=deq, source=np.array(w))


def make_q3k():
    from gguf.quants import Q3_K
    rng = np.random.default_rng(20240602)
    blocks = O.random_q3_K(rng, 64).view(np.uint8).reshape(-1, 110).copy()
    zero = np.zeros((1, 110), np.uint8)
    ext = np.zeros((1, 110), np.uint8)
    ext[0, :32] = 0x00          # every high bit clear: q = low bits - 4
    ext[0, 32:96] = 0xFF        # low bits 3
    ext[0, 96:104] = np.array([0x00, 0xFF, 0x0F, 0xF0] * 2, np.uint8)
    ext[0, 104:108] = np.array([0x00, 0xFF, 0x1B, 0xE4], np.uint8)
    ext[0, 108:110] = np.frombuffer(np.float16(0.125).tobytes(), np.uint8)
    blocks = np.concatenate([blocks, zero, ext], axis=0)
    deq = Q3_K.dequantize_blocks(blocks).astype(np.float32).reshape(-1)
    np.savez_compressed(os.path.join(HERE, "q3k_gguf.npz"), blocks=blocks, dequant=deq)


def make_q6k():
    from gguf.quants import Q6_K
    rng = np.random.default_rng(20240603)
    blocks = O.random_q6_K(rng, 64).view(np.uint8).reshape(-1, 210).copy()
    zero = np.zeros((1, 210), np.uint8)
    ext = np.zeros((1, 210), np.uint8)
    ext[0, :128] = np.tile(np.array([0x0F, 0xF0, 0xFF, 0x00], np.uint8), 32)
    ext[0, 128:192] = np.tile(np.array([0xFF, 0x00, 0x1B, 0xE4], np.uint8), 16)
    ext[0, 192:208] = np.array([127, -128, -1, 0, 1, 64, -64, 3] * 2, np.int8).view(np.uint8)
    ext[0, 208:210] = np.frombuffer(np.float16(0.0625).tobytes(), np.uint8)
    blocks = np.concatenate([blocks, zero, ext], axis=0)
    deq = Q6_K.dequantize_blocks(blocks).astype(np.float32).reshape(-1)
    np.savez_compressed(os.path.join(HERE, "q6k_gguf.npz"), blocks=blocks, dequant=deq)


def make_demo_linear():
    B, K, N = 2, 16, 16
    x = np.array([((i % 7) - 3) * 0.125 for i in range(B * K)], np.float32)
    w = np.array([((i % 11) - 5) * 0.0625 for i in range(K * N)], np.float32)
    b = np.array([((i % 5) - 2) * 0.03125 for i in range(N)], np.float32)
    out = np.empty((B, N), np.float32)
    for r in range(B):
        for c in range(N):
            acc = sum(Fraction(float(x[r * K + k])) * Fraction(float(w[k * N + c])) for k in range(K))
            acc += Fraction(float(b[c]))
            out[r, c] = float(acc)
            assert Fraction(float(out[r, c])) == acc  # exactly representable
    np.savez_compressed(os.path.join(HERE, "demo_linear.npz"), x16=x.astype(np.float16).view(np.uint16),
                        w16=w.astype(np.float16).view(np.uint16), bias=b, expected=out)


def make_lcg():
    arrays = {}
    for seed, count in ((1001, 8 * 128), (1002, 128 * 128), (1003, 128)):
        v = lcg_py(count, seed)
        arrays[f"f32_{seed}"] = v
        arrays[f"f16_{seed}"] = v.astype(np.float16).view(np.uint16)
    np.savez_compressed(os.path.join(HERE, "lcg.npz"), **arrays)


if __name__ == "__main__":
    O.build()
    make_q2k()
    make_q3k()
    make_q6k()
    make_demo_linear()
    make_lcg()
    print("fixtures written to", HERE)
