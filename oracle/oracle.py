"""ctypes view of the CPU oracle (oracle/smeai_oracle.c).

TEST INFRASTRUCTURE ONLY: imported by tests/ and ``__graft_entry__.smoke()`` for
the expected results, and timed by the CPU-baseline leg of ``bench.py``.  The
product library never imports it.

Arrays are numpy; Q2_K / Q8_K blocks are structured numpy arrays whose byte
layout equals ggml's block_q2_K (84 B) and block_q8_K (292 B).
"""
from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "_build", "libsmeai_oracle.so")

QK_K = 256
BLOCK_Q2_K = np.dtype([("scales", np.uint8, 16), ("qs", np.uint8, 64),
                       ("d", np.uint16), ("dmin", np.uint16)])
BLOCK_Q3_K = np.dtype([("hmask", np.uint8, 32), ("qs", np.uint8, 64), ("scales", np.uint8, 12),
                       ("d", np.uint16)])
BLOCK_Q6_K = np.dtype([("ql", np.uint8, 128), ("qh", np.uint8, 64), ("scales", np.int8, 16), ("d", np.uint16)])
BLOCK_Q8_K = np.dtype([("d", np.float32), ("qs", np.int8, 256), ("bsums", np.int16, 16)])
assert BLOCK_Q2_K.itemsize == 84 and BLOCK_Q3_K.itemsize == 110 and BLOCK_Q6_K.itemsize == 210
assert BLOCK_Q8_K.itemsize == 292

ROUND_FUSED, ROUND_SEPARATE = 0, 1
COMBINE_FUSED, COMBINE_SEPARATE = 0, 1
Q3K_GGML, Q3K_BLOCK_ORDER = 0, 1
ACT_NONE, ACT_RELU, ACT_GELU, ACT_SILU = 0, 1, 2, 3

NATIVE_PATH = os.path.join(HERE, "_build", "native", "libsmeai_oracle.so")
NATIVE_CPU = os.path.join(HERE, "_build", "native", "cpu.txt")

_libs = {}
_native = False


def cpu_model() -> str:
    try:
        for line in open("/proc/cpuinfo"):
            if line.startswith("model name"):
                return line.split(":", 1)[1].strip()
    except OSError:
        pass
    return "unknown"


def build() -> str:
    """Compile the oracle with its Makefile (gcc) if the library is missing or stale."""
    src = os.path.join(HERE, "smeai_oracle.c")
    if (not os.path.exists(LIB_PATH)) or os.path.getmtime(LIB_PATH) < os.path.getmtime(src):
        subprocess.run(["make", "-C", HERE, "-s"], check=True)
    return LIB_PATH


def build_native() -> str:
    """The CPU-baseline copy compiled with -march=native on THIS host (rebuilt
    when the source changed or the host's CPU model differs from the one it
    was built on)."""
    src = os.path.join(HERE, "smeai_oracle.c")
    model = cpu_model()
    stale = (not os.path.exists(NATIVE_PATH)) or os.path.getmtime(NATIVE_PATH) < os.path.getmtime(src)
    try:
        stale = stale or open(NATIVE_CPU).read().strip() != model
    except OSError:
        stale = True
    if stale:
        subprocess.run(["make", "-C", HERE, "-s", "native"], check=True)
        with open(NATIVE_CPU, "w") as f:
            f.write(model + "\n")
    return NATIVE_PATH


def select(native: bool) -> None:
    """Route the wrappers below to the -march=native build (the CPU baseline)
    or to the portable build (the tests)."""
    global _native
    if native:
        build_native()
    _native = bool(native)


def lib() -> ctypes.CDLL:
    path = NATIVE_PATH if _native else LIB_PATH
    if path not in _libs:
        if not os.path.exists(path):
            build_native() if _native else build()
        L = ctypes.CDLL(path)
        P, U64, I64, I = ctypes.c_void_p, ctypes.c_uint64, ctypes.c_int64, ctypes.c_int
        F = ctypes.c_float
        sig = {
            "orc_lcg_fill_f16": (None, [P, U64, ctypes.c_uint32]),
            "orc_lcg_fill_f32": (None, [P, U64, ctypes.c_uint32]),
            "orc_linear_f16f32": (I, [P, U64, U64, P, U64, P, P, I]),
            "orc_linear_f32f32": (I, [P, U64, U64, P, U64, P, P, I]),
            "orc_mlp_f16f32": (I, [P, U64, U64, P, U64, P, P, U64, P, P, I]),
            "orc_swiglu_f16f32": (I, [P, U64, U64, P, U64, P, P, P, P, U64, P, P]),
            "orc_pack_weight_f16_tiles": (None, [P, P, U64, U64]),
            "orc_self_attention_f16f32": (I, [P, U64, U64, U64, P, P, P, P, P, P, P, P, I, P, P]),
            "orc_quantize_row_q8_K": (None, [P, P, I64, I]),
            "orc_quantize_row_q2_K": (None, [P, P, I64]),
            "orc_dequantize_row_q2_K": (None, [P, P, I64]),
            "orc_q2k_block_sums": (None, [I, P, P, P, P]),
            "orc_vec_dot_q2_K_q8_K": (F, [I, P, P, I]),
            "orc_q2k_mul_mat": (None, [P, I64, I64, P, I64, P, I64, I, I]),
            "orc_q3k_scales": (None, [P, P]),
            "orc_dequantize_row_q3_K": (None, [P, P, I64]),
            "orc_q3k_block_sums": (None, [I, P, P, P]),
            "orc_vec_dot_q3_K_q8_K": (F, [I, P, P, I]),
            "orc_q3k_mul_mat": (None, [P, I64, I64, P, I64, P, I64, I, I]),
            "orc_dequantize_row_q6_K": (None, [P, P, I64]),
            "orc_q6k_block_sums": (None, [I, P, P, P]),
            "orc_vec_dot_q6_K_q8_K": (F, [I, P, P, I]),
            "orc_q6k_mul_mat": (None, [P, I64, I64, P, I64, P, I64, I, I]),
            "orc_rms_inv": (F, [P, I64, F]),
            "orc_rms_sumsq": (F, [P, I64]),
            "orc_rmsnorm_quantize_q8_K": (None, [P, P, I64, F, I]),
            "orc_rmsnorm_w_quantize_q8_K": (None, [P, P, P, I64, F, I]),
            "orc_silu_mul": (None, [P, P, P, I64]),
        }
        for name, (res, args) in sig.items():
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _libs[path] = L
    return _libs[path]


def _p(a: np.ndarray):
    assert a.flags["C_CONTIGUOUS"]
    return a.ctypes.data


# ---------------------------------------------------------------- generators
def lcg_f16(count: int, seed: int) -> np.ndarray:
    out = np.empty(count, np.uint16)
    lib().orc_lcg_fill_f16(_p(out), count, seed)
    return out


def lcg_f32(count: int, seed: int) -> np.ndarray:
    out = np.empty(count, np.float32)
    lib().orc_lcg_fill_f32(_p(out), count, seed)
    return out


# ---------------------------------------------------------------- Path A
def linear_f16f32(x16, batch, k, w16, n, bias=None, act=ACT_NONE):
    out = np.empty(batch * n, np.float32)
    rc = lib().orc_linear_f16f32(_p(x16), batch, k, _p(w16), n,
                                 None if bias is None else _p(bias), _p(out), act)
    assert rc == 0
    return out.reshape(batch, n)


def linear_f32f32(x, batch, k, w, n, bias=None, act=ACT_NONE):
    out = np.empty(batch * n, np.float32)
    rc = lib().orc_linear_f32f32(_p(x), batch, k, _p(w), n,
                                 None if bias is None else _p(bias), _p(out), act)
    assert rc == 0
    return out.reshape(batch, n)


def mlp_f16f32(x16, batch, k, w1, hidden, b1, w2, n, b2, act):
    out = np.empty(batch * n, np.float32)
    rc = lib().orc_mlp_f16f32(_p(x16), batch, k, _p(w1), hidden, None if b1 is None else _p(b1),
                              _p(w2), n, None if b2 is None else _p(b2), _p(out), act)
    assert rc == 0
    return out.reshape(batch, n)


def swiglu_f16f32(x16, batch, k, wg, hidden, bg, wu, bu, wd, n, bd):
    out = np.empty(batch * n, np.float32)
    nz = lambda a: None if a is None else _p(a)
    rc = lib().orc_swiglu_f16f32(_p(x16), batch, k, _p(wg), hidden, nz(bg), _p(wu), nz(bu),
                                 _p(wd), n, nz(bd), _p(out))
    assert rc == 0
    return out.reshape(batch, n)


def self_attention_f16f32(x16, seq_len, model_dim, num_heads, wq, bq, wk, bk, wv, bv, wo, bo, causal,
                          with_context=False):
    """sme_ai_self_attention_ref_f16f32; with_context also returns the fp16 context."""
    out = np.empty(seq_len * model_dim, np.float32)
    ctx = np.empty(seq_len * model_dim, np.uint16)
    nz = lambda a: None if a is None else _p(a)
    rc = lib().orc_self_attention_f16f32(_p(x16), seq_len, model_dim, num_heads, _p(wq), nz(bq), _p(wk), nz(bk),
                                         _p(wv), nz(bv), _p(wo), nz(bo), int(causal), _p(out), _p(ctx))
    assert rc == 0
    out = out.reshape(seq_len, model_dim)
    return (out, ctx.reshape(seq_len, model_dim)) if with_context else out


def pack_weight_f16_tiles(w16, k, n):
    kp, np_ = (k + 15) // 16 * 16, (n + 15) // 16 * 16
    out = np.empty(kp * np_, np.float32)
    lib().orc_pack_weight_f16_tiles(_p(w16), _p(out), k, n)
    return out


# ---------------------------------------------------------------- Path B
def quantize_q8_K(x: np.ndarray, rounding=ROUND_FUSED) -> np.ndarray:
    x = np.ascontiguousarray(x, np.float32)
    assert x.size % QK_K == 0
    out = np.zeros(x.size // QK_K, BLOCK_Q8_K)
    lib().orc_quantize_row_q8_K(_p(x), _p(out), x.size, rounding)
    return out


def quantize_q2_K(x: np.ndarray) -> np.ndarray:
    x = np.ascontiguousarray(x, np.float32)
    assert x.size % QK_K == 0
    out = np.zeros(x.size // QK_K, BLOCK_Q2_K)
    lib().orc_quantize_row_q2_K(_p(x), _p(out), x.size)
    return out


def dequantize_q2_K(blocks: np.ndarray) -> np.ndarray:
    blocks = np.ascontiguousarray(blocks)
    out = np.empty(blocks.size * QK_K, np.float32)
    lib().orc_dequantize_row_q2_K(_p(blocks), _p(out), out.size)
    return out


def q2k_block_sums(wrow: np.ndarray, xq: np.ndarray):
    wrow, xq = np.ascontiguousarray(wrow), np.ascontiguousarray(xq)
    nb = wrow.size
    isum = np.empty(nb, np.int32)
    summs = np.empty(nb, np.int32)
    lib().orc_q2k_block_sums(nb * QK_K, _p(wrow), _p(xq), _p(isum), _p(summs))
    return isum, summs


def vec_dot_q2_K_q8_K(wrow, xq, combine=COMBINE_FUSED) -> float:
    wrow, xq = np.ascontiguousarray(wrow), np.ascontiguousarray(xq)
    return lib().orc_vec_dot_q2_K_q8_K(wrow.size * QK_K, _p(wrow), _p(xq), combine)


def random_q3_K(rng, n_blocks: int) -> np.ndarray:
    """Valid Q3_K blocks of random bits (every bit pattern of hmask, qs and
    scales is a valid block) with d a positive normal fp16 of the magnitude a
    quantized N(0, 0.02) weight has (parity is defined on identical blocks,
    so the quantizer's search is not needed)."""
    b = rng.integers(0, 256, size=(n_blocks, 110), dtype=np.uint8)
    d = (np.abs(rng.standard_normal(n_blocks)) * 0.0005 + 1e-5).astype(np.float16)
    b[:, 108:110] = d.view(np.uint8).reshape(-1, 2)
    return b.reshape(-1).view(BLOCK_Q3_K)


def q3k_scales(block) -> np.ndarray:
    block = np.ascontiguousarray(np.asarray(block).reshape(1))
    out = np.empty(16, np.int8)
    lib().orc_q3k_scales(_p(block), _p(out))
    return out


def dequantize_q3_K(blocks: np.ndarray) -> np.ndarray:
    blocks = np.ascontiguousarray(blocks)
    out = np.empty(blocks.size * QK_K, np.float32)
    lib().orc_dequantize_row_q3_K(_p(blocks), _p(out), out.size)
    return out


def q3k_block_sums(wrow: np.ndarray, xq: np.ndarray) -> np.ndarray:
    wrow, xq = np.ascontiguousarray(wrow), np.ascontiguousarray(xq)
    isum = np.empty(wrow.size, np.int32)
    lib().orc_q3k_block_sums(wrow.size * QK_K, _p(wrow), _p(xq), _p(isum))
    return isum


def vec_dot_q3_K_q8_K(wrow, xq, order=Q3K_GGML) -> float:
    wrow, xq = np.ascontiguousarray(wrow), np.ascontiguousarray(xq)
    return lib().orc_vec_dot_q3_K_q8_K(wrow.size * QK_K, _p(wrow), _p(xq), order)


def q3k_mul_mat(w: np.ndarray, n_rows: int, k: int, xq: np.ndarray, n_cols: int, order=Q3K_GGML,
                n_threads: int = 1) -> np.ndarray:
    """Returns y[n_cols, n_rows] (ggml dst layout)."""
    w, xq = np.ascontiguousarray(w), np.ascontiguousarray(xq)
    y = np.empty((n_cols, n_rows), np.float32)
    lib().orc_q3k_mul_mat(_p(w), n_rows, k, _p(xq), n_cols, _p(y), n_rows, order, n_threads)
    return y


def random_q6_K(rng, n_blocks: int) -> np.ndarray:
    """Valid Q6_K blocks of random bits (any ql/qh/scales bytes) with d a
    positive normal fp16 of the magnitude of a quantized N(0, 0.02) weight."""
    b = rng.integers(0, 256, size=(n_blocks, 210), dtype=np.uint8)
    d = (np.abs(rng.standard_normal(n_blocks)) * 0.00005 + 1e-6).astype(np.float16)
    b[:, 208:210] = d.view(np.uint8).reshape(-1, 2)
    return b.reshape(-1).view(BLOCK_Q6_K)


def dequantize_q6_K(blocks: np.ndarray) -> np.ndarray:
    blocks = np.ascontiguousarray(blocks)
    out = np.empty(blocks.size * QK_K, np.float32)
    lib().orc_dequantize_row_q6_K(_p(blocks), _p(out), out.size)
    return out


def q6k_block_sums(wrow: np.ndarray, xq: np.ndarray) -> np.ndarray:
    wrow, xq = np.ascontiguousarray(wrow), np.ascontiguousarray(xq)
    isum = np.empty(wrow.size, np.int32)
    lib().orc_q6k_block_sums(wrow.size * QK_K, _p(wrow), _p(xq), _p(isum))
    return isum


def vec_dot_q6_K_q8_K(wrow, xq, order=Q3K_GGML) -> float:
    wrow, xq = np.ascontiguousarray(wrow), np.ascontiguousarray(xq)
    return lib().orc_vec_dot_q6_K_q8_K(wrow.size * QK_K, _p(wrow), _p(xq), order)


def q6k_mul_mat(w: np.ndarray, n_rows: int, k: int, xq: np.ndarray, n_cols: int, order=Q3K_GGML,
                n_threads: int = 1) -> np.ndarray:
    w, xq = np.ascontiguousarray(w), np.ascontiguousarray(xq)
    y = np.empty((n_cols, n_rows), np.float32)
    lib().orc_q6k_mul_mat(_p(w), n_rows, k, _p(xq), n_cols, _p(y), n_rows, order, n_threads)
    return y


def q2k_mul_mat(w: np.ndarray, n_rows: int, k: int, xq: np.ndarray, n_cols: int,
                combine=COMBINE_FUSED, n_threads: int = 1) -> np.ndarray:
    """Returns y[n_cols, n_rows] (ggml dst layout, rows contiguous)."""
    w, xq = np.ascontiguousarray(w), np.ascontiguousarray(xq)
    y = np.empty((n_cols, n_rows), np.float32)
    lib().orc_q2k_mul_mat(_p(w), n_rows, k, _p(xq), n_cols, _p(y), n_rows, combine, n_threads)
    return y


def rms_inv(x, eps):
    x = np.ascontiguousarray(x, np.float32)
    return lib().orc_rms_inv(_p(x), x.size, eps)


def rms_sumsq(x):
    """Sum of squares in the fixed order of the RMSNorm (group sums, then the fold)."""
    x = np.ascontiguousarray(x, np.float32)
    return lib().orc_rms_sumsq(_p(x), x.size)


def rmsnorm_quantize_q8_K(x, eps, rounding=ROUND_FUSED, weight=None):
    """RMSNorm (times `weight` when given: sme_ai_rmsnorm_f32's weight operand), then Q8_K."""
    x = np.ascontiguousarray(x, np.float32)
    out = np.zeros(x.size // QK_K, BLOCK_Q8_K)
    if weight is None:
        lib().orc_rmsnorm_quantize_q8_K(_p(x), _p(out), x.size, eps, rounding)
    else:
        weight = np.ascontiguousarray(weight, np.float32)
        assert weight.size == x.size
        lib().orc_rmsnorm_w_quantize_q8_K(_p(x), _p(weight), _p(out), x.size, eps, rounding)
    return out


def silu_mul(g, u):
    g, u = np.ascontiguousarray(g, np.float32), np.ascontiguousarray(u, np.float32)
    h = np.empty_like(g)
    lib().orc_silu_mul(_p(g), _p(u), _p(h), g.size)
    return h
