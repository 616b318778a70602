"""Python view of libsmeai_b200.so (the sm_100a Q2_K / packed-Linear library).

Everything here calls the C-ABI declared in include/sme_ai_ops.h and
include/smeai_q2k.h through ctypes; torch is used only for device memory and
streams.  There is no fallback: if the shared library is missing or cannot
be loaded, ``lib()`` raises.
"""
from __future__ import annotations

import ctypes
import os

PKG = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(PKG, "_lib", "libsmeai_b200.so")
INCLUDE_DIR = os.path.abspath(os.path.join(PKG, "..", "..", "include"))

QK_K = 256
Q2K_BLOCK_BYTES = 84
Q3K_BLOCK_BYTES = 110
Q6K_BLOCK_BYTES = 210
Q8K_BLOCK_BYTES = 292
EPI_STORE, EPI_RESIDUAL, EPI_SILU_MUL = 0, 1, 2
ACT_NONE, ACT_RELU, ACT_GELU, ACT_SILU = 0, 1, 2, 3

SME_AI_OK = 0
SME_AI_BAD_ARGUMENT = -1
SME_AI_ALLOC_FAILED = -2
SME_AI_UNSUPPORTED = -3
SME_AI_WORKSPACE_TOO_SMALL = -4

_lib = None


class SmeaiError(RuntimeError):
    pass


class Workspace(ctypes.Structure):
    """sme_ai_workspace (same field order and types as the C struct)."""
    _fields_ = [(n, ctypes.c_uint64) for n in
                ("max_batch", "max_in_features", "max_out_features", "cntb", "cntw", "max_h",
                 "max_m_pad", "max_k_pad", "max_n_pad")] + \
               [(n, ctypes.c_void_p) for n in
                ("a_pairs", "a_mod", "b_pack", "tmp_f32", "tmp2_f32", "tmp_f16", "gemm_c_tile", "attn_scores")]


class PackedWeight(ctypes.Structure):
    """sme_ai_packed_linear_weight."""
    _fields_ = [("in_features", ctypes.c_uint64), ("out_features", ctypes.c_uint64),
                ("k_pad", ctypes.c_uint64), ("n_pad", ctypes.c_uint64), ("packed_weight", ctypes.c_void_p)]


IN_Q8K, IN_F32, IN_F32_RMS = 0, 1, 2


class Q2KPhase(ctypes.Structure):
    """smeai_q2k_phase: one GEMV of a decode program."""
    _fields_ = [("w", ctypes.c_void_p), ("input", ctypes.c_int), ("x", ctypes.c_void_p),
                ("ld_x", ctypes.c_size_t), ("y", ctypes.c_void_p), ("ldy", ctypes.c_size_t),
                ("epilogue", ctypes.c_int), ("resid", ctypes.c_void_p), ("ld_resid", ctypes.c_size_t),
                ("norm_w", ctypes.c_void_p)]


class Q2KMGPhase(ctypes.Structure):
    """smeai_q2k_mg_phase: one phase of a multi-GPU decode program."""
    _fields_ = [("w", ctypes.c_void_p), ("input", ctypes.c_int), ("x_src", ctypes.c_int),
                ("x_row0", ctypes.c_int64), ("x", ctypes.c_void_p), ("ld_x", ctypes.c_size_t),
                ("epilogue", ctypes.c_int), ("resid_src", ctypes.c_int), ("resid_row0", ctypes.c_int64),
                ("resid", ctypes.c_void_p), ("ld_resid", ctypes.c_size_t), ("norm_w", ctypes.c_void_p),
                ("out_rows", ctypes.c_int64), ("ex_lo", ctypes.c_int64), ("ex_hi", ctypes.c_int64),
                ("ex_row0", ctypes.c_int64), ("y", ctypes.c_void_p), ("ldy", ctypes.c_size_t)]


class PeerExchange(ctypes.Structure):
    """smeai_peer_exchange: the fused all-gather of a row-sharded GEMV."""
    _fields_ = [("n_dst", ctypes.c_int), ("dst", ctypes.c_void_p * 8), ("ld_dst", ctypes.c_int64),
                ("row0", ctypes.c_int64), ("n_sig", ctypes.c_int), ("sig", ctypes.c_void_p * 8),
                ("wait_sig", ctypes.c_void_p), ("wait_count", ctypes.c_uint), ("epoch", ctypes.c_void_p)]


def _declare(L: ctypes.CDLL) -> None:
    P, U64, I64, I, F, SZ = (ctypes.c_void_p, ctypes.c_uint64, ctypes.c_int64, ctypes.c_int,
                             ctypes.c_float, ctypes.c_size_t)
    WS, PW = ctypes.POINTER(Workspace), ctypes.POINTER(PackedWeight)
    sig = {
        # smeai_q2k.h
        "quantize_row_q8_K": (None, [P, P, I64]),
        "quantize_row_q2_K": (None, [P, P, I64]),
        "dequantize_row_q2_K": (None, [P, P, I64]),
        "ggml_vec_dot_q2_K_q8_K": (None, [I, P, SZ, P, SZ, P, SZ, I]),
        "smeai_device_ready": (I, []),
        "smeai_last_error": (ctypes.c_char_p, []),
        "smeai_take_device_error": (I, [ctypes.POINTER(ctypes.c_uint)]),
        "smeai_set_wait_timeouts": (None, [U64, U64]),
        "smeai_debug_fail_next_allocs": (None, [I]),
        "smeai_q2k_repack": (I, [P, I64, I64, ctypes.POINTER(ctypes.c_void_p)]),
        "dequantize_row_q3_K": (None, [P, P, I64]),
        "ggml_vec_dot_q3_K_q8_K": (None, [I, P, SZ, P, SZ, P, SZ, I]),
        "smeai_q3k_repack": (I, [P, I64, I64, ctypes.POINTER(ctypes.c_void_p)]),
        "smeai_q3k_free": (None, [P]),
        "smeai_q3k_mul_mat": (I, [P, P, I64, P, SZ, P]),
        "smeai_q3k_mul_mat_f32": (I, [P, P, SZ, I64, P, SZ, F, P]),
        "smeai_q3k_block_sums": (I, [P, P, P, P, P]),
        "smeai_q3k_dequantize_device": (I, [P, I64, P, P]),
        "smeai_gguf_load_q3k": (I, [P, I64, ctypes.POINTER(ctypes.c_void_p)]),
        "dequantize_row_q6_K": (None, [P, P, I64]),
        "ggml_vec_dot_q6_K_q8_K": (None, [I, P, SZ, P, SZ, P, SZ, I]),
        "smeai_q6k_repack": (I, [P, I64, I64, ctypes.POINTER(ctypes.c_void_p)]),
        "smeai_q6k_free": (None, [P]),
        "smeai_q6k_mul_mat": (I, [P, P, I64, P, SZ, P]),
        "smeai_q6k_mul_mat_f32": (I, [P, P, SZ, I64, P, SZ, F, P]),
        "smeai_q6k_block_sums": (I, [P, P, P, P, P]),
        "smeai_q6k_dequantize_device": (I, [P, I64, P, P]),
        "smeai_gguf_load_q6k": (I, [P, I64, ctypes.POINTER(ctypes.c_void_p)]),
        # smeai_gguf.h
        "smeai_gguf_open": (I, [ctypes.c_char_p, ctypes.POINTER(ctypes.c_void_p)]),
        "smeai_gguf_close": (None, [P]),
        "smeai_gguf_version": (I, [P]),
        "smeai_gguf_alignment": (U64, [P]),
        "smeai_gguf_data_offset": (U64, [P]),
        "smeai_gguf_n_tensors": (I64, [P]),
        "smeai_gguf_find_tensor": (I64, [P, ctypes.c_char_p]),
        "smeai_gguf_tensor_info": (I, [P, I64, ctypes.POINTER(ctypes.c_char_p), ctypes.POINTER(I),
                                       ctypes.POINTER(I), ctypes.POINTER(I64), ctypes.POINTER(U64),
                                       ctypes.POINTER(U64)]),
        "smeai_gguf_read_tensor": (I, [P, I64, P, U64]),
        "smeai_gguf_load_q2k": (I, [P, I64, ctypes.POINTER(ctypes.c_void_p)]),
        "smeai_gguf_n_kv": (I64, [P]),
        "smeai_gguf_find_key": (I64, [P, ctypes.c_char_p]),
        "smeai_gguf_key_type": (I, [P, ctypes.c_char_p]),
        "smeai_gguf_get_u64": (I, [P, ctypes.c_char_p, ctypes.POINTER(U64)]),
        "smeai_gguf_get_f64": (I, [P, ctypes.c_char_p, ctypes.POINTER(ctypes.c_double)]),
        "smeai_gguf_get_str": (I, [P, ctypes.c_char_p, ctypes.POINTER(ctypes.c_char_p)]),
        "smeai_q2k_free": (None, [P]),
        "smeai_q2k_weight_bytes": (SZ, [P]),
        "smeai_q8k_quantize": (I, [P, I64, I64, I64, P, P]),
        "smeai_rms_q8k_quantize": (I, [P, I64, I64, I64, F, P, P]),
        "smeai_rms_q8k_quantize_w": (I, [P, I64, I64, I64, P, F, P, P]),
        "smeai_q2k_mul_mat": (I, [P, I64, I64, P, I64, P, SZ, P]),
        "smeai_q2k_mul_mat_ex": (I, [P, P, I64, P, SZ, I, P, SZ, P]),
        "smeai_q2k_mul_mat_tc": (I, [P, P, I64, P, SZ, P]),
        "smeai_q2k_mul_mat_tc_ex": (I, [P, P, I64, P, SZ, I, P, SZ, P]),
        "smeai_q2k_mul_mat_f32": (I, [P, P, I64, P, SZ, P]),
        "smeai_q2k_mul_mat_f32_ex": (I, [P, P, SZ, I64, P, SZ, I, P, SZ, F, P]),
        "smeai_q2k_mul_mat_f32_norm": (I, [P, P, SZ, I64, P, SZ, I, P, SZ, F, P, P]),
        "smeai_q2k_mul_mat_f32_peer": (I, [P, P, SZ, I64, P, SZ, I, P, SZ, F, P, ctypes.POINTER(PeerExchange), P]),
        "smeai_peer_step_end": (I, [P, ctypes.c_uint, P, P]),
        "smeai_ipc_alloc": (I, [SZ, ctypes.POINTER(ctypes.c_void_p), P]),
        "smeai_ipc_free": (None, [P]),
        "smeai_ipc_open": (I, [P, ctypes.POINTER(ctypes.c_void_p)]),
        "smeai_ipc_close": (None, [P]),
        "smeai_q2k_block_sums": (I, [P, P, P, P, P]),
        "smeai_q2k_program_create": (I, [ctypes.POINTER(Q2KPhase), I, I64, F, ctypes.POINTER(ctypes.c_void_p)]),
        "smeai_q2k_program_run": (I, [P, P]),
        "smeai_q2k_mg_program_create": (I, [ctypes.POINTER(Q2KMGPhase), I, I64, F, I, I,
                                             ctypes.POINTER(ctypes.c_void_p)]),
        "smeai_q2k_program_ipc_handle": (I, [P, P]),
        "smeai_q2k_program_connect": (I, [P, P, I]),
        "smeai_q2k_program_gather": (I, [P, I, P, SZ, P]),
        "smeai_q2k_program_reset": (I, [P, P]),
        "smeai_q2k_program_free": (None, [P]),
        "smeai_q2k_quantize_device": (I, [P, I64, P, P]),
        "smeai_q2k_dequantize_device": (I, [P, I64, P, P]),
        # sme_ai_ops.h
        "sme_ai_has_sme": (I, []),
        "sme_ai_has_sme2": (I, []),
        "sme_ai_cntb": (U64, []),
        "sme_ai_cntw": (U64, []),
        "sme_ai_workspace_init": (I, [WS, U64, U64, U64]),
        "sme_ai_workspace_destroy": (None, [WS]),
        "sme_ai_packed_linear_weight_init": (I, [PW, P, U64, U64]),
        "sme_ai_packed_linear_weight_init_f32": (I, [PW, P, U64, U64]),
        "sme_ai_packed_linear_weight_destroy": (None, [PW]),
        "sme_ai_linear_sme_packed_f32f32": (I, [WS, P, U64, PW, P, P]),
        "sme_ai_linear_packed_f16f32_device": (I, [P, U64, PW, P, I, P, P]),
        "sme_ai_linear_sme_simple_f16f32": (I, [WS, P, U64, U64, P, U64, P, P]),
        "sme_ai_swiglu_ref_f16f32": (I, [WS, P, U64, U64, P, U64, P, P, P, P, U64, P, P]),
        "sme_ai_swiglu_sme_packed_f16f32": (I, [WS, P, U64, PW, P, PW, P, PW, P, P]),
        "sme_ai_swiglu_packed_f16f32_noalloc": (I, [P, U64, PW, P, PW, P, PW, P, P, P]),
        "sme_ai_self_attention_ref_f16f32": (I, [WS, P, U64, U64, U64, P, P, P, P, P, P, P, P, I, P]),
        "sme_ai_self_attention_sme_packed_f16f32": (I, [WS, P, U64, U64, U64, PW, P, PW, P, PW, P, PW, P, I, P]),
        "sme_ai_self_attention_packed_f16f32_device": (I, [WS, P, U64, U64, U64, PW, P, PW, P, PW, P, PW, P, I, P,
                                                           P]),
        "sme_ai_self_attention_core_f32_device": (I, [P, P, P, U64, U64, U64, I, P, P]),
        "sme_ai_add_f32": (None, [P, P, P, U64]),
        "sme_ai_mul_f32": (None, [P, P, P, U64]),
        "sme_ai_residual_add_f32": (None, [P, P, P, U64]),
        "sme_ai_add_bias_rowwise_f32": (None, [P, P, P, U64, U64]),
        "sme_ai_relu_inplace_f32": (None, [P, U64]),
        "sme_ai_gelu_inplace_f32": (None, [P, U64]),
        "sme_ai_silu_inplace_f32": (None, [P, U64]),
    }
    for act in ("", "relu_", "gelu_", "silu_"):
        sig[f"sme_ai_linear_{act}ref_f16f32"] = (I, [P, U64, U64, P, U64, P, P])
        sig[f"sme_ai_linear_{act}sme_packed_f16f32"] = (I, [WS, P, U64, PW, P, P])
    for act in ("relu", "gelu"):
        sig[f"sme_ai_mlp_{act}_ref_f16f32"] = (I, [WS, P, U64, U64, P, U64, P, P, U64, P, P])
        sig[f"sme_ai_mlp_{act}_sme_packed_f16f32"] = (I, [WS, P, U64, PW, P, PW, P, P])
    for name, (res, args) in sig.items():
        fn = getattr(L, name)
        fn.restype = res
        fn.argtypes = args


def lib() -> ctypes.CDLL:
    """Load the library (raises if it is missing: there is no fallback)."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise SmeaiError(f"{LIB_PATH} is missing: run __graft_entry__.build() (nvcc, sm_100a)")
        L = ctypes.CDLL(LIB_PATH)
        _declare(L)
        _lib = L
    return _lib


def last_error() -> str:
    return lib().smeai_last_error().decode(errors="replace")


def check(status: int, what: str = "") -> None:
    if status != 0:
        raise SmeaiError(f"{what} failed with status {status}: {last_error()}")


def device_ready() -> bool:
    return bool(lib().smeai_device_ready())


def take_device_error() -> int:
    """The device error word of the current GPU (a bounded wait that timed
    out sets it), cleared; 0 when no kernel reported one."""
    code = ctypes.c_uint(0)
    check(lib().smeai_take_device_error(ctypes.byref(code)), "take_device_error")
    return code.value


def exported_symbols_from_headers() -> list[str]:
    """Function names declared in include/*.h (what the library must export)."""
    import re
    names = []
    for h in sorted(os.listdir(INCLUDE_DIR)):
        if not h.endswith(".h"):
            continue
        text = open(os.path.join(INCLUDE_DIR, h)).read()
        text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
        for m in re.finditer(r"^\s*(?:[A-Za-z_][\w\s\*]*?)\b([A-Za-z_]\w*)\s*\(", text, flags=re.M):
            name = m.group(1)
            if name in ("defined", "if", "sizeof"):
                continue
            names.append(name)
    return sorted(set(names))
