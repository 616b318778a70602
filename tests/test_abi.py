"""CPU tests of the C-ABI boundary: the library loads, exports every symbol
the public headers declare, keeps the reference struct layouts, and its
argument checks answer without a GPU (no compute is launched here)."""
import ctypes
import os
import subprocess

import pytest

import smeai_b200 as S

ROOT = os.path.abspath(os.path.join(os.path.dirname(__file__), ".."))


def test_library_exports_every_declared_symbol():
    L = S.lib()
    names = S.exported_symbols_from_headers()
    assert len(names) >= 45
    missing = [n for n in names if not hasattr(L, n)]
    assert not missing, missing


def test_headers_declare_the_reference_entry_points():
    names = set(S.exported_symbols_from_headers())
    for n in ("sme_ai_workspace_init", "sme_ai_workspace_destroy", "sme_ai_packed_linear_weight_init",
              "sme_ai_packed_linear_weight_destroy", "sme_ai_linear_ref_f16f32",
              "sme_ai_linear_sme_simple_f16f32", "sme_ai_linear_sme_packed_f16f32",
              "sme_ai_mlp_relu_sme_packed_f16f32", "sme_ai_mlp_gelu_sme_packed_f16f32",
              "sme_ai_swiglu_ref_f16f32", "sme_ai_swiglu_sme_packed_f16f32", "sme_ai_has_sme", "sme_ai_cntw",
              "quantize_row_q8_K", "ggml_vec_dot_q2_K_q8_K", "smeai_q2k_mul_mat", "smeai_q2k_repack"):
        assert n in names


def test_struct_layout_matches_reference():
    # sme_ai_ops.h:61-79 and :92-98: 9 uint64 then 8 pointers; 4 uint64 then 1 pointer
    assert ctypes.sizeof(S.Workspace) == 9 * 8 + 8 * 8
    assert ctypes.sizeof(S.PackedWeight) == 4 * 8 + 8
    assert S.Workspace.a_pairs.offset == 72 and S.Workspace.attn_scores.offset == 128
    assert S.PackedWeight.packed_weight.offset == 32


def test_plain_c_caller_builds_and_links(tmp_path):
    exe = tmp_path / "abi_check"
    libdir = os.path.dirname(S.LIB_PATH)
    cmd = ["gcc", "-std=gnu11", "-Wall", "-Werror", "-I", os.path.join(ROOT, "include"),
           os.path.join(ROOT, "tests", "c", "abi_check.c"), "-L", libdir, "-lsmeai_b200",
           f"-Wl,-rpath,{libdir}", "-o", str(exe)]
    # the library's file name is libsmeai_b200.so, so -lsmeai_b200 resolves it
    subprocess.run(cmd, check=True)
    out = subprocess.run([str(exe)], check=True, capture_output=True, text=True).stdout
    kv = dict(tok.split("=") for line in out.split("\n") for tok in line.split() if "=" in tok)
    assert kv["sizeof_ws"] == "136" and kv["sizeof_packed"] == "40" and kv["sizeof_fp16"] == "2"
    assert kv["off_a_pairs"] == "72" and kv["off_tmp_f16"] == "112" and kv["off_packed"] == "32"
    assert kv["cntb"] == "64" and kv["cntw"] == "16"
    assert kv["bad_ws"] == "-1" and kv["bad_zero"] == "-1" and kv["bad_ref"] == "-1"
    assert kv["bad_packed"] == "-1" and kv["bad_repack"] == "-1" and kv["bad_mulmat"] == "-1"
    assert kv["block_bytes"] == "84,292"


def test_argument_checks_without_device():
    L = S.lib()
    ws = S.Workspace()
    assert L.sme_ai_workspace_init(None, 1, 1, 1) == S.SME_AI_BAD_ARGUMENT
    assert L.sme_ai_workspace_init(ctypes.byref(ws), 0, 4, 4) == S.SME_AI_BAD_ARGUMENT
    pw = S.PackedWeight()
    assert L.sme_ai_packed_linear_weight_init(ctypes.byref(pw), None, 4, 4) == S.SME_AI_BAD_ARGUMENT
    assert L.smeai_q2k_repack(None, 1, 256, None) == S.SME_AI_BAD_ARGUMENT
    h = ctypes.c_void_p()
    buf = (ctypes.c_uint8 * 84)()
    assert L.smeai_q2k_repack(buf, 1, 100, ctypes.byref(h)) == S.SME_AI_BAD_ARGUMENT  # k % 256 != 0
    bogus = (ctypes.c_uint8 * 64)()
    assert L.smeai_q2k_mul_mat(bogus, 1, 256, bogus, 1, bogus, 1, None) == S.SME_AI_BAD_ARGUMENT
    assert "handle" in S.last_error()
    assert L.sme_ai_cntw() == 16 and L.sme_ai_cntb() == 64 and L.sme_ai_has_sme2() == 0


@pytest.mark.skipif(__import__("torch").cuda.is_available(), reason="only meaningful on a host without a GPU")
def test_no_device_reports_unsupported():
    L = S.lib()
    ws = S.Workspace()
    assert L.sme_ai_has_sme() == 0
    assert L.sme_ai_workspace_init(ctypes.byref(ws), 4, 4, 4) == S.SME_AI_UNSUPPORTED
    h = ctypes.c_void_p()
    buf = (ctypes.c_uint8 * 84)()
    assert L.smeai_q2k_repack(buf, 1, 256, ctypes.byref(h)) == S.SME_AI_UNSUPPORTED
