"""GPU parity of the sme_ai_ops.h packed Linear / MLP / SwiGLU operators
against the CPU oracle, through the C-ABI with host pointers (as a reference
caller uses them) and device pointers.

Bar: Linear outputs are bit-exact (k-ascending fp32 sums of exact fp16
products); ReLU likewise; GELU/SiLU (CUDA tanhf/expf vs glibc) within
rel 1e-6 + abs 1e-7; MLP/SwiGLU, whose hidden state is rounded to fp16, within
the reference bench's own bars (abs 0.08 / rel 0.02) and in practice far
tighter (checked at 1e-3 abs).
"""
import ctypes

import numpy as np
import pytest
import torch

import smeai_b200 as S

pytestmark = pytest.mark.gpu
P = ctypes.c_void_p


def p(a):
    return P(a.ctypes.data) if a is not None else None


@pytest.fixture
def L(cuda):
    return S.lib()


def make_ws(L, batch, kin, kout):
    ws = S.Workspace()
    assert L.sme_ai_workspace_init(ctypes.byref(ws), batch, kin, kout) == 0, S.last_error()
    assert ws.cntw == 16 and ws.cntb == 64 and ws.max_k_pad == (kin + 15) // 16 * 16
    return ws


def make_packed(L, w16, kin, kout):
    pw = S.PackedWeight()
    assert L.sme_ai_packed_linear_weight_init(ctypes.byref(pw), p(w16), kin, kout) == 0, S.last_error()
    assert pw.k_pad == (kin + 15) // 16 * 16 and pw.n_pad == (kout + 15) // 16 * 16 and pw.packed_weight
    return pw


def test_demo_linear_exact_golden(L, golden):
    """examples/demo_linear.c: batch 2, 16->16; exact expected output."""
    g = golden("demo_linear.npz")
    ws = make_ws(L, 2, 16, 16)
    pw = make_packed(L, g["w16"], 16, 16)
    out = np.zeros((2, 16), np.float32)
    assert L.sme_ai_linear_sme_packed_f16f32(ctypes.byref(ws), p(g["x16"]), 2, ctypes.byref(pw), p(g["bias"]),
                                             p(out)) == 0
    assert np.array_equal(out, g["expected"])
    ref = np.zeros((2, 16), np.float32)
    assert L.sme_ai_linear_ref_f16f32(p(g["x16"]), 2, 16, p(g["w16"]), 16, p(g["bias"]), p(ref)) == 0
    assert np.array_equal(ref, g["expected"])
    L.sme_ai_packed_linear_weight_destroy(ctypes.byref(pw))
    assert pw.packed_weight is None and pw.in_features == 0
    L.sme_ai_workspace_destroy(ctypes.byref(ws))
    assert ws.max_batch == 0 and ws.a_pairs is None


@pytest.mark.parametrize("act,name", [(0, ""), (1, "relu_"), (2, "gelu_"), (3, "silu_")])
def test_linear_bench_case(L, oracle, act, name):
    """bench_sme_full_timing.c run_linear_case: batch 8, 128->128, seeds 1001-1003."""
    B, K, N = 8, 128, 128
    x16, w16, b = oracle.lcg_f16(B * K, 1001), oracle.lcg_f16(K * N, 1002), oracle.lcg_f32(N, 1003)
    ws = make_ws(L, B, K, N)
    pw = make_packed(L, w16, K, N)
    out = np.zeros((B, N), np.float32)
    ref = np.zeros((B, N), np.float32)
    assert getattr(L, f"sme_ai_linear_{name}sme_packed_f16f32")(ctypes.byref(ws), p(x16), B, ctypes.byref(pw),
                                                                  p(b), p(out)) == 0
    assert getattr(L, f"sme_ai_linear_{name}ref_f16f32")(p(x16), B, K, p(w16), N, p(b), p(ref)) == 0
    exp = oracle.linear_f16f32(x16, B, K, w16, N, b, act=act)
    if act in (0, 1):
        assert np.array_equal(out, exp) and np.array_equal(ref, exp)
    else:
        assert np.allclose(out, exp, rtol=1e-6, atol=1e-7) and np.allclose(ref, exp, rtol=1e-6, atol=1e-7)
    L.sme_ai_packed_linear_weight_destroy(ctypes.byref(pw))
    L.sme_ai_workspace_destroy(ctypes.byref(ws))


def test_linear_simple_path(L, oracle):
    B, K, N = 5, 70, 33          # neither K nor N a multiple of 16
    x16, w16, b = oracle.lcg_f16(B * K, 11), oracle.lcg_f16(K * N, 12), oracle.lcg_f32(N, 13)
    ws = make_ws(L, 8, 128, 64)
    out = np.zeros((B, N), np.float32)
    assert L.sme_ai_linear_sme_simple_f16f32(ctypes.byref(ws), p(x16), B, K, p(w16), N, p(b), p(out)) == 0
    assert np.array_equal(out, oracle.linear_f16f32(x16, B, K, w16, N, b))
    L.sme_ai_workspace_destroy(ctypes.byref(ws))


@pytest.mark.parametrize("B,K,N", [(1, 16, 16), (3, 17, 5), (17, 300, 129), (128, 512, 512), (200, 1024, 768)])
def test_linear_shapes_bit_exact(L, oracle, B, K, N):
    x16, w16 = oracle.lcg_f16(B * K, B + 1), oracle.lcg_f16(K * N, K + 2)
    b = oracle.lcg_f32(N, N + 3)
    ws = make_ws(L, B, K, N)
    pw = make_packed(L, w16, K, N)
    out = np.zeros((B, N), np.float32)
    assert L.sme_ai_linear_sme_packed_f16f32(ctypes.byref(ws), p(x16), B, ctypes.byref(pw), p(b), p(out)) == 0
    assert np.array_equal(out, oracle.linear_f16f32(x16, B, K, w16, N, b))
    # NULL bias is allowed
    assert L.sme_ai_linear_sme_packed_f16f32(ctypes.byref(ws), p(x16), B, ctypes.byref(pw), None, p(out)) == 0
    assert np.array_equal(out, oracle.linear_f16f32(x16, B, K, w16, N, None))
    L.sme_ai_packed_linear_weight_destroy(ctypes.byref(pw))
    L.sme_ai_workspace_destroy(ctypes.byref(ws))


def test_linear_config1_fp32(L, oracle):
    """X[128,512] ~N(0,1), W[512,512] ~U(+-1/sqrt(512)), bias ~N(0,0.02), seed 0:
    the true-fp32 operator, bit-exact with the sequential fused oracle; and the
    fp16 drop-in on the fp16-rounded draws, bit-exact."""
    rng = np.random.default_rng(0)
    B, K, N = 128, 512, 512
    x = rng.standard_normal((B, K)).astype(np.float32)
    wt = rng.uniform(-1 / np.sqrt(K), 1 / np.sqrt(K), (N, K)).astype(np.float32)   # W[out,in]
    b = (rng.standard_normal(N) * 0.02).astype(np.float32)
    w = np.ascontiguousarray(wt.T)                                                 # [in,out]: Y = X W^T + b
    ws = make_ws(L, B, K, N)
    pw = S.PackedWeight()
    assert L.sme_ai_packed_linear_weight_init_f32(ctypes.byref(pw), p(w), K, N) == 0
    out = np.zeros((B, N), np.float32)
    assert L.sme_ai_linear_sme_packed_f32f32(ctypes.byref(ws), p(x), B, ctypes.byref(pw), p(b), p(out)) == 0
    exp = oracle.linear_f32f32(x, B, K, w, N, b)
    assert np.array_equal(out, exp)
    ref64 = x.astype(np.float64) @ w.astype(np.float64) + b
    assert np.all(np.abs(out - ref64) <= 1e-5 * np.maximum(np.abs(ref64), np.abs(ref64).max()))
    L.sme_ai_packed_linear_weight_destroy(ctypes.byref(pw))
    x16, w16 = x.astype(np.float16).view(np.uint16), w.astype(np.float16).view(np.uint16)
    pw = make_packed(L, w16, K, N)
    assert L.sme_ai_linear_sme_packed_f16f32(ctypes.byref(ws), p(x16), B, ctypes.byref(pw), p(b), p(out)) == 0
    assert np.array_equal(out, oracle.linear_f16f32(x16, B, K, w16, N, b))
    L.sme_ai_packed_linear_weight_destroy(ctypes.byref(pw))
    L.sme_ai_workspace_destroy(ctypes.byref(ws))


def test_linear_device_pointers(L, oracle, cuda):
    B, K, N = 64, 256, 384
    x16, w16, b = oracle.lcg_f16(B * K, 5), oracle.lcg_f16(K * N, 6), oracle.lcg_f32(N, 7)
    pw = make_packed(L, w16, K, N)
    xd = torch.from_numpy(x16.view(np.int16)).to(cuda)
    bd = torch.from_numpy(b).to(cuda)
    yd = torch.zeros((B, N), device=cuda)
    st = L.sme_ai_linear_packed_f16f32_device(P(xd.data_ptr()), B, ctypes.byref(pw), P(bd.data_ptr()), 3,
                                              P(yd.data_ptr()), P(torch.cuda.current_stream().cuda_stream))
    assert st == 0
    exp = oracle.linear_f16f32(x16, B, K, w16, N, b, act=oracle.ACT_SILU)
    assert np.allclose(yd.cpu().numpy(), exp, rtol=1e-6, atol=1e-7)
    # the host-pointer entry also accepts device pointers in place
    ws = make_ws(L, B, K, N)
    yd.zero_()
    assert L.sme_ai_linear_sme_packed_f16f32(ctypes.byref(ws), P(xd.data_ptr()), B, ctypes.byref(pw),
                                             P(bd.data_ptr()), P(yd.data_ptr())) == 0
    assert np.array_equal(yd.cpu().numpy(), oracle.linear_f16f32(x16, B, K, w16, N, b))
    L.sme_ai_packed_linear_weight_destroy(ctypes.byref(pw))
    L.sme_ai_workspace_destroy(ctypes.byref(ws))


@pytest.mark.parametrize("act,name", [(1, "relu"), (2, "gelu")])
def test_mlp_bench_case(L, oracle, act, name):
    """run_mlp_case shape: batch 4, 128 -> 256 -> 128."""
    B, K, H, N = 4, 128, 256, 128
    x16, w1, w2 = oracle.lcg_f16(B * K, 2001), oracle.lcg_f16(K * H, 2002), oracle.lcg_f16(H * N, 2003)
    b1, b2 = oracle.lcg_f32(H, 2004), oracle.lcg_f32(N, 2005)
    ws = make_ws(L, B, H, H)
    p1, p2 = make_packed(L, w1, K, H), make_packed(L, w2, H, N)
    out = np.zeros((B, N), np.float32)
    ref = np.zeros((B, N), np.float32)
    assert getattr(L, f"sme_ai_mlp_{name}_sme_packed_f16f32")(ctypes.byref(ws), p(x16), B, ctypes.byref(p1), p(b1),
                                                                ctypes.byref(p2), p(b2), p(out)) == 0
    assert getattr(L, f"sme_ai_mlp_{name}_ref_f16f32")(ctypes.byref(ws), p(x16), B, K, p(w1), H, p(b1), p(w2), N,
                                                         p(b2), p(ref)) == 0
    exp = oracle.mlp_f16f32(x16, B, K, w1, H, b1, w2, N, b2, act)
    if act == 1:
        assert np.array_equal(out, exp) and np.array_equal(ref, exp)
    else:
        assert np.abs(out - exp).max() <= 1e-3 and np.abs(ref - exp).max() <= 1e-3
    for a in (p1, p2):
        L.sme_ai_packed_linear_weight_destroy(ctypes.byref(a))
    L.sme_ai_workspace_destroy(ctypes.byref(ws))


def test_swiglu_bench_case(L, oracle):
    """run_swiglu_case: batch 4, 128 -> 256 -> 128, seeds 3001-3007, bars abs 0.08 / rel 0.02."""
    B, K, H, N = 4, 128, 256, 128
    x16, wg, wu, wd = (oracle.lcg_f16(n, s) for n, s in
                       ((B * K, 3001), (K * H, 3002), (K * H, 3003), (H * N, 3004)))
    bg, bu, bd = oracle.lcg_f32(H, 3005), oracle.lcg_f32(H, 3006), oracle.lcg_f32(N, 3007)
    ws = make_ws(L, B, H, H)
    pg, pu, pd = make_packed(L, wg, K, H), make_packed(L, wu, K, H), make_packed(L, wd, H, N)
    out = np.zeros((B, N), np.float32)
    ref = np.zeros((B, N), np.float32)
    assert L.sme_ai_swiglu_sme_packed_f16f32(ctypes.byref(ws), p(x16), B, ctypes.byref(pg), p(bg), ctypes.byref(pu),
                                             p(bu), ctypes.byref(pd), p(bd), p(out)) == 0
    assert L.sme_ai_swiglu_ref_f16f32(ctypes.byref(ws), p(x16), B, K, p(wg), H, p(bg), p(wu), p(bu), p(wd), N, p(bd),
                                      p(ref)) == 0
    exp = oracle.swiglu_f16f32(x16, B, K, wg, H, bg, wu, bu, wd, N, bd)
    for got in (out, ref):
        err = np.abs(got - exp)
        assert np.all((err <= 0.08) | (err <= 0.02 * np.abs(exp)))   # the reference bench's own bar
        assert err.max() <= 1e-3
    # mismatched shapes are refused
    assert L.sme_ai_swiglu_sme_packed_f16f32(ctypes.byref(ws), p(x16), B, ctypes.byref(pg), p(bg), ctypes.byref(pu),
                                             p(bu), ctypes.byref(pg), p(bd), p(out)) == S.SME_AI_BAD_ARGUMENT
    for a in (pg, pu, pd):
        L.sme_ai_packed_linear_weight_destroy(ctypes.byref(a))
    L.sme_ai_workspace_destroy(ctypes.byref(ws))


def test_status_codes(L, oracle):
    x16, w16 = oracle.lcg_f16(4 * 32, 1), oracle.lcg_f16(32 * 32, 2)
    ws = make_ws(L, 4, 32, 32)
    pw = make_packed(L, w16, 32, 32)
    out = np.zeros((8, 32), np.float32)
    assert L.sme_ai_linear_sme_packed_f16f32(ctypes.byref(ws), p(x16), 8, ctypes.byref(pw), None,
                                             p(out)) == S.SME_AI_WORKSPACE_TOO_SMALL
    assert L.sme_ai_linear_sme_packed_f16f32(ctypes.byref(ws), p(x16), 0, ctypes.byref(pw), None,
                                             p(out)) == S.SME_AI_BAD_ARGUMENT
    assert L.sme_ai_linear_sme_packed_f16f32(None, p(x16), 4, ctypes.byref(pw), None,
                                             p(out)) == S.SME_AI_BAD_ARGUMENT
    assert L.sme_ai_linear_sme_packed_f16f32(ctypes.byref(ws), None, 4, ctypes.byref(pw), None,
                                             p(out)) == S.SME_AI_BAD_ARGUMENT
    big = make_packed(L, oracle.lcg_f16(64 * 32, 3), 64, 32)
    assert L.sme_ai_linear_sme_packed_f16f32(ctypes.byref(ws), p(x16), 4, ctypes.byref(big), None,
                                             p(out)) == S.SME_AI_WORKSPACE_TOO_SMALL
    for a in (pw, big):
        L.sme_ai_packed_linear_weight_destroy(ctypes.byref(a))
    L.sme_ai_workspace_destroy(ctypes.byref(ws))


def test_elementwise_helpers(L):
    rng = np.random.default_rng(0)
    a = rng.standard_normal(1000).astype(np.float32)
    b = rng.standard_normal(1000).astype(np.float32)
    out = np.zeros_like(a)
    L.sme_ai_add_f32(p(out), p(a), p(b), 1000)
    assert np.array_equal(out, a + b)
    L.sme_ai_mul_f32(p(out), p(a), p(b), 1000)
    assert np.array_equal(out, a * b)
    m = a.reshape(10, 100).copy()
    bias = b[:100].copy()
    o2 = np.zeros_like(m)
    L.sme_ai_add_bias_rowwise_f32(p(o2), p(m), p(bias), 10, 100)
    assert np.array_equal(o2, m + bias)
    r = a.copy()
    L.sme_ai_relu_inplace_f32(p(r), 1000)
    assert np.array_equal(r, np.maximum(a, 0))
    s = a.copy()
    L.sme_ai_silu_inplace_f32(p(s), 1000)
    assert np.allclose(s, a / (1 + np.exp(-a.astype(np.float64))), rtol=1e-6, atol=1e-7)
