"""GPU parity of the packed Linear / MLP / SwiGLU at prefill-sized shapes,
where the launcher picks the register-tiled kernel (linear_tiled_kernel:
128 x 128 output tiles, 128 x 64 for the gate/up pair).  Rows are independent,
so the oracle is run on sampled row blocks (first, middle, last) and the
device output must match it there bit for bit (GELU / SiLU within the CUDA
tanhf / expf vs glibc bar of the small-shape tests)."""
import ctypes

import numpy as np
import pytest

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
    return ws


def make_packed(L, w16, kin, kout):
    pw = S.PackedWeight()
    assert L.sme_ai_packed_linear_weight_init(ctypes.byref(pw), p(w16), kin, kout) == 0, S.last_error()
    return pw


def row_blocks(M, width=8):
    return [slice(0, width), slice(M // 2 - width // 2, M // 2 + width // 2), slice(M - width, M)]


@pytest.mark.parametrize("M,K,N", [(600, 264, 4000), (512, 4096, 4096), (600, 260, 4000), (129, 512, 16384)])
@pytest.mark.parametrize("act,name", [(0, ""), (1, "relu_"), (3, "silu_")])
def test_linear_large(L, oracle, M, K, N, act, name):
    """K = 264: a half-empty last k step; N = 4000: a ragged last column tile
    (packed width 4000); K = 260: not a multiple of 8 (the 64x64 kernel);
    M = 129: one valid row in the last row tile."""
    x16, w16, b = oracle.lcg_f16(M * K, 11 + K), oracle.lcg_f16(K * N, 12 + N), oracle.lcg_f32(N, 13)
    ws = make_ws(L, M, K, N)
    pw = make_packed(L, w16, K, N)
    out = np.zeros((M, N), np.float32)
    assert getattr(L, f"sme_ai_linear_{name}sme_packed_f16f32")(ctypes.byref(ws), p(x16), M, ctypes.byref(pw),
                                                                  p(b), p(out)) == 0, S.last_error()
    xs = x16.reshape(M, K)
    for sl in row_blocks(M):
        rows = np.ascontiguousarray(xs[sl]).reshape(-1)
        exp = oracle.linear_f16f32(rows, sl.stop - sl.start, K, w16, N, b, act=act)
        got = out[sl]
        if act in (0, 1):
            assert np.array_equal(got, exp), (sl, np.abs(got - exp).max())
        else:
            assert np.allclose(got, exp, rtol=1e-6, atol=1e-7)
    L.sme_ai_packed_linear_weight_destroy(ctypes.byref(pw))
    L.sme_ai_workspace_destroy(ctypes.byref(ws))


def test_mlp_relu_large(L, oracle):
    """fc1 512 x 256 -> 4096 through the tiled kernel's fp16 epilogue, fc2 -> 384."""
    M, K, H, N = 512, 256, 4096, 384
    x16, w1, w2 = oracle.lcg_f16(M * K, 21), oracle.lcg_f16(K * H, 22), oracle.lcg_f16(H * N, 23)
    b1, b2 = oracle.lcg_f32(H, 24), oracle.lcg_f32(N, 25)
    ws = make_ws(L, M, H, H)
    p1, p2 = make_packed(L, w1, K, H), make_packed(L, w2, H, N)
    out = np.zeros((M, N), np.float32)
    assert L.sme_ai_mlp_relu_sme_packed_f16f32(ctypes.byref(ws), p(x16), M, ctypes.byref(p1), p(b1),
                                               ctypes.byref(p2), p(b2), p(out)) == 0, S.last_error()
    xs = x16.reshape(M, K)
    for sl in row_blocks(M):
        rows = np.ascontiguousarray(xs[sl]).reshape(-1)
        exp = oracle.mlp_f16f32(rows, sl.stop - sl.start, K, w1, H, b1, w2, N, b2, 1)
        assert np.array_equal(out[sl], exp)
    for a in (p1, p2):
        L.sme_ai_packed_linear_weight_destroy(ctypes.byref(a))
    L.sme_ai_workspace_destroy(ctypes.byref(ws))


def test_swiglu_large(L, oracle):
    """gate/up 512 x 256 -> 2048 through the tiled pair kernel (128 x 64 tiles), down -> 256."""
    M, K, H, N = 512, 256, 2048, 256
    x16, wg, wu, wd = (oracle.lcg_f16(n, s) for n, s in ((M * K, 31), (K * H, 32), (K * H, 33), (H * N, 34)))
    bg, bu, bd = oracle.lcg_f32(H, 35), oracle.lcg_f32(H, 36), oracle.lcg_f32(N, 37)
    ws = make_ws(L, M, H, H)
    pg, pu, pd = make_packed(L, wg, K, H), make_packed(L, wu, K, H), make_packed(L, wd, H, N)
    out = np.zeros((M, N), np.float32)
    assert L.sme_ai_swiglu_sme_packed_f16f32(ctypes.byref(ws), p(x16), M, ctypes.byref(pg), p(bg), ctypes.byref(pu),
                                             p(bu), ctypes.byref(pd), p(bd), p(out)) == 0, S.last_error()
    xs = x16.reshape(M, K)
    for sl in row_blocks(M):
        rows = np.ascontiguousarray(xs[sl]).reshape(-1)
        exp = oracle.swiglu_f16f32(rows, sl.stop - sl.start, K, wg, H, bg, wu, bu, wd, N, bd)
        err = np.abs(out[sl] - exp)
        assert np.all((err <= 0.08) | (err <= 0.02 * np.abs(exp)))
        assert err.max() <= 1e-3
    for a in (pg, pu, pd):
        L.sme_ai_packed_linear_weight_destroy(ctypes.byref(a))
    L.sme_ai_workspace_destroy(ctypes.byref(ws))
