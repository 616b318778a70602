"""GPU parity of the Q2_K x Q8_K path against the CPU oracle, through the C-ABI.

Bar: Q8_K blocks, Q2_K blocks and the per-super-block integer sums are
bit-exact; mul_mat outputs are bit-exact with the oracle's sequential
ggml-order combine (ORC_COMBINE_FUSED) -- stricter than the 1e-4 relative
tolerance the path allows; the silu*mul epilogue (CUDA expf vs glibc expf)
is held to rel 1e-5.
"""
import ctypes

import numpy as np
import pytest
import torch

import smeai_b200 as S
from smeai_b200 import q2k as Q

pytestmark = pytest.mark.gpu
QK = 256


def q8k_bytes(blocks):
    return np.ascontiguousarray(blocks).view(np.uint8).reshape(-1)


def gpu_q2k_weights(cuda, rows, k, seed, std=0.02):
    g = torch.Generator(device=cuda).manual_seed(seed)
    w = torch.randn((rows, k), generator=g, device=cuda) * std
    return Q.quantize_q2k(w)


def to_np_blocks(t, dtype):
    return t.cpu().numpy().reshape(-1).view(dtype)


# ------------------------------------------------------------------ quantizers
@pytest.mark.parametrize("rows,k", [(1, 256), (1, 4096), (3, 11008), (64, 4096)])
def test_q8k_quantize_bit_exact(cuda, oracle, rows, k):
    rng = np.random.default_rng(rows * 7 + k)
    x = rng.standard_normal((rows, k)).astype(np.float32) * np.float32(rng.uniform(0.01, 100))
    x[0, :QK] = 0.0                      # an all-zero block
    if k >= 2 * QK:
        x[0, QK:2 * QK] = 0.0
        x[0, QK + 3], x[0, QK + 9] = 1.0, -1.0   # tie in |max|: first wins
    got = Q.quantize_q8k(torch.from_numpy(x).to(cuda)).cpu().numpy().reshape(-1)
    exp = q8k_bytes(oracle.quantize_q8_K(x.reshape(-1)))
    assert np.array_equal(got, exp)


def test_q8k_quantize_strided_rows(cuda, oracle):
    rng = np.random.default_rng(2)
    x = rng.standard_normal((5, 1024 + 64)).astype(np.float32)
    t = torch.from_numpy(x).to(cuda)[:, :1024]            # ld_x = 1088
    got = Q.quantize_q8k(t).cpu().numpy().reshape(-1)
    exp = q8k_bytes(oracle.quantize_q8_K(np.ascontiguousarray(x[:, :1024]).reshape(-1)))
    assert np.array_equal(got, exp)


@pytest.mark.parametrize("rows,k", [(1, 4096), (2, 11008), (7, 2048)])
def test_rms_q8k_bit_exact(cuda, oracle, rows, k):
    rng = np.random.default_rng(k + rows)
    x = rng.standard_normal((rows, k)).astype(np.float32) * 5
    got = Q.rms_quantize_q8k(torch.from_numpy(x).to(cuda), 1e-5).cpu().numpy().reshape(rows, -1)
    for r in range(rows):
        exp = q8k_bytes(oracle.rmsnorm_quantize_q8_K(x[r], 1e-5))
        assert np.array_equal(got[r], exp), r


@pytest.mark.parametrize("rows,k", [(1, 4096), (3, 11008), (2, 512)])
def test_rms_q8k_weighted_bit_exact(cuda, oracle, rows, k):
    """RMSNorm with the reference's weight operand (sme_ai_rmsnorm_f32:
    (x * inv_rms) * weight[j], each product rounded), then Q8_K."""
    rng = np.random.default_rng(k + 3 * rows)
    x = rng.standard_normal((rows, k)).astype(np.float32) * 3
    w = (1.0 + 0.25 * rng.standard_normal(k)).astype(np.float32)
    w[:7] = 0.0                                  # zero weights: quants 0 there
    w[7] = -2.5                                  # a negative weight flips the sign
    got = Q.rms_quantize_q8k(torch.from_numpy(x).to(cuda), 1e-5,
                             norm_w=torch.from_numpy(w).to(cuda)).cpu().numpy().reshape(rows, -1)
    for r in range(rows):
        exp = q8k_bytes(oracle.rmsnorm_quantize_q8_K(x[r], 1e-5, weight=w))
        assert np.array_equal(got[r], exp), r
    # a unit weight gives the unweighted blocks
    ones = torch.ones(k, device=cuda)
    a = Q.rms_quantize_q8k(torch.from_numpy(x).to(cuda), 1e-5, norm_w=ones)
    b = Q.rms_quantize_q8k(torch.from_numpy(x).to(cuda), 1e-5)
    assert torch.equal(a, b)


def test_q2k_quantize_bit_exact(cuda, oracle):
    rng = np.random.default_rng(4)
    x = (rng.standard_normal(64 * 4096) * 0.02).astype(np.float32)
    x[:QK] = 0.0
    x[QK:2 * QK] = 0.5                    # constant block
    got = Q.quantize_q2k(torch.from_numpy(x).to(cuda).reshape(64, 4096)).cpu().numpy().reshape(-1)
    exp = q8k_bytes(oracle.quantize_q2_K(x))
    assert np.array_equal(got, exp)


def test_q2k_dequant_matches_gguf(cuda, golden):
    g = golden("q2k_gguf.npz")
    blocks = torch.from_numpy(g["blocks"].reshape(-1)).to(cuda)
    got = Q.dequantize_q2k(blocks, g["blocks"].shape[0] * QK).cpu().numpy().reshape(-1)
    assert np.array_equal(got.view(np.uint32), g["dequant"].view(np.uint32))


# ------------------------------------------------------------------ integer core
@pytest.mark.parametrize("rows,k", [(4096, 4096), (100, 512), (33, 11008)])
def test_block_sums_bit_exact(cuda, oracle, rows, k):
    wb = gpu_q2k_weights(cuda, rows, k, seed=rows + k)
    rng = np.random.default_rng(rows)
    x = rng.standard_normal(k).astype(np.float32)
    xq_np = oracle.quantize_q8_K(x)
    m = Q.Q2KMatrix(wb, rows, k)
    isum, summs = m.block_sums(torch.from_numpy(q8k_bytes(xq_np)).to(cuda))
    w_np = to_np_blocks(wb, oracle.BLOCK_Q2_K)
    nb = k // QK
    ei = np.empty((rows, nb), np.int32)
    es = np.empty((rows, nb), np.int32)
    for r in range(rows):
        ei[r], es[r] = oracle.q2k_block_sums(w_np[r * nb:(r + 1) * nb], xq_np)
    assert np.array_equal(isum.cpu().numpy(), ei)
    assert np.array_equal(summs.cpu().numpy(), es)


def test_block_sums_extreme_values(cuda, oracle):
    """Max scales/mins, all codes 3, activations at +-127: the largest sums."""
    rows, k = 32, 1024
    blk = np.zeros((rows * 4, 84), np.uint8)
    blk[:, :16] = 0xFF
    blk[:, 16:80] = 0xFF
    blk[:, 80:82] = np.frombuffer(np.float16(0.01).tobytes(), np.uint8)
    blk[:, 82:84] = np.frombuffer(np.float16(0.02).tobytes(), np.uint8)
    x = np.where(np.arange(k) % 2 == 0, 7.0, -7.0).astype(np.float32)
    x[:QK] = -7.0
    xq_np = oracle.quantize_q8_K(x)
    m = Q.Q2KMatrix(blk, rows, k)
    isum, summs = m.block_sums(torch.from_numpy(q8k_bytes(xq_np)).to(cuda))
    ei, es = oracle.q2k_block_sums(blk[:4].reshape(-1).view(oracle.BLOCK_Q2_K), xq_np)
    assert np.array_equal(isum.cpu().numpy()[0], ei) and np.array_equal(summs.cpu().numpy()[0], es)
    assert np.abs(ei).max() > 1_000_000 or np.abs(es).max() > 100_000


# ------------------------------------------------------------------ mul_mat
def _check_mul_mat(cuda, oracle, rows, k, cols, seed, threads=8):
    wb = gpu_q2k_weights(cuda, rows, k, seed)
    rng = np.random.default_rng(seed)
    x = rng.standard_normal((cols, k)).astype(np.float32)
    xq_np = oracle.quantize_q8_K(x.reshape(-1))
    m = Q.Q2KMatrix(wb, rows, k)
    y = m.mul_mat(torch.from_numpy(q8k_bytes(xq_np)).to(cuda), cols).cpu().numpy()
    exp = oracle.q2k_mul_mat(to_np_blocks(wb, oracle.BLOCK_Q2_K), rows, k, xq_np, cols,
                             combine=oracle.COMBINE_FUSED, n_threads=threads)
    return y, exp


def test_mul_mat_config2_bit_exact(cuda, oracle):
    """W[4096,4096] ~N(0,0.02) -> Q2_K, x[4096] ~N(0,1) -> Q8_K, y[4096]."""
    y, exp = _check_mul_mat(cuda, oracle, 4096, 4096, 1, seed=0)
    assert np.array_equal(y.view(np.uint32), exp.view(np.uint32))
    # and within the 1e-4 bar of the ggml-order sum with separately rounded products
    assert np.isfinite(y).all()


@pytest.mark.parametrize("cols", [1, 2, 3, 4, 5, 6, 7, 8, 11])
def test_mul_mat_token_counts(cuda, oracle, cols):
    y, exp = _check_mul_mat(cuda, oracle, 96, 2048, cols, seed=cols)
    assert np.array_equal(y.view(np.uint32), exp.view(np.uint32))


@pytest.mark.parametrize("rows,k", [(1, 256), (31, 256), (33, 768), (257, 11008)])
def test_mul_mat_ragged_shapes(cuda, oracle, rows, k):
    y, exp = _check_mul_mat(cuda, oracle, rows, k, 2, seed=rows)
    assert np.array_equal(y.view(np.uint32), exp.view(np.uint32))


def test_mul_mat_tolerance_vs_separate_rounding(cuda, oracle):
    """The other evaluation of ggml's combine (both products rounded) stays
    within the path's stated 1e-4 relative bar."""
    rows, k = 512, 4096
    wb = gpu_q2k_weights(cuda, rows, k, 9)
    x = np.random.default_rng(9).standard_normal(k).astype(np.float32)
    xq_np = oracle.quantize_q8_K(x)
    y = Q.Q2KMatrix(wb, rows, k).mul_mat(torch.from_numpy(q8k_bytes(xq_np)).to(cuda), 1).cpu().numpy()[0]
    exp = oracle.q2k_mul_mat(to_np_blocks(wb, oracle.BLOCK_Q2_K), rows, k, xq_np, 1,
                             combine=oracle.COMBINE_SEPARATE, n_threads=8)[0]
    scale = np.abs(exp).max()
    assert np.all(np.abs(y - exp) <= 1e-4 * np.maximum(np.abs(exp), 1e-3 * scale))


def test_mul_mat_residual_epilogue(cuda, oracle):
    rows, k = 200, 1024
    wb = gpu_q2k_weights(cuda, rows, k, 5)
    rng = np.random.default_rng(5)
    x = rng.standard_normal((2, k)).astype(np.float32)
    r = rng.standard_normal((2, rows)).astype(np.float32)
    xq_np = oracle.quantize_q8_K(x.reshape(-1))
    m = Q.Q2KMatrix(wb, rows, k)
    out = torch.from_numpy(r.copy()).to(cuda)
    m.mul_mat(torch.from_numpy(q8k_bytes(xq_np)).to(cuda), 2, out=out, epilogue=S.EPI_RESIDUAL, resid=out)
    exp = oracle.q2k_mul_mat(to_np_blocks(wb, oracle.BLOCK_Q2_K), rows, k, xq_np, 2) + r
    assert np.array_equal(out.cpu().numpy().view(np.uint32), exp.view(np.uint32))


def test_mul_mat_silu_mul_epilogue(cuda, oracle):
    hidden, k = 300, 1024
    wg = gpu_q2k_weights(cuda, hidden, k, 21)
    wu = gpu_q2k_weights(cuda, hidden, k, 22)
    inter = torch.stack([wg, wu], dim=1).reshape(2 * hidden, -1)   # rows g0,u0,g1,u1,...
    rng = np.random.default_rng(6)
    x = rng.standard_normal((3, k)).astype(np.float32)
    xq_np = oracle.quantize_q8_K(x.reshape(-1))
    m = Q.Q2KMatrix(inter, 2 * hidden, k)
    h = m.mul_mat(torch.from_numpy(q8k_bytes(xq_np)).to(cuda), 3, epilogue=S.EPI_SILU_MUL).cpu().numpy()
    g = oracle.q2k_mul_mat(to_np_blocks(wg, oracle.BLOCK_Q2_K), hidden, k, xq_np, 3)
    u = oracle.q2k_mul_mat(to_np_blocks(wu, oracle.BLOCK_Q2_K), hidden, k, xq_np, 3)
    exp = oracle.silu_mul(g.reshape(-1), u.reshape(-1)).reshape(3, hidden)
    assert h.shape == (3, hidden)
    assert np.all(np.abs(h - exp) <= 1e-5 * np.abs(exp) + 1e-30)


def test_mul_mat_f32_entry(cuda, oracle):
    rows, k = 128, 2048
    wb = gpu_q2k_weights(cuda, rows, k, 31)
    x = np.random.default_rng(31).standard_normal((3, k)).astype(np.float32)
    m = Q.Q2KMatrix(wb, rows, k)
    y = m.mul_mat_f32(torch.from_numpy(x).to(cuda)).cpu().numpy()
    exp = oracle.q2k_mul_mat(to_np_blocks(wb, oracle.BLOCK_Q2_K), rows, k,
                             oracle.quantize_q8_K(x.reshape(-1)), 3)
    assert np.array_equal(y.view(np.uint32), exp.view(np.uint32))


def test_full_size_linearity_exact(cuda):
    """Q8_K(2x) has the same quants and twice the scale, so every float in the
    combine doubles exactly: y(2x) == 2*y(x) bit for bit at the SwiGLU shape."""
    rows, k = 11008, 4096
    wb = gpu_q2k_weights(cuda, rows, k, 77)
    m = Q.Q2KMatrix(wb, rows, k)
    x = torch.randn((8, k), generator=torch.Generator(device=cuda).manual_seed(1), device=cuda)
    y1 = m.mul_mat(Q.quantize_q8k(x), 8)
    y2 = m.mul_mat(Q.quantize_q8k(2 * x), 8)
    assert torch.equal(y2, 2 * y1)
    assert torch.isfinite(y1).all()


# ------------------------------------------------------------------ ggml-shaped
def test_ggml_shaped_entry_points(cuda, oracle):
    L = S.lib()
    rng = np.random.default_rng(12)
    k = 2048
    x = rng.standard_normal(k).astype(np.float32)
    y = np.zeros(k // QK * 292, np.uint8)
    L.quantize_row_q8_K(x.ctypes.data, y.ctypes.data, k)
    assert np.array_equal(y, q8k_bytes(oracle.quantize_q8_K(x)))
    w = (rng.standard_normal(k) * 0.02).astype(np.float32)
    wq = np.zeros(k // QK * 84, np.uint8)
    L.quantize_row_q2_K(w.ctypes.data, wq.ctypes.data, k)
    assert np.array_equal(wq, q8k_bytes(oracle.quantize_q2_K(w)))
    deq = np.zeros(k, np.float32)
    L.dequantize_row_q2_K(wq.ctypes.data, deq.ctypes.data, k)
    assert np.array_equal(deq, oracle.dequantize_q2_K(wq.view(oracle.BLOCK_Q2_K)))
    s = ctypes.c_float(-1.0)
    L.ggml_vec_dot_q2_K_q8_K(k, ctypes.byref(s), 0, wq.ctypes.data, 0, y.ctypes.data, 0, 1)
    exp = oracle.vec_dot_q2_K_q8_K(wq.view(oracle.BLOCK_Q2_K), y.view(oracle.BLOCK_Q8_K))
    assert np.float32(s.value).view(np.uint32) == np.float32(exp).view(np.uint32)
    # nrc != 1 is refused (ggml never asks for it with Q2_K): result zeroed
    L.ggml_vec_dot_q2_K_q8_K(k, ctypes.byref(s), 0, wq.ctypes.data, 0, y.ctypes.data, 0, 2)
    assert s.value == 0.0 and "nrc" in S.last_error()


def test_coarse_api_errors(cuda):
    L = S.lib()
    wb = gpu_q2k_weights(cuda, 64, 512, 3)
    m = Q.Q2KMatrix(wb, 64, 512)
    xq = torch.zeros(2 * 292, dtype=torch.uint8, device=cuda)
    y = torch.zeros(64, device=cuda)
    st = L.smeai_q2k_mul_mat(m.handle, 65, 512, ctypes.c_void_p(xq.data_ptr()), 1,
                             ctypes.c_void_p(y.data_ptr()), 64, None)
    assert st == S.SME_AI_BAD_ARGUMENT and "does not match" in S.last_error()
    st = L.smeai_q2k_mul_mat_ex(m.handle, ctypes.c_void_p(xq.data_ptr()), 1, ctypes.c_void_p(y.data_ptr()), 64,
                                S.EPI_RESIDUAL, None, 64, None)
    assert st == S.SME_AI_BAD_ARGUMENT
    st = L.smeai_q2k_mul_mat(m.handle, 64, 512, ctypes.c_void_p(xq.data_ptr()), 1,
                             ctypes.c_void_p(y.data_ptr()), 10, None)
    assert st == S.SME_AI_BAD_ARGUMENT
    m.free()
    torch.cuda.synchronize()


# ------------------------------------------------------------------ fused fp32-input GEMV
@pytest.mark.parametrize("rows,k,cols", [(4096, 4096, 1), (128, 11008, 3), (300, 2048, 8), (64, 256, 5)])
def test_fused_prologue_bit_identical(cuda, rows, k, cols):
    """Quantizing in the GEMV prologue (with and without RMSNorm, strided rows)
    gives exactly the two-kernel result; the cluster split (4096 rows -> 128
    groups) and the unsplit path agree too."""
    wb = gpu_q2k_weights(cuda, rows, k, rows + cols)
    m = Q.Q2KMatrix(wb, rows, k)
    g = torch.Generator(device=cuda).manual_seed(cols)
    xs = torch.randn((cols, k + 64), generator=g, device=cuda) * 3
    x = xs[:, :k]                                  # row stride k + 64
    y_two = m.mul_mat(Q.quantize_q8k(x.contiguous()), cols)
    y_one = m.mul_mat_f32_ex(x, cols)
    assert torch.equal(y_one, y_two)
    y_two = m.mul_mat(Q.rms_quantize_q8k(x.contiguous(), 1e-5), cols)
    y_one = m.mul_mat_f32_ex(x, cols, rms_eps=1e-5)
    assert torch.equal(y_one, y_two)
    r = torch.randn((cols, rows), generator=g, device=cuda)
    y_res = m.mul_mat_f32_ex(x, cols, out=r.clone(), epilogue=S.EPI_RESIDUAL, resid=r, rms_eps=1e-5)
    assert torch.equal(y_res, r + y_two)
    nw = 1.0 + 0.3 * torch.randn(k, generator=g, device=cuda)       # RMSNorm weight
    y_two = m.mul_mat(Q.rms_quantize_q8k(x.contiguous(), 1e-5, norm_w=nw), cols)
    y_one = m.mul_mat_f32_ex(x, cols, rms_eps=1e-5, norm_w=nw)
    assert torch.equal(y_one, y_two)
    assert torch.equal(m.mul_mat_f32(x.contiguous()), m.mul_mat(Q.quantize_q8k(x.contiguous()), cols))


def test_fused_silu_epilogue_matches_two_kernel(cuda):
    hidden, k = 1000, 4096
    wg = gpu_q2k_weights(cuda, hidden, k, 41)
    wu = gpu_q2k_weights(cuda, hidden, k, 42)
    m = Q.Q2KMatrix(torch.stack([wg, wu], 1).reshape(2 * hidden, -1), 2 * hidden, k)
    x = torch.randn((2, k), generator=torch.Generator(device=cuda).manual_seed(4), device=cuda)
    h1 = m.mul_mat_f32_ex(x, 2, epilogue=S.EPI_SILU_MUL, rms_eps=1e-5)
    h2 = m.mul_mat(Q.rms_quantize_q8k(x, 1e-5), 2, epilogue=S.EPI_SILU_MUL)
    assert torch.equal(h1, h2)


@pytest.mark.parametrize("rows,k,cols", [(148 * 4 * 32 + 40, 512, 1), (148 * 3 * 32, 256, 4), (600 * 32, 768, 2)])
def test_mul_mat_many_row_groups_per_cta(cuda, oracle, rows, k, cols):
    """More 32-row groups than SMs: each persistent CTA walks several groups
    through the double-buffered terms (and a ring shorter than its stages)."""
    y, exp = _check_mul_mat(cuda, oracle, rows, k, cols, seed=rows % 97, threads=16)
    assert np.array_equal(y.view(np.uint32), exp.view(np.uint32))


def test_no_device_error_recorded(cuda):
    """Every bounded wait in the GEMV completed: the device error word is clear."""
    import ctypes as C
    L = S.lib()
    code = C.c_uint(0)
    assert L.smeai_take_device_error(C.byref(code)) == 0
    assert code.value == 0
