"""The tensor-core prefill GEMM (tcgen05.mma, kind::f16 on exact small-integer
operands, TMEM accumulators) against the CPU oracle and the GEMV: outputs must
be bit-identical (integer super-block sums are exact; ggml's combine runs in
ascending super-block order)."""
import numpy as np
import pytest
import torch

import smeai_b200 as S
from smeai_b200 import q2k as Q

pytestmark = pytest.mark.gpu


def _weights(cuda, rows, k, seed):
    g = torch.Generator(device=cuda).manual_seed(seed)
    return Q.quantize_q2k(torch.randn((rows, k), generator=g, device=cuda) * 0.02)


@pytest.mark.parametrize("rows,k,cols", [(128, 256, 1), (128, 256, 128), (300, 512, 20), (256, 4096, 130),
                                         (96, 11008, 16), (1000, 768, 257)])
def test_gemm_tc_bit_exact_vs_oracle(cuda, oracle, rows, k, cols):
    wb = _weights(cuda, rows, k, rows + cols)
    rng = np.random.default_rng(cols)
    x = rng.standard_normal((cols, k)).astype(np.float32) * 2
    xq_np = oracle.quantize_q8_K(x.reshape(-1))
    m = Q.Q2KMatrix(wb, rows, k)
    xq = torch.from_numpy(np.ascontiguousarray(xq_np).view(np.uint8)).to(cuda)
    y = m.mul_mat_tc(xq, cols).cpu().numpy()
    exp = oracle.q2k_mul_mat(wb.cpu().numpy().reshape(-1).view(oracle.BLOCK_Q2_K), rows, k, xq_np, cols,
                             n_threads=16)
    assert np.array_equal(y.view(np.uint32), exp.view(np.uint32))
    if cols >= 16:   # the default mul_mat entry takes the tensor-core path here
        assert torch.equal(m.mul_mat(xq, cols), torch.from_numpy(y).to(cuda))


def test_gemm_tc_prefill_shape_matches_gemv(cuda, oracle):
    """Config 4: activations [512, 4096] x W[11008, 4096] -> [512, 11008]:
    the tensor-core result equals the GEMV's bit for bit, and the oracle's on a
    sample of rows."""
    rows, k, cols = 11008, 4096, 512
    wb = _weights(cuda, rows, k, 4)
    x = torch.randn((cols, k), generator=torch.Generator(device=cuda).manual_seed(5), device=cuda)
    xq = Q.quantize_q8k(x)
    m = Q.Q2KMatrix(wb, rows, k)
    y_tc = m.mul_mat_tc(xq, cols)
    y_gv = torch.empty_like(y_tc)
    for c0 in range(0, cols, 8):
        m.mul_mat(xq[c0:c0 + 8], 8, out=y_gv[c0:c0 + 8])
    assert torch.equal(y_tc, y_gv)
    nb = k // 256
    sel = np.arange(0, rows, 997)
    w_np = wb.cpu().numpy().reshape(rows, -1)[sel].reshape(-1).view(oracle.BLOCK_Q2_K)
    xq_np = xq.cpu().numpy().reshape(-1).view(oracle.BLOCK_Q8_K)
    exp = oracle.q2k_mul_mat(w_np, len(sel), k, xq_np, cols, n_threads=16)
    got = y_tc.cpu().numpy()[:, sel]
    assert np.array_equal(np.ascontiguousarray(got).view(np.uint32), exp.view(np.uint32))


def test_gemm_tc_zz_no_device_error(cuda):
    import ctypes
    code = ctypes.c_uint(0)
    assert S.lib().smeai_take_device_error(ctypes.byref(code)) == 0
    assert code.value == 0
