"""GPU parity of the Q6_K x Q8_K path (smeai_q6k_*) against the CPU oracle,
through the C-ABI.

Bar: the block decode is bit-exact with gguf-py's decoder (golden fixture);
the per-(row, super-block) integer sums are bit-exact with the oracle's
restatement of ggml's loop; mul_mat outputs are bit-exact with the oracle's
block-order combine and within 1e-5 of max|y| of ggml's generic 8-lane
combine (the same integers, floats accumulated in a different order;
the integers can exceed 2^24, so their conversion to float rounds too).
"""
import ctypes

import numpy as np
import pytest
import torch

import smeai_b200 as S
from smeai_b200 import q2k as Q

pytestmark = pytest.mark.gpu
QK = 256


def _xq(oracle, rng, cols, k):
    x = rng.standard_normal((cols, k)).astype(np.float32) * 2
    return x, np.concatenate([oracle.quantize_q8_K(x[c]) for c in range(cols)])


def test_q6k_decode_matches_gguf_py(cuda, oracle, golden):
    g = golden("q6k_gguf.npz")
    blocks = g["blocks"]
    t = torch.from_numpy(blocks.reshape(-1).copy()).to(cuda)
    y = Q.dequantize_q6k(t, blocks.shape[0] * QK).cpu().numpy()
    assert np.array_equal(y, g["dequant"])
    host = np.empty(blocks.shape[0] * QK, np.float32)
    S.lib().dequantize_row_q6_K(blocks.ctypes.data, host.ctypes.data, host.size)
    assert np.array_equal(host, g["dequant"])


@pytest.mark.parametrize("rows,k", [(32, 256), (77, 1024), (256, 11008)])
def test_q6k_block_sums_bit_exact(cuda, oracle, rows, k):
    rng = np.random.default_rng(rows + k)
    nb = k // QK
    w = oracle.random_q6_K(rng, rows * nb)
    _, xq = _xq(oracle, rng, 1, k)
    m = Q.Q6KMatrix(w, rows, k)
    isum, summs = m.block_sums(torch.from_numpy(xq.view(np.uint8).copy()).to(cuda))
    exp = np.stack([oracle.q6k_block_sums(w[r * nb:(r + 1) * nb], xq) for r in range(rows)])
    assert np.array_equal(isum.cpu().numpy(), exp)
    # summs = sum_j scale_j * bsums_j
    exp_m = np.array([[int((w[r * nb + b]["scales"].astype(np.int64) *
                            xq[b]["bsums"].astype(np.int64)).sum()) for b in range(nb)] for r in range(rows)])
    assert np.array_equal(summs.cpu().numpy(), exp_m)
    m.free()


@pytest.mark.parametrize("rows,k,cols", [(32, 256, 1), (100, 1024, 3), (4096, 4096, 1), (4096, 11008, 8),
                                         (300, 2048, 17)])
def test_q6k_mul_mat_matches_oracle(cuda, oracle, rows, k, cols):
    rng = np.random.default_rng(rows * 3 + cols)
    w = oracle.random_q6_K(rng, rows * k // QK)
    x, xq = _xq(oracle, rng, cols, k)
    m = Q.Q6KMatrix(w, rows, k)
    y = m.mul_mat(torch.from_numpy(xq.view(np.uint8).copy()).to(cuda), cols).cpu().numpy()
    blk = oracle.q6k_mul_mat(w, rows, k, xq, cols, oracle.Q3K_BLOCK_ORDER, n_threads=8)
    assert np.array_equal(y, blk)
    ggml = oracle.q6k_mul_mat(w, rows, k, xq, cols, oracle.Q3K_GGML, n_threads=8)
    assert np.abs(y - ggml).max() <= 1e-5 * np.abs(ggml).max()
    # fp32 activations quantized inside the kernel: the same bits
    yf = m.mul_mat_f32(torch.from_numpy(x).to(cuda)).cpu().numpy()
    assert np.array_equal(yf, y)
    m.free()


def test_q6k_ggml_shaped_vec_dot(cuda, oracle):
    rng = np.random.default_rng(11)
    k = 4096
    w = oracle.random_q6_K(rng, k // QK)
    _, xq = _xq(oracle, rng, 1, k)
    s = ctypes.c_float()
    S.lib().ggml_vec_dot_q6_K_q8_K(k, ctypes.byref(s), 0, w.ctypes.data, 0, xq.ctypes.data, 0, 1)
    assert s.value == oracle.vec_dot_q6_K_q8_K(w, xq, oracle.Q3K_BLOCK_ORDER)


def test_formats_are_not_mixed(cuda, oracle):
    rng = np.random.default_rng(3)
    w3 = Q.Q6KMatrix(oracle.random_q6_K(rng, 32), 32, 256)
    w2 = Q.Q2KMatrix(oracle.quantize_q2_K(rng.standard_normal(32 * 256).astype(np.float32) * 0.02), 32, 256)
    xq = torch.from_numpy(oracle.quantize_q8_K(rng.standard_normal(256).astype(np.float32)).view(np.uint8)
                          .copy()).to(cuda)
    y = torch.empty((1, 32), device=cuda)
    assert S.lib().smeai_q2k_mul_mat(w3.handle, 32, 256, Q._ptr(xq), 1, Q._ptr(y), 32, None) != 0
    assert "Q6_K" in S.last_error()
    assert S.lib().smeai_q6k_mul_mat(w2.handle, Q._ptr(xq), 1, Q._ptr(y), 32, None) != 0
    assert "Q2_K" in S.last_error()
    w2.free()
    w3.free()


def test_gguf_q6k_tensor(tmp_path, cuda, oracle):
    import gguf
    from smeai_b200 import gguf as G
    rng = np.random.default_rng(5)
    rows, k = 64, 1024
    w = oracle.random_q6_K(rng, rows * k // QK)
    path = tmp_path / "q3.gguf"
    wr = gguf.GGUFWriter(str(path), arch="llama")
    wr.add_tensor("blk.0.ffn_down.weight", w.view(np.uint8).reshape(rows, -1),
                  raw_dtype=gguf.GGMLQuantizationType.Q6_K)
    wr.write_header_to_file()
    wr.write_kv_data_to_file()
    wr.write_tensors_to_file()
    wr.close()
    _, xq = _xq(oracle, rng, 2, k)
    with G.GGUFFile(path) as f:
        assert f.by_name["blk.0.ffn_down.weight"].ggml_type == G.GGML_Q6_K
        m = f.load_q6k("blk.0.ffn_down.weight")
        with pytest.raises(S.SmeaiError):
            f.load_q2k("blk.0.ffn_down.weight")
    y = m.mul_mat(torch.from_numpy(xq.view(np.uint8).copy()).to(cuda), 2).cpu().numpy()
    assert np.array_equal(y, oracle.q6k_mul_mat(w, rows, k, xq, 2, oracle.Q3K_BLOCK_ORDER))
    m.free()
