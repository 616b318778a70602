"""Q6_K oracle (CPU restatement of ggml's generic Q6_K decode and dot),
pinned against gguf-py's decoder and checked for internal consistency."""
import numpy as np
import pytest

QK = 256


def test_q6k_decode_matches_gguf_py(oracle, golden):
    g = golden("q6k_gguf.npz")
    blocks = g["blocks"].reshape(-1).view(oracle.BLOCK_Q6_K)
    assert np.array_equal(oracle.dequantize_q6_K(blocks), g["dequant"])


@pytest.mark.parametrize("nb", [1, 16, 43])
def test_q6k_integer_sums_match_numpy(oracle, nb):
    rng = np.random.default_rng(nb + 100)
    blocks = oracle.random_q6_K(rng, nb)
    xq = oracle.quantize_q8_K(rng.standard_normal(nb * QK).astype(np.float32) * 3)
    isum = oracle.q6k_block_sums(blocks, xq)
    deq = oracle.dequantize_q6_K(blocks).reshape(nb, 16, 16).astype(np.float64)
    d = blocks["d"].view(np.float16).astype(np.float64)
    for b in range(nb):
        sc = blocks[b]["scales"].astype(np.int64)
        q8 = xq[b]["qs"].astype(np.int64).reshape(16, 16)
        tot = 0
        for j in range(16):
            if sc[j] == 0:
                continue
            q = np.rint(deq[b, j] / (d[b] * sc[j])).astype(np.int64)
            assert np.all((q >= -32) & (q <= 31))
            tot += sc[j] * int((q * q8[j]).sum())
        assert isum[b] == tot


def test_q6k_combines_agree_within_tolerance(oracle):
    rng = np.random.default_rng(9)
    rows, k, cols = 40, 4096, 2
    w = oracle.random_q6_K(rng, rows * k // QK)
    xq = oracle.quantize_q8_K(rng.standard_normal(cols * k).astype(np.float32))
    ggml = oracle.q6k_mul_mat(w, rows, k, xq, cols, oracle.Q3K_GGML)
    blk = oracle.q6k_mul_mat(w, rows, k, xq, cols, oracle.Q3K_BLOCK_ORDER)
    assert np.abs(ggml - blk).max() <= 1e-5 * np.abs(ggml).max()
