"""Q3_K oracle (CPU restatement of ggml's generic Q3_K decode and dot),
pinned against gguf-py's independent decoder and checked for internal
consistency: integer sums against numpy, both float combines against the
decoded weights."""
import numpy as np
import pytest

QK = 256


def test_q3k_decode_matches_gguf_py(oracle, golden):
    g = golden("q3k_gguf.npz")
    blocks = g["blocks"].reshape(-1).view(oracle.BLOCK_Q3_K)
    assert np.array_equal(oracle.dequantize_q3_K(blocks), g["dequant"])


def test_q3k_scales_known_answers(oracle, golden):
    blocks = golden("q3k_gguf.npz")["blocks"].reshape(-1).view(oracle.BLOCK_Q3_K)
    assert np.array_equal(oracle.q3k_scales(blocks[-2]), np.full(16, -32, np.int8))  # all-zero block
    ext = oracle.q3k_scales(blocks[-1])
    # bytes 0..7 = 00 FF 0F F0 00 FF 0F F0, bytes 8..11 = 00 FF 1B E4
    lo = [0x0, 0xF, 0xF, 0x0, 0x0, 0xF, 0xF, 0x0, 0x0, 0xF, 0x0, 0xF, 0x0, 0xF, 0x0, 0xF]
    hb = [0x00, 0xFF, 0x1B, 0xE4]
    hi = [(hb[j % 4] >> (2 * (j // 4))) & 3 for j in range(16)]
    assert ext.tolist() == [(lo[j] | (hi[j] << 4)) - 32 for j in range(16)]


@pytest.mark.parametrize("nb", [1, 4, 16, 43])
def test_q3k_integer_sums_match_numpy(oracle, nb):
    rng = np.random.default_rng(nb)
    blocks = oracle.random_q3_K(rng, nb)
    x = rng.standard_normal(nb * QK).astype(np.float32) * 3
    xq = oracle.quantize_q8_K(x)
    isum = oracle.q3k_block_sums(blocks, xq)
    # independent: integer weights from the decoded values (d * sc * q, exact
    # in fp32) divided back by d * sc, then an int64 dot per sub-block
    deq = oracle.dequantize_q3_K(blocks).reshape(nb, 16, 16).astype(np.float64)
    d = blocks["d"].view(np.float16).astype(np.float64)
    for b in range(nb):
        sc = oracle.q3k_scales(blocks[b]).astype(np.int64)
        q8 = xq[b]["qs"].astype(np.int64).reshape(16, 16)
        tot = 0
        for j in range(16):
            if sc[j] == 0 or d[b] == 0:
                continue  # q unrecoverable from the decode; the term is 0 either way
            q = np.rint(deq[b, j] / (d[b] * sc[j])).astype(np.int64)
            assert np.all((q >= -4) & (q <= 3))
            tot += sc[j] * int((q * q8[j]).sum())
        assert isum[b] == tot


def test_q3k_combines_agree_within_tolerance(oracle):
    rng = np.random.default_rng(7)
    rows, k, cols = 48, 4096, 3
    w = oracle.random_q3_K(rng, rows * k // QK)
    xq = oracle.quantize_q8_K(rng.standard_normal(cols * k).astype(np.float32))
    ggml = oracle.q3k_mul_mat(w, rows, k, xq, cols, oracle.Q3K_GGML)
    blk = oracle.q3k_mul_mat(w, rows, k, xq, cols, oracle.Q3K_BLOCK_ORDER)
    ref = (oracle.dequantize_q3_K(w).reshape(rows, k).astype(np.float64) @
           np.stack([(xq[c * 16:(c + 1) * 16]["qs"].astype(np.float64) *
                      xq[c * 16:(c + 1) * 16]["d"].astype(np.float64)[:, None]).reshape(-1)
                     for c in range(cols)]).T).T
    scale = np.abs(ref).max()
    assert np.abs(ggml - ref).max() <= 1e-5 * scale
    assert np.abs(blk - ref).max() <= 1e-5 * scale
    assert np.abs(ggml - blk).max() <= 1e-5 * scale
