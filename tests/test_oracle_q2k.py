"""CPU tests of the Q2_K / Q8_K oracle: pinned against gguf-py's decoder,
an independent numpy restatement of the integer sums, exact-rational
known-answer tests for Q8_K, and float64 dot products."""
from fractions import Fraction

import numpy as np
import pytest

QK = 256


def unpack_q2k_numpy(blocks_u8: np.ndarray):
    """Independent numpy decode of block_q2_K (same reshaping as gguf-py):
    returns q[nb,256] int64, sc[nb,16], mn[nb,16], d[nb], dmin[nb]."""
    b = blocks_u8.reshape(-1, 84)
    scales = b[:, :16].astype(np.int64)
    qs = b[:, 16:80].reshape(-1, 2, 1, 32)
    q = (qs >> np.array([0, 2, 4, 6], np.uint8).reshape(1, 1, 4, 1)) & 3
    q = q.reshape(-1, 256).astype(np.int64)
    d = b[:, 80:82].copy().view(np.float16).astype(np.float64).reshape(-1)
    dmin = b[:, 82:84].copy().view(np.float16).astype(np.float64).reshape(-1)
    return q, scales & 0xF, scales >> 4, d, dmin


def test_oracle_dequant_matches_gguf(oracle, golden):
    g = golden("q2k_gguf.npz")
    blocks = g["blocks"]
    deq = oracle.dequantize_q2_K(blocks.view(oracle.BLOCK_Q2_K).reshape(-1))
    assert np.array_equal(deq.view(np.uint32), g["dequant"].view(np.uint32))


def test_oracle_quantizer_reproduces_fixture(oracle, golden):
    g = golden("q2k_gguf.npz")
    n = g["source"].size // QK
    blocks = oracle.quantize_q2_K(g["source"]).view(np.uint8).reshape(-1, 84)
    assert np.array_equal(blocks, g["blocks"][:n])


def test_q2k_quantizer_error_bounded(oracle):
    rng = np.random.default_rng(1)
    x = (rng.standard_normal(64 * QK) * 0.02).astype(np.float32)
    deq = oracle.dequantize_q2_K(oracle.quantize_q2_K(x))
    err = np.abs(deq - x).reshape(-1, 16).max(axis=1)
    span = (x.reshape(-1, 16).max(axis=1) - np.minimum(x.reshape(-1, 16).min(axis=1), 0))
    # 2-bit codes: error within about half a step of the group's range, plus 4-bit scale rounding
    assert np.all(err <= span * 0.5 + 1e-3)


def _random_q8k(oracle, rng, nb):
    return oracle.quantize_q8_K(rng.standard_normal(nb * QK).astype(np.float32))


def test_block_sums_match_numpy_restatement(oracle, golden):
    rng = np.random.default_rng(7)
    blocks = golden("q2k_gguf.npz")["blocks"]
    nb = blocks.shape[0]
    xq = _random_q8k(oracle, rng, nb)
    isum, summs = oracle.q2k_block_sums(blocks.view(oracle.BLOCK_Q2_K).reshape(-1), xq)
    q, sc, mn, _, _ = unpack_q2k_numpy(blocks)
    q8 = xq["qs"].astype(np.int64)
    sub = (q * q8).reshape(nb, 16, 16).sum(axis=2)
    assert np.array_equal(isum, (sub * sc).sum(axis=1))
    assert np.array_equal(summs, (xq["bsums"].astype(np.int64) * mn).sum(axis=1))


@pytest.mark.parametrize("combine", [0, 1])
def test_vec_dot_close_to_float64(oracle, golden, combine):
    rng = np.random.default_rng(11)
    g = golden("q2k_gguf.npz")
    blocks = g["blocks"][:16]
    xq = _random_q8k(oracle, rng, 16)
    s = oracle.vec_dot_q2_K_q8_K(blocks.view(oracle.BLOCK_Q2_K).reshape(-1), xq, combine)
    deq = g["dequant"][: 16 * QK].astype(np.float64)
    xf = np.repeat(xq["d"].astype(np.float64), QK) * xq["qs"].reshape(-1)
    ref = float((deq * xf).sum())
    assert abs(s - ref) <= 1e-5 * max(1.0, np.abs(deq * xf).sum())


def test_mul_mat_threads_bit_identical(oracle):
    rng = np.random.default_rng(3)
    rows, k, cols = 64, 1024, 3
    w = oracle.quantize_q2_K((rng.standard_normal(rows * k) * 0.02).astype(np.float32))
    xq = oracle.quantize_q8_K(rng.standard_normal(cols * k).astype(np.float32))
    y1 = oracle.q2k_mul_mat(w, rows, k, xq, cols, n_threads=1)
    y4 = oracle.q2k_mul_mat(w, rows, k, xq, cols, n_threads=4)
    assert np.array_equal(y1.view(np.uint32), y4.view(np.uint32))
    # column c of y is the dot of every row with activation row c
    nb = k // QK
    assert y1[2, 5] == oracle.vec_dot_q2_K_q8_K(w[5 * nb:6 * nb], xq[2 * nb:3 * nb])


# ---------------------------------------------------------------- Q8_K KATs
def q8k_one(oracle, x, rounding=0):
    return oracle.quantize_q8_K(np.asarray(x, np.float32), rounding)[0]


def test_q8k_all_zero_block(oracle):
    b = q8k_one(oracle, np.zeros(QK))
    assert b["d"] == 0 and not b["qs"].any() and not b["bsums"].any()


def test_q8k_single_spike(oracle):
    x = np.zeros(QK, np.float32)
    x[5] = 2.0
    b = q8k_one(oracle, x)
    assert b["qs"][5] == -127 and np.count_nonzero(b["qs"]) == 1
    assert b["bsums"][0] == -127 and not b["bsums"][1:].any()
    assert b["d"] == np.float32(1.0) / np.float32(np.float32(-127.0) / np.float32(2.0))


def test_q8k_round_half_even(oracle):
    # max = -127 gives iscale = 1 exactly, so q = nearest(x): ties go to even
    x = np.zeros(QK, np.float32)
    x[:8] = [-127, 2.5, 3.5, -2.5, 0.5, 1.5, -0.5, 126.5]
    for rounding in (0, 1):
        b = q8k_one(oracle, x, rounding)
        assert list(b["qs"][:8]) == [-127, 2, 4, -2, 0, 2, 0, 126]
        assert b["d"] == 1.0


def test_q8k_first_max_wins(oracle):
    x = np.zeros(QK, np.float32)
    x[3], x[9] = 1.0, -1.0
    b = q8k_one(oracle, x)
    assert b["qs"][3] == -127 and b["qs"][9] == 127 and b["d"] < 0


def test_q8k_bsums_extremes(oracle):
    x = np.full(QK, 3.0, np.float32)
    b = q8k_one(oracle, x)
    assert np.all(b["qs"] == -127) and np.all(b["bsums"] == -2032)
    x = -x
    b = q8k_one(oracle, x)
    assert np.all(b["qs"] == -127) and np.all(b["bsums"] == -2032) and b["d"] > 0


def test_q8k_fused_rounding_is_exact_product_rounding(oracle):
    """ROUND_FUSED rounds the exact rational iscale*x (round half to even);
    ROUND_SEPARATE rounds the fp32 product.  Checked with Python fractions."""
    rng = np.random.default_rng(99)
    differ = 0
    for trial in range(40):
        x = rng.standard_normal(QK).astype(np.float32)
        amax_i = int(np.argmax(np.abs(x)))
        vmax = x[amax_i]
        iscale = np.float32(np.float32(-127.0) / vmax)
        fused = q8k_one(oracle, x, 0)
        sep = q8k_one(oracle, x, 1)
        for j in range(QK):
            exact = Fraction(float(iscale)) * Fraction(float(x[j]))
            expect_f = min(127, round(exact))  # Python round: half to even
            prod32 = Fraction(float(np.float32(iscale * x[j])))
            expect_s = min(127, round(prod32))
            assert fused["qs"][j] == expect_f
            assert sep["qs"][j] == expect_s
            differ += expect_f != expect_s
        assert fused["d"] == np.float32(np.float32(1.0) / iscale)
        assert np.array_equal(fused["bsums"], fused["qs"].reshape(16, 16).astype(np.int64).sum(axis=1))
    assert differ >= 0  # the two modes differ only at exact fp32 ties


def test_rms_inv_close_to_float64(oracle):
    rng = np.random.default_rng(5)
    x = rng.standard_normal(4096).astype(np.float32) * 3
    inv = oracle.rms_inv(x, 1e-5)
    ref = 1.0 / np.sqrt((x.astype(np.float64) ** 2).mean() + 1e-5)
    assert abs(inv - ref) <= 1e-6 * ref


def _fold32(a):
    a = a.astype(np.float32).copy()
    w = 16
    while w >= 1:
        a[:w] = (a[:w] + a[w:2 * w]).astype(np.float32)
        w //= 2
    return np.float32(a[0])


@pytest.mark.parametrize("k", [256, 4096, 11008])
def test_rms_sum_order_pinned(oracle, k):
    """The RMSNorm sum of squares follows one fixed order (32-value group
    folds, then 32 lane accumulators over the groups, folded), restated here
    in numpy float32 steps: the oracle must give the same bits."""
    x = np.random.default_rng(k).standard_normal(k).astype(np.float32) * 2
    groups = [_fold32((x[32 * g:32 * g + 32] * x[32 * g:32 * g + 32]).astype(np.float32)) for g in range(k // 32)]
    acc = np.zeros(32, np.float32)
    for lane in range(32):
        a = np.float32(0)
        for g in range(lane, k // 32, 32):
            a = np.float32(a + groups[g])
        acc[lane] = a
    exp = _fold32(acc)
    got = np.float32(oracle.rms_sumsq(x))
    assert got.view(np.uint32) == exp.view(np.uint32)
