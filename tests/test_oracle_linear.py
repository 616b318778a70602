"""CPU tests of the fp16 Linear / MLP / SwiGLU oracle (Path A)."""
import numpy as np

from golden.make_golden import lcg_py


def test_lcg_generator_matches_python_restatement(oracle, golden):
    g = golden("lcg.npz")
    for seed, count in ((1001, 8 * 128), (1002, 128 * 128), (1003, 128)):
        assert np.array_equal(oracle.lcg_f32(count, seed), g[f"f32_{seed}"])
        assert np.array_equal(oracle.lcg_f16(count, seed), g[f"f16_{seed}"])
    assert np.array_equal(lcg_py(16, 1001), g["f32_1001"][:16])


def test_demo_linear_exact(oracle, golden):
    g = golden("demo_linear.npz")
    out = oracle.linear_f16f32(g["x16"], 2, 16, g["w16"], 16, g["bias"])
    assert np.array_equal(out, g["expected"])


def test_linear_close_to_float64(oracle, golden):
    g = golden("lcg.npz")
    x16, w16, b = g["f16_1001"], g["f16_1002"], g["f32_1003"]
    out = oracle.linear_f16f32(x16, 8, 128, w16, 128, b)
    x = x16.view(np.float16).astype(np.float64).reshape(8, 128)
    w = w16.view(np.float16).astype(np.float64).reshape(128, 128)
    ref = x @ w + b.astype(np.float64)
    assert np.abs(out - ref).max() <= 1e-5


def test_linear_f32_matches_sequential_fma(oracle):
    rng = np.random.default_rng(0)
    x = rng.standard_normal((3, 40)).astype(np.float32)
    w = rng.standard_normal((40, 5)).astype(np.float32)
    out = oracle.linear_f32f32(x, 3, 40, w, 5)
    ref = x.astype(np.float64) @ w.astype(np.float64)
    assert np.abs(out - ref).max() <= 1e-5 * np.abs(ref).max()


def test_activations(oracle):
    x16 = np.array([0x3C00, 0xBC00], np.uint16)  # +1, -1
    w16 = np.array([0x3C00], np.uint16)          # 1x1 weight = 1
    relu = oracle.linear_f16f32(x16, 2, 1, w16, 1, act=oracle.ACT_RELU)
    assert list(relu[:, 0]) == [1.0, 0.0]
    silu = oracle.linear_f16f32(x16, 2, 1, w16, 1, act=oracle.ACT_SILU)
    assert np.allclose(silu[:, 0], [1 / (1 + np.exp(-1)), -1 / (1 + np.exp(1))], rtol=1e-6)
    gelu = oracle.linear_f16f32(x16, 2, 1, w16, 1, act=oracle.ACT_GELU)
    ref = [0.5 * v * (1 + np.tanh(0.7978845608 * (v + 0.044715 * v ** 3))) for v in (1.0, -1.0)]
    assert np.allclose(gelu[:, 0], ref, rtol=1e-6)


def test_swiglu_matches_numpy(oracle):
    B, K, H, N = 4, 128, 256, 128
    x16, wg, wu, wd = (oracle.lcg_f16(n, s) for n, s in
                       ((B * K, 3001), (K * H, 3002), (K * H, 3003), (H * N, 3004)))
    bg, bu, bd = oracle.lcg_f32(H, 3005), oracle.lcg_f32(H, 3006), oracle.lcg_f32(N, 3007)
    out = oracle.swiglu_f16f32(x16, B, K, wg, H, bg, wu, bu, wd, N, bd)
    f = lambda a, *s: a.view(np.float16).astype(np.float64).reshape(*s)
    x = f(x16, B, K)
    g = x @ f(wg, K, H) + bg
    u = x @ f(wu, K, H) + bu
    h = (g / (1 + np.exp(-g)) * u).astype(np.float16).astype(np.float64)
    ref = h @ f(wd, H, N) + bd
    # fp16 rounding of h may flip by one ulp where fp32 and fp64 disagree
    assert np.abs(out - ref).max() <= 5e-3


def test_pack_layout(oracle):
    w16 = np.arange(20 * 18, dtype=np.float16).view(np.uint16)
    p = oracle.pack_weight_f16_tiles(w16, 20, 18).reshape(2, 32, 16)
    w = np.arange(20 * 18, dtype=np.float16).astype(np.float32).reshape(20, 18)
    assert np.array_equal(p[0, :20], w[:, :16])
    assert np.array_equal(p[1, :20, :2], w[:, 16:])
    assert not p[1, :, 2:].any() and not p[:, 20:].any()
