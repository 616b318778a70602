"""CPU tests of the self-attention restatement (sme_ai_self_attention_ref_f16f32,
sme_ai_ops.c:1320-1410).  The reference's SVE code does not run on this host,
so the restatement is pinned against an independent float64 formulation of
the same operator (projections, scaled scores, softmax, weighted sum, fp16
context, output projection) and against the structural properties the
operator has: causality, head independence and bias handling."""
import numpy as np
import pytest


def f16(a, *shape):
    return a.view(np.float16).astype(np.float64).reshape(*shape)


def attention_f64(x16, S, D, H, wq, bq, wk, bk, wv, bv, wo, bo, causal):
    hd = D // H
    x = f16(x16, S, D)
    lin = lambda a, w, b: a @ f16(w, D, D) + (0.0 if b is None else b.astype(np.float64))
    q, k, v = lin(x, wq, bq), lin(x, wk, bk), lin(x, wv, bv)
    ctx = np.zeros((S, D))
    for h in range(H):
        sl = slice(h * hd, (h + 1) * hd)
        s = q[:, sl] @ k[:, sl].T / np.sqrt(hd)
        if causal:
            s = np.where(np.tril(np.ones((S, S), bool)), s, -np.inf)
        s = np.exp(s - s.max(1, keepdims=True))
        ctx[:, sl] = (s / s.sum(1, keepdims=True)) @ v[:, sl]
    c16 = ctx.astype(np.float16).astype(np.float64)
    return lin(c16, wo, bo), ctx


def case(oracle, S, D, seed0):
    x16 = oracle.lcg_f16(S * D, seed0)
    ws = [oracle.lcg_f16(D * D, seed0 + i) for i in (1, 2, 3, 4)]
    bs = [oracle.lcg_f32(D, seed0 + i) for i in (5, 6, 7, 8)]
    return x16, ws, bs


@pytest.mark.parametrize("S,D,H,causal,seed", [(16, 128, 4, 1, 4001), (8, 64, 4, 1, 801), (16, 128, 4, 0, 4001),
                                               (37, 96, 3, 0, 7), (70, 64, 1, 1, 11)])
def test_attention_matches_float64(oracle, S, D, H, causal, seed):
    x16, (wq, wk, wv, wo), (bq, bk, bv, bo) = case(oracle, S, D, seed)
    out, c16 = oracle.self_attention_f16f32(x16, S, D, H, wq, bq, wk, bk, wv, bv, wo, bo, causal, with_context=True)
    ref, ctx = attention_f64(x16, S, D, H, wq, bq, wk, bk, wv, bv, wo, bo, causal)
    # the context before its fp16 rounding agrees to fp32 accuracy; after it,
    # at most a rounding step of fp16 apart
    c = c16.view(np.float16).astype(np.float64)
    assert np.all(np.abs(c - ctx) <= np.abs(ctx) * 2.0 ** -10 + 1e-6)
    err = np.abs(out - ref)
    assert np.all((err <= 0.08) | (err <= 0.02 * np.abs(ref)))   # the reference bench's bar
    assert err.max() <= 2e-3 * max(1.0, np.abs(ref).max())


def test_attention_causal_rows_ignore_later_tokens(oracle):
    S, D, H = 24, 64, 2
    x16, (wq, wk, wv, wo), (bq, bk, bv, bo) = case(oracle, S, D, 500)
    a = oracle.self_attention_f16f32(x16, S, D, H, wq, bq, wk, bk, wv, bv, wo, bo, 1)
    y16 = x16.copy().reshape(S, D)
    y16[10:] = oracle.lcg_f16((S - 10) * D, 999).reshape(S - 10, D)
    b = oracle.self_attention_f16f32(y16.reshape(-1), S, D, H, wq, bq, wk, bk, wv, bv, wo, bo, 1)
    assert np.array_equal(a[:10], b[:10]) and not np.array_equal(a[10:], b[10:])
    # the first row attends only to itself: its context is V_0
    out, c16 = oracle.self_attention_f16f32(x16, S, D, H, wq, bq, wk, bk, wv, bv, wo, bo, 1, with_context=True)
    v0 = oracle.linear_f16f32(x16[:D], 1, D, wv, D, bv)[0]
    assert np.array_equal(c16[0], v0.astype(np.float16).view(np.uint16))


def test_attention_one_head_per_column_block(oracle):
    """With a block-diagonal Q/K/V weight (head h reads only its own input
    columns), each head's context matches a one-head run on that slice."""
    S, D, H = 12, 64, 4
    hd = D // H
    x16, (wq, wk, wv, wo), _ = case(oracle, S, D, 42)
    mask = np.kron(np.eye(H), np.ones((hd, hd))).astype(bool).reshape(-1)
    zero = np.float16(0).view(np.uint16)
    wq, wk, wv = (np.where(mask, w, zero).astype(np.uint16) for w in (wq, wk, wv))
    _, c = oracle.self_attention_f16f32(x16, S, D, H, wq, None, wk, None, wv, None, wo, None, 0, with_context=True)
    xs = x16.reshape(S, D)
    for h in range(H):
        sl = slice(h * hd, (h + 1) * hd)
        sub = lambda w: np.ascontiguousarray(w.reshape(D, D)[sl, sl]).reshape(-1)
        _, ch = oracle.self_attention_f16f32(np.ascontiguousarray(xs[:, sl]).reshape(-1), S, hd, 1, sub(wq), None,
                                             sub(wk), None, sub(wv), None, sub(wo), None, 0, with_context=True)
        assert np.array_equal(c[:, sl], ch)


def test_attention_bad_arguments(oracle):
    x16 = oracle.lcg_f16(4 * 30, 1)
    w = oracle.lcg_f16(30 * 30, 2)
    with pytest.raises(AssertionError):
        oracle.self_attention_f16f32(x16, 4, 30, 4, w, None, w, None, w, None, w, None, 0)  # 30 % 4 != 0
