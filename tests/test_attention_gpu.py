"""GPU parity of sme_ai_self_attention_{ref,sme_packed}_f16f32 against the CPU
restatement, through the C-ABI with host pointers (as a reference caller uses
them) and with device pointers.

The projections are bit-exact (k-ascending fp32 sums of exact fp16 products),
the score dot products and every sum follow the restatement's order, so the
only difference is CUDA's expf against glibc's (a few ulp on each
probability).  A context value sitting on an fp16 rounding boundary can
therefore round one fp16 step the other way, which moves the output rows by
about |w| * 2^-11 * |context|; the bar is the reference bench's own (abs 0.08
/ rel 0.02, bench_sme_full_timing.c:84-105, :653) and 1e-3 absolute, and at
least 99% of the fp16 context values must be bit-identical.
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
    return ws


def make_packed(L, w16, kin, kout):
    pw = S.PackedWeight()
    assert L.sme_ai_packed_linear_weight_init(ctypes.byref(pw), p(w16), kin, kout) == 0, S.last_error()
    return pw


def data(oracle, S_, D, seed0, biases=True):
    x16 = oracle.lcg_f16(S_ * D, seed0)
    ws = [oracle.lcg_f16(D * D, seed0 + i) for i in (1, 2, 3, 4)]
    bs = [oracle.lcg_f32(D, seed0 + i) if biases else None for i in (5, 6, 7, 8)]
    return x16, ws, bs


def check(got, exp):
    err = np.abs(got - exp)
    assert np.all((err <= 0.08) | (err <= 0.02 * np.abs(exp)))
    assert err.max() <= 1e-3, err.max()


def identity16(D):
    return np.eye(D, dtype=np.float16).view(np.uint16).reshape(-1)


def run_both(L, oracle, S_, D, H, causal, seed0, biases=True):
    """Both device paths against the restatement; then again with an identity
    output projection and no output bias, which makes the output the fp16
    context itself (an exact fp32 copy of each half)."""
    x16, (wq, wk, wv, wo), (bq, bk, bv, bo) = data(oracle, S_, D, seed0, biases)
    ws = make_ws(L, S_, D, D)
    results = []
    for wo_, bo_ in ((wo, bo), (identity16(D), None)):
        exp = oracle.self_attention_f16f32(x16, S_, D, H, wq, bq, wk, bk, wv, bv, wo_, bo_, causal)
        pws = [make_packed(L, w, D, D) for w in (wq, wk, wv, wo_)]
        ref = np.zeros((S_, D), np.float32)
        out = np.zeros((S_, D), np.float32)
        assert L.sme_ai_self_attention_ref_f16f32(ctypes.byref(ws), p(x16), S_, D, H, p(wq), p(bq), p(wk), p(bk),
                                                  p(wv), p(bv), p(wo_), p(bo_), causal, p(ref)) == 0, S.last_error()
        assert L.sme_ai_self_attention_sme_packed_f16f32(
            ctypes.byref(ws), p(x16), S_, D, H, ctypes.byref(pws[0]), p(bq), ctypes.byref(pws[1]), p(bk),
            ctypes.byref(pws[2]), p(bv), ctypes.byref(pws[3]), p(bo_), causal, p(out)) == 0, S.last_error()
        for a in pws:
            L.sme_ai_packed_linear_weight_destroy(ctypes.byref(a))
        # the two device paths share every step's order: identical results
        assert np.array_equal(ref, out)
        results.append((ref, exp))
    (got, exp), (ctx, ctx_exp) = results
    check(got, exp)
    assert np.mean(ctx == ctx_exp) >= 0.99
    assert np.all(np.abs(ctx - ctx_exp) <= np.abs(ctx_exp) * 2.0 ** -10 + 1e-7)  # one fp16 step at most
    if causal:
        assert np.array_equal(ctx[0], ctx_exp[0])  # row 0 attends only to itself: V_0
    L.sme_ai_workspace_destroy(ctypes.byref(ws))


def test_attention_bench_case(L, oracle):
    """bench_sme_full_timing.c run_attention_case: seq 16, d 128, 4 heads, causal, seeds 4001-4009."""
    run_both(L, oracle, 16, 128, 4, 1, 4001)


def test_attention_verify_case(L, oracle):
    """verify_sme_ai_timing.c run_attention_case: seq 8, d 64, 4 heads (head_dim 16), causal, seeds 801-809."""
    run_both(L, oracle, 8, 64, 4, 1, 801)


@pytest.mark.parametrize("S_,D,H,causal", [(16, 128, 4, 0), (37, 96, 3, 0), (70, 96, 2, 1), (50, 80, 5, 1),
                                           (33, 640, 2, 1), (9, 24, 3, 0), (1, 64, 2, 1), (200, 256, 2, 1)])
def test_attention_shapes(L, oracle, S_, D, H, causal):
    """Ragged tiles (seq not a multiple of 8 rows / 32 keys), head_dim 48, 16,
    320, 8 and 128, a single token, causal and full."""
    run_both(L, oracle, S_, D, H, causal, 17 + S_)


def test_attention_null_biases(L, oracle):
    run_both(L, oracle, 20, 64, 2, 1, 300, biases=False)


@pytest.mark.slow
def test_attention_long_sequence(L, oracle):
    """2048 tokens: 256 CTAs per head, 64 key tiles, score rows of 8 KB."""
    run_both(L, oracle, 2048, 256, 4, 1, 900)


def test_attention_device_pointers(L, oracle):
    S_, D, H = 24, 128, 4
    x16, (wq, wk, wv, wo), (bq, bk, bv, bo) = data(oracle, S_, D, 4001)
    exp = oracle.self_attention_f16f32(x16, S_, D, H, wq, bq, wk, bk, wv, bv, wo, bo, 1)
    dev = lambda a: torch.from_numpy(a).cuda()
    xd, wqd, wkd, wvd, wod = (dev(a) for a in (x16, wq, wk, wv, wo))
    bqd, bkd, bvd, bod = (dev(a) for a in (bq, bk, bv, bo))
    od = torch.zeros(S_ * D, dtype=torch.float32, device="cuda")
    ws = make_ws(L, S_, D, D)
    d = lambda t: P(t.data_ptr())
    assert L.sme_ai_self_attention_ref_f16f32(ctypes.byref(ws), d(xd), S_, D, H, d(wqd), d(bqd), d(wkd), d(bkd),
                                              d(wvd), d(bvd), d(wod), d(bod), 1, d(od)) == 0, S.last_error()
    check(od.cpu().numpy().reshape(S_, D), exp)
    L.sme_ai_workspace_destroy(ctypes.byref(ws))


def test_attention_status_codes(L, oracle):
    S_, D, H = 8, 64, 4
    x16, (wq, wk, wv, wo), (bq, bk, bv, bo) = data(oracle, S_, D, 801)
    ws = make_ws(L, S_, D, D)
    out = np.zeros((2 * S_, D), np.float32)
    ref = L.sme_ai_self_attention_ref_f16f32
    args = lambda s, d, h: (ctypes.byref(ws), p(x16), s, d, h, p(wq), p(bq), p(wk), p(bk), p(wv), p(bv), p(wo),
                            p(bo), 1, p(out))
    assert ref(*args(S_, D, 3)) == S.SME_AI_BAD_ARGUMENT           # 64 % 3
    assert ref(*args(S_, D, 0)) == S.SME_AI_BAD_ARGUMENT
    assert ref(*args(0, D, H)) == S.SME_AI_BAD_ARGUMENT
    assert ref(*args(2 * S_, D, H)) == S.SME_AI_WORKSPACE_TOO_SMALL  # seq_len > max_batch
    assert ref(None, p(x16), S_, D, H, p(wq), p(bq), p(wk), p(bk), p(wv), p(bv), p(wo), p(bo), 1,
               p(out)) == S.SME_AI_BAD_ARGUMENT
    assert ref(ctypes.byref(ws), p(x16), S_, D, H, None, p(bq), p(wk), p(bk), p(wv), p(bv), p(wo), p(bo), 1,
               p(out)) == S.SME_AI_BAD_ARGUMENT
    small = make_ws(L, S_, 32, 64)
    assert ref(ctypes.byref(small), p(x16), S_, D, H, p(wq), p(bq), p(wk), p(bk), p(wv), p(bv), p(wo), p(bo), 1,
               p(out)) == S.SME_AI_WORKSPACE_TOO_SMALL                # model_dim > max_in_features
    pws = [make_packed(L, w, D, D) for w in (wq, wk, wv, wo)]
    narrow = make_packed(L, oracle.lcg_f16(D * 32, 5), D, 32)
    pk = L.sme_ai_self_attention_sme_packed_f16f32
    assert pk(ctypes.byref(ws), p(x16), S_, D, H, ctypes.byref(pws[0]), p(bq), ctypes.byref(narrow), p(bk),
              ctypes.byref(pws[2]), p(bv), ctypes.byref(pws[3]), p(bo), 1, p(out)) == S.SME_AI_BAD_ARGUMENT
    assert pk(ctypes.byref(ws), p(x16), S_, D, H, ctypes.byref(pws[0]), p(bq), ctypes.byref(pws[1]), p(bk),
              ctypes.byref(pws[2]), p(bv), ctypes.byref(pws[3]), p(bo), 1, p(out)) == 0
    for a in pws + [narrow]:
        L.sme_ai_packed_linear_weight_destroy(ctypes.byref(a))
    for w in (ws, small):
        L.sme_ai_workspace_destroy(ctypes.byref(w))


def test_attention_device_entry_points(L, oracle):
    """The asynchronous device-pointer form on a caller's stream equals the
    synchronous call bit for bit; the core alone, fed the restatement's Q, K
    and V, reproduces its fp16 context."""
    S_, D, H = 40, 128, 4
    x16, (wq, wk, wv, wo), (bq, bk, bv, bo) = data(oracle, S_, D, 4001)
    ws = make_ws(L, S_, D, D)
    pws = [make_packed(L, w, D, D) for w in (wq, wk, wv, wo)]
    host = np.zeros((S_, D), np.float32)
    assert L.sme_ai_self_attention_sme_packed_f16f32(ctypes.byref(ws), p(x16), S_, D, H, ctypes.byref(pws[0]), p(bq),
                                                     ctypes.byref(pws[1]), p(bk), ctypes.byref(pws[2]), p(bv),
                                                     ctypes.byref(pws[3]), p(bo), 1, p(host)) == 0
    dev = lambda a: torch.from_numpy(a).cuda()
    d = lambda t: P(t.data_ptr())
    xd, bqd, bkd, bvd, bod = (dev(a) for a in (x16, bq, bk, bv, bo))
    od = torch.zeros(S_ * D, dtype=torch.float32, device="cuda")
    st = torch.cuda.Stream()
    assert L.sme_ai_self_attention_packed_f16f32_device(
        ctypes.byref(ws), d(xd), S_, D, H, ctypes.byref(pws[0]), d(bqd), ctypes.byref(pws[1]), d(bkd),
        ctypes.byref(pws[2]), d(bvd), ctypes.byref(pws[3]), d(bod), 1, d(od), P(st.cuda_stream)) == 0
    st.synchronize()
    assert np.array_equal(od.cpu().numpy().reshape(S_, D), host)

    _, c_exp = oracle.self_attention_f16f32(x16, S_, D, H, wq, bq, wk, bk, wv, bv, wo, bo, 1, with_context=True)
    q, k, v = (dev(oracle.linear_f16f32(x16, S_, D, w, D, b)) for w, b in ((wq, bq), (wk, bk), (wv, bv)))
    ctx = torch.zeros(S_ * D, dtype=torch.float16, device="cuda")
    assert L.sme_ai_self_attention_core_f32_device(d(q), d(k), d(v), S_, D, H, 1, d(ctx), P(st.cuda_stream)) == 0
    st.synchronize()
    c = ctx.cpu().numpy().view(np.uint16).reshape(S_, D)
    assert np.mean(c == c_exp) >= 0.99
    cf, ef = c.view(np.float16).astype(np.float64), c_exp.view(np.float16).astype(np.float64)
    assert np.all(np.abs(cf - ef) <= np.abs(ef) * 2.0 ** -10 + 1e-7)
    assert L.sme_ai_self_attention_core_f32_device(d(q), d(k), d(v), S_, D, 3, 1, d(ctx), None) == \
        S.SME_AI_BAD_ARGUMENT
    for a in pws:
        L.sme_ai_packed_linear_weight_destroy(ctypes.byref(a))
    L.sme_ai_workspace_destroy(ctypes.byref(ws))


@pytest.mark.parametrize("S_,D,H,causal", [(300, 128, 4, 1), (300, 128, 4, 0), (257, 256, 2, 1), (640, 128, 2, 0),
                                           (256, 64, 2, 1)])
def test_attention_tiled_shapes(L, oracle, S_, D, H, causal):
    """Shapes served by the tiled kernels (head_dim 32 / 64 / 128, 256 <= S):
    ragged last query / key tiles (S = 300, 257), causal and full."""
    run_both(L, oracle, S_, D, H, causal, 40 + S_)


def test_attention_tiled_head_chunks(L, oracle, monkeypatch):
    """A score budget of one head's matrix: heads are processed one chunk at a time."""
    monkeypatch.setenv("SMEAI_ATTN_SCORE_BUDGET", str(300 * 320 * 4 * 2))  # two heads per chunk
    run_both(L, oracle, 300, 160, 5, 1, 77)
    monkeypatch.setenv("SMEAI_ATTN_SCORE_BUDGET", "1")                      # one head per chunk
    run_both(L, oracle, 300, 96, 3, 0, 78)
