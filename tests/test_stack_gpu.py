"""The Llama-shape Q2_K decode stack (the benchmark workload) against the CPU
oracle run step by step on the same blocks, at reduced sizes."""
import numpy as np
import pytest
import torch

import smeai_b200 as S
from smeai_b200.stack import Q2KDecodeStack, shard_range

pytestmark = pytest.mark.gpu


def oracle_stack(O, st: Q2KDecodeStack, x0: np.ndarray):
    """Same computation on the CPU: rmsnorm+Q8_K, Q2_K GEMVs, silu*mul, residuals."""
    B2 = lambda t: t.cpu().numpy().reshape(-1).view(O.BLOCK_Q2_K)
    H, F, V = st.H, st.F, st.V
    x = x0.astype(np.float32).copy()
    nw = lambda t: None if t is None else t.cpu().numpy()
    for li, blk in enumerate(st.blocks):
        xq = O.rmsnorm_quantize_q8_K(x, st.eps, weight=nw(st.attn_norm[li]))
        v = O.q2k_mul_mat(B2(blk["v"]), H, H, xq, 1, n_threads=8)[0]
        x = (x + O.q2k_mul_mat(B2(blk["o"]), H, H, O.quantize_q8_K(v), 1, n_threads=8)[0]).astype(np.float32)
        xq = O.rmsnorm_quantize_q8_K(x, st.eps, weight=nw(st.ffn_norm[li]))
        g = O.q2k_mul_mat(B2(blk["g"]), F, H, xq, 1, n_threads=8)[0]
        u = O.q2k_mul_mat(B2(blk["u"]), F, H, xq, 1, n_threads=8)[0]
        h = O.silu_mul(g, u)
        x = (x + O.q2k_mul_mat(B2(blk["d"]), H, F, O.quantize_q8_K(h), 1, n_threads=8)[0]).astype(np.float32)
    xq = O.rmsnorm_quantize_q8_K(x, st.eps, weight=nw(st.out_norm))
    return O.q2k_mul_mat(B2(st.lm_blocks), V, H, xq, 1, n_threads=8)[0]


def test_stack_matches_oracle(cuda, oracle):
    st = Q2KDecodeStack(n_layers=2, hidden=1024, ffn=2816, vocab=4000, device=cuda, seed=3, keep_blocks=True)
    logits = st.step().clone()
    torch.cuda.synchronize()
    exp = oracle_stack(oracle, st, st.x0.cpu().numpy()[0])
    got = logits.cpu().numpy()[0]
    assert np.isfinite(got).all()
    # silu uses CUDA expf vs glibc expf; a last-bit difference can move one
    # Q8_K code, so the stack is held to a relative bar, not bit identity
    scale = np.abs(exp).max()
    assert np.abs(got - exp).max() <= 1e-3 * scale


def test_full_shape_layer_and_lm_head_match_oracle(cuda, oracle):
    """One layer at the 7B shape (hidden 4096, ffn 11008, RMSNorm weights) and
    the 32000 x 4096 lm_head, step by step against the oracle; the one-kernel
    program gives the separate launches' bits."""
    st = Q2KDecodeStack(n_layers=1, hidden=4096, ffn=11008, vocab=32000, device=cuda, seed=11, keep_blocks=True,
                        quant="separate")
    logits = st.step().clone()
    torch.cuda.synchronize()
    exp = oracle_stack(oracle, st, st.x0.cpu().numpy()[0])
    got = logits.cpu().numpy()[0]
    assert np.isfinite(got).all()
    scale = np.abs(exp).max()
    assert np.abs(got - exp).max() <= 1e-3 * scale
    st.quant = "program"
    assert torch.equal(st.step(), logits)
    assert torch.equal(st.step(), logits)
    st.free()


@pytest.mark.parametrize("quant", ["fused", "separate", "mixed", "program"])
@pytest.mark.parametrize("batch", [1, 2, 3, 4, 8])
def test_stack_quant_placements_identical(cuda, quant, batch):
    """Fused, separate and mixed Q8_K placement, and the whole step as one
    persistent kernel, give bit-identical logits."""
    ref = Q2KDecodeStack(n_layers=2, hidden=1024, ffn=2816, vocab=2048, batch=batch, device=cuda, seed=9,
                         quant="fused")
    a = ref.step().clone()
    st = Q2KDecodeStack(n_layers=2, hidden=1024, ffn=2816, vocab=2048, batch=batch, device=cuda, seed=9,
                        quant=quant)
    assert torch.equal(st.step(), a)
    assert torch.equal(st.step(), a)   # again: the program's counters and tags roll over


def test_stack_graph_replay_is_deterministic(cuda):
    st = Q2KDecodeStack(n_layers=3, hidden=1024, ffn=2816, vocab=2048, device=cuda, seed=5)
    eager = st.step().clone()
    stream = torch.cuda.Stream()
    with torch.cuda.stream(stream):
        st.step()
    stream.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=stream):
        st.step()
    for _ in range(3):
        with torch.cuda.stream(stream):
            g.replay()
    stream.synchronize()
    assert torch.equal(st.logits, eager)
    assert st.launches_per_step() == 3 * 4 + 1 + 3 * 4 + 1


def test_shard_ranges_partition_rows():
    for n in (4096, 11008, 32000, 12288):
        for world in (1, 2, 4, 8):
            spans = [shard_range(n, r, world) for r in range(world)]
            assert spans[0][0] == 0 and spans[-1][1] == n
            assert all(a[1] == b[0] for a, b in zip(spans, spans[1:]))
            assert all((hi - lo) % 32 == 0 for lo, hi in spans[:-1])


def test_program_phase_inputs_and_graph_capture(cuda):
    """A program whose first phase takes Q8_K rows and whose later phases take
    fp32 rows (plain and RMS-normalized), against the separate GEMV launches,
    eagerly and replayed from a CUDA graph."""
    from smeai_b200 import IN_F32, IN_F32_RMS, IN_Q8K
    from smeai_b200 import q2k as Q
    g = torch.Generator(device=cuda).manual_seed(4)
    mk = lambda rows, k: Q.Q2KMatrix(Q.quantize_q2k(torch.randn((rows, k), generator=g, device=cuda) * 0.02),
                                     rows, k)
    B = 2
    a, b, c = mk(768, 512), mk(2 * 512, 768), mk(300, 512)
    xq = Q.quantize_q8k(torch.randn((B, 512), generator=g, device=cuda))
    r = torch.randn((B, 768), generator=g, device=cuda)
    y0, y1, y2 = torch.empty((B, 768), device=cuda), torch.empty((B, 512), device=cuda), \
        torch.empty((B, 300), device=cuda)
    prog = Q.Q2KProgram([dict(w=a, x=xq, input=IN_Q8K, y=y0, epilogue=S.EPI_RESIDUAL, resid=r),
                         dict(w=b, x=y0, input=IN_F32_RMS, y=y1, epilogue=S.EPI_SILU_MUL),
                         dict(w=c, x=y1, input=IN_F32, y=y2)], B, rms_eps=1e-5)
    e0 = a.mul_mat(xq, B, epilogue=S.EPI_RESIDUAL, resid=r)
    e1 = b.mul_mat_f32_ex(e0, B, epilogue=S.EPI_SILU_MUL, rms_eps=1e-5)
    e2 = c.mul_mat_f32_ex(e1, B)
    prog.run()
    torch.cuda.synchronize()
    assert torch.equal(y0, e0) and torch.equal(y1, e1) and torch.equal(y2, e2)
    stream = torch.cuda.Stream()
    y2.zero_()
    torch.cuda.synchronize()
    gr = torch.cuda.CUDAGraph()
    with torch.cuda.graph(gr, stream=stream):
        prog.run()
    for _ in range(3):
        with torch.cuda.stream(stream):
            gr.replay()
    stream.synchronize()
    assert torch.equal(y2, e2)
    del gr
    prog.free()


def test_program_rejects_bad_phases(cuda):
    from smeai_b200 import IN_F32
    from smeai_b200 import q2k as Q
    m = Q.Q2KMatrix(Q.quantize_q2k(torch.randn((64, 512), device=cuda)), 64, 512)
    x, y = torch.zeros((3, 512), device=cuda), torch.zeros((3, 64), device=cuda)
    with pytest.raises(RuntimeError):      # 3 tokens: not 1, 2, 4 or 8
        Q.Q2KProgram([dict(w=m, x=x, input=IN_F32, y=y)], 3)
    with pytest.raises(RuntimeError):      # residual epilogue without a residual
        Q.Q2KProgram([dict(w=m, x=x[:2], input=IN_F32, y=y[:2], epilogue=S.EPI_RESIDUAL)], 2)
    with pytest.raises(RuntimeError):      # input rows shorter than k
        Q.Q2KProgram([dict(w=m, x=torch.zeros((2, 256), device=cuda), input=IN_F32, y=y[:2])], 2)


@pytest.mark.parametrize("batch", [8, 130])
def test_prefill_stack_on_tensor_cores_matches_decode_stack(cuda, batch):
    """The stack over `batch` tokens with every linear on the tcgen05 GEMM
    (residual and silu*mul in its epilogue) gives the GEMV stack's bits:
    tokens are independent (attention over one position), and the GEMM, its
    epilogues and the quantizers equal the decode path's."""
    kw = dict(n_layers=2, hidden=1024, ffn=2816, vocab=2048, batch=batch, device=cuda, seed=21)
    ref = Q2KDecodeStack(quant="fused", **kw)
    a = ref.step().clone()
    st = Q2KDecodeStack(quant="tc", **kw)
    b = st.step()
    torch.cuda.synchronize()
    assert torch.equal(b, a)
    assert torch.isfinite(b).all()


def test_token_sharded_prefill_rows_match_whole_batch(cuda):
    """Sequence sharding of the prefill (the multi-GPU prefill-stack bench):
    a stack over tokens [lo, hi) of the batch gives rows lo..hi-1 of the
    whole batch's logits bit for bit, for every rank of 3 (tokens are
    independent through the linear stack; each rank holds the full weights)."""
    from smeai_b200.stack import token_range
    kw = dict(n_layers=2, hidden=1024, ffn=2816, vocab=2048, batch=130, device=cuda, seed=21, quant="tc")
    whole = Q2KDecodeStack(**kw)
    ref = whole.step().clone()
    whole.free()
    for r in range(3):
        lo, hi = token_range(130, r, 3)
        part = Q2KDecodeStack(tokens=(lo, hi), **kw)
        assert part.B == hi - lo
        assert torch.equal(part.step(), ref[lo:hi]), r
        part.free()


def test_tc_gemm_epilogues_match_gemv(cuda):
    from smeai_b200 import q2k as Q
    g = torch.Generator(device=cuda).manual_seed(8)
    rows, k, cols = 600, 1024, 37
    m = Q.Q2KMatrix(Q.quantize_q2k(torch.randn((rows, k), generator=g, device=cuda) * 0.02), rows, k)
    xq = Q.quantize_q8k(torch.randn((cols, k), generator=g, device=cuda))
    r = torch.randn((cols, rows), generator=g, device=cuda)
    assert torch.equal(m.mul_mat_tc(xq, cols), m.mul_mat(xq, cols))
    assert torch.equal(m.mul_mat_tc(xq, cols, epilogue=S.EPI_RESIDUAL, resid=r),
                       m.mul_mat(xq, cols, epilogue=S.EPI_RESIDUAL, resid=r))
    y = r.clone()                                  # in place: resid aliases the output
    m.mul_mat_tc(xq, cols, out=y, epilogue=S.EPI_RESIDUAL, resid=y)
    assert torch.equal(y, m.mul_mat(xq, cols, epilogue=S.EPI_RESIDUAL, resid=r))
    assert torch.equal(m.mul_mat_tc(xq, cols, epilogue=S.EPI_SILU_MUL),
                       m.mul_mat(xq, cols, epilogue=S.EPI_SILU_MUL))


@pytest.mark.parametrize("batch", [1, 2])
def test_mg_program_wiring_on_one_gpu(cuda, batch):
    """The multi-GPU program's explicit phase wiring, run with one rank (no
    peers), gives the one-GPU program's logits bit for bit, eagerly and
    twice from a CUDA graph (tags advance, the double-buffered sets swap)."""
    kw = dict(n_layers=2, hidden=1024, ffn=2816, vocab=2048, batch=batch, device=cuda, seed=13)
    a = Q2KDecodeStack(quant="program", **kw).step().clone()
    st = Q2KDecodeStack(quant="mgprog", **kw)
    assert torch.equal(st.step(), a)
    stream = torch.cuda.Stream()
    st.logits.zero_()
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=stream):
        st.step()
    for _ in range(2):
        with torch.cuda.stream(stream):
            g.replay()
        stream.synchronize()
        assert torch.equal(st.logits, a)
    del g
    st.free()
    assert S.take_device_error() == 0
