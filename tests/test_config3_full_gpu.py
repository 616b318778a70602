"""SwiGLU MLP decode at its full size against the oracle, through the C ABI.

Hidden 4096, ffn 11008: W_gate / W_up [11008, 4096] and W_down [4096, 11008]
drawn N(0, 0.02) and quantized to Q2_K, x ~ N(0, 1), batch 1 and 8;
y = W_down . Q8_K(silu(W_gate . Q8_K(x)) * (W_up . Q8_K(x))).

Bar, step by step on the same blocks:
  * Q8_K of x, the gate and up pre-activations (11008 x B each) and the down
    projection of the GPU's own h: bit-exact with the oracle's ggml-order dot;
  * h = silu(g) * u: within rel 1e-5 (CUDA expf against glibc expf);
  * the fused-prologue GEMVs and the one-kernel decode program give the same
    bits as the separate launches.
"""
import os

import numpy as np
import pytest
import torch

import smeai_b200 as S
from smeai_b200 import q2k as Q

pytestmark = pytest.mark.gpu
H, F = 4096, 11008
THREADS = os.cpu_count() or 1


@pytest.fixture(scope="module")
def mlp(cuda):
    g = torch.Generator(device=cuda).manual_seed(3)
    wg = Q.quantize_q2k(torch.randn((F, H), generator=g, device=cuda) * 0.02)
    wu = Q.quantize_q2k(torch.randn((F, H), generator=g, device=cuda) * 0.02)
    wd = Q.quantize_q2k(torch.randn((H, F), generator=g, device=cuda) * 0.02)
    gu = Q.Q2KMatrix(torch.stack([wg, wu], 1).reshape(2 * F, -1), 2 * F, H)   # rows g0, u0, g1, u1, ...
    down = Q.Q2KMatrix(wd, H, F)
    blk = lambda t: t.cpu().numpy().reshape(-1)
    yield dict(gu=gu, down=down, wg=blk(wg), wu=blk(wu), wd=blk(wd))
    gu.free()
    down.free()


def _as_q2k(oracle, b):
    return b.view(oracle.BLOCK_Q2_K)


@pytest.mark.parametrize("batch", [1, 8])
def test_swiglu_full_size_matches_oracle(cuda, oracle, mlp, batch):
    x = torch.randn((batch, H), generator=torch.Generator(device=cuda).manual_seed(batch), device=cuda)
    x_np = x.cpu().numpy()
    # Q8_K of x
    xq = Q.quantize_q8k(x)
    xq_o = oracle.quantize_q8_K(x_np.reshape(-1))
    assert np.array_equal(xq.cpu().numpy().reshape(-1), xq_o.view(np.uint8))
    # gate and up pre-activations (store epilogue over the interleaved rows)
    gu = mlp["gu"].mul_mat(xq, batch).cpu().numpy()                       # [B, 2F]
    g_o = oracle.q2k_mul_mat(_as_q2k(oracle, mlp["wg"]), F, H, xq_o, batch, n_threads=THREADS)
    u_o = oracle.q2k_mul_mat(_as_q2k(oracle, mlp["wu"]), F, H, xq_o, batch, n_threads=THREADS)
    assert np.array_equal(gu[:, 0::2].view(np.uint32), g_o.view(np.uint32))
    assert np.array_equal(gu[:, 1::2].view(np.uint32), u_o.view(np.uint32))
    # silu * mul epilogue
    h = mlp["gu"].mul_mat(xq, batch, epilogue=S.EPI_SILU_MUL)
    h_np = h.cpu().numpy()
    h_o = oracle.silu_mul(g_o.reshape(-1), u_o.reshape(-1)).reshape(batch, F)
    assert np.all(np.abs(h_np - h_o) <= 1e-5 * np.abs(h_o) + 1e-30)
    # down on the GPU's own h: quantizer and GEMV bit-exact
    hq = Q.quantize_q8k(h)
    hq_o = oracle.quantize_q8_K(h_np.reshape(-1))
    assert np.array_equal(hq.cpu().numpy().reshape(-1), hq_o.view(np.uint8))
    y = mlp["down"].mul_mat(hq, batch).cpu().numpy()
    y_o = oracle.q2k_mul_mat(_as_q2k(oracle, mlp["wd"]), H, F, hq_o, batch, n_threads=THREADS)
    assert np.array_equal(y.view(np.uint32), y_o.view(np.uint32))
    # the fused-prologue GEMVs: same bits
    h_f = mlp["gu"].mul_mat_f32_ex(x, batch, epilogue=S.EPI_SILU_MUL)
    assert torch.equal(h_f, h)
    y_f = mlp["down"].mul_mat_f32_ex(h_f, batch)
    assert np.array_equal(y_f.cpu().numpy().view(np.uint32), y.view(np.uint32))


@pytest.mark.parametrize("batch", [1, 8])
def test_swiglu_full_size_program_matches_launches(cuda, mlp, batch):
    """The two phases (gate/up with silu*mul, then down) as one persistent
    decode-program launch give the separate launches' bits."""
    x = torch.randn((batch, H), generator=torch.Generator(device=cuda).manual_seed(10 + batch), device=cuda)
    h_ref = mlp["gu"].mul_mat_f32_ex(x, batch, epilogue=S.EPI_SILU_MUL)
    y_ref = mlp["down"].mul_mat_f32_ex(h_ref, batch)
    h = torch.full((batch, F), float("nan"), device=cuda)
    y = torch.full((batch, H), float("nan"), device=cuda)
    prog = Q.Q2KProgram([dict(w=mlp["gu"], x=x, input=S.IN_F32, y=h, epilogue=S.EPI_SILU_MUL),
                         dict(w=mlp["down"], x=h, input=S.IN_F32, y=y)], batch)
    for _ in range(2):                     # twice: the second run reuses the program's state
        prog.run()
        torch.cuda.synchronize()
        assert torch.equal(h, h_ref)
        assert torch.equal(y, y_ref)
    prog.free()
    assert S.take_device_error() == 0
