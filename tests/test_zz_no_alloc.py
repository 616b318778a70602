"""The SwiGLU entry point that allocates nothing
(sme_ai_swiglu_packed_f16f32_noalloc) against the allocating one
(sme_ai_swiglu_sme_packed_f16f32), through the C ABI.

It exists for callers that may not call cudaMalloc (their framework's pool
allocator owns the device heap, or their steady-state loop must never
allocate): its hidden state lives in a fixed 1 MiB device array inside the
library.  This file is named so pytest collects it last.
"""
import ctypes

import numpy as np
import pytest
import torch

import smeai_b200 as S

pytestmark = pytest.mark.gpu
P = ctypes.c_void_p
# Both entry points run the same two kernels in the same order (gate/up with
# the silu*mul and fp16 rounding of the hidden state, then the down Linear),
# so their outputs must agree bit for bit.
LIMIT = 512 * 1024   # fp16 values of the fixed scratch (batch * hidden_features)


def _host(a):
    return P(a.ctypes.data)


def _dev(t):
    return P(t.data_ptr())


def _half_bits(rng, n, scale=0.5):
    return (rng.uniform(-scale, scale, n).astype(np.float16)).view(np.uint16)


@pytest.mark.parametrize("B,K,H,N", [(4, 128, 256, 128), (8, 512, 1376, 512), (128, 64, 4096, 64)])
def test_noalloc_swiglu_matches_allocating_entry(cuda, B, K, H, N):
    L = S.lib()
    rng = np.random.default_rng(B * 1000 + H)
    wg, wu, wd = _half_bits(rng, K * H, 0.1), _half_bits(rng, K * H, 0.1), _half_bits(rng, H * N, 0.1)
    bg, bu, bd = (rng.uniform(-0.5, 0.5, n).astype(np.float32) for n in (H, H, N))

    ws = S.Workspace()
    assert L.sme_ai_workspace_init(ctypes.byref(ws), B, max(K, H), max(H, N)) == S.SME_AI_OK, S.last_error()
    packed = []
    for w, k_in, k_out in ((wg, K, H), (wu, K, H), (wd, H, N)):
        pw = S.PackedWeight()
        assert L.sme_ai_packed_linear_weight_init(ctypes.byref(pw), _host(w), k_in, k_out) == S.SME_AI_OK
        packed.append(pw)
    pg, pu, pd = packed
    bg_d, bu_d, bd_d = (torch.from_numpy(b).to(cuda) for b in (bg, bu, bd))
    stream = torch.cuda.current_stream()

    # two calls in a row, each with fresh inputs, each checked against the
    # allocating entry point on the same inputs
    for call in range(2):
        x16 = _half_bits(rng, B * K)
        ref = np.zeros((B, N), np.float32)
        assert L.sme_ai_swiglu_sme_packed_f16f32(ctypes.byref(ws), _host(x16), B, ctypes.byref(pg), _host(bg),
                                                 ctypes.byref(pu), _host(bu), ctypes.byref(pd), _host(bd),
                                                 _host(ref)) == S.SME_AI_OK, S.last_error()
        x_d = torch.from_numpy(x16.view(np.int16)).to(cuda)
        y_d = torch.full((B, N), float("nan"), device=cuda)
        st = L.sme_ai_swiglu_packed_f16f32_noalloc(_dev(x_d), B, ctypes.byref(pg), _dev(bg_d), ctypes.byref(pu),
                                                   _dev(bu_d), ctypes.byref(pd), _dev(bd_d), _dev(y_d),
                                                   P(stream.cuda_stream))
        assert st == S.SME_AI_OK, S.last_error()
        stream.synchronize()
        got = y_d.cpu().numpy()
        assert np.isfinite(got).all(), f"call {call}"
        assert np.array_equal(got.view(np.uint32), ref.view(np.uint32)), f"call {call}"

    for pw in packed:
        L.sme_ai_packed_linear_weight_destroy(ctypes.byref(pw))
    L.sme_ai_workspace_destroy(ctypes.byref(ws))


def test_noalloc_swiglu_rejects_sizes_beyond_its_scratch(cuda):
    L = S.lib()
    rng = np.random.default_rng(1)
    K, H, N = 64, 4096, 64
    packed = []
    for k_in, k_out in ((K, H), (K, H), (H, N)):
        pw = S.PackedWeight()
        assert L.sme_ai_packed_linear_weight_init(ctypes.byref(pw), _host(_half_bits(rng, k_in * k_out)), k_in,
                                                  k_out) == S.SME_AI_OK
        packed.append(pw)
    pg, pu, pd = packed
    B = LIMIT // H + 1                       # 129 * 4096 > 524288 fp16 values
    x_d = torch.zeros((B, K), dtype=torch.int16, device=cuda)
    y_d = torch.zeros((B, N), device=cuda)
    st = L.sme_ai_swiglu_packed_f16f32_noalloc(_dev(x_d), B, ctypes.byref(pg), None, ctypes.byref(pu), None,
                                               ctypes.byref(pd), None, _dev(y_d), None)
    assert st == S.SME_AI_WORKSPACE_TOO_SMALL
    assert "exceeds the fixed scratch" in S.last_error()
    for pw in packed:
        L.sme_ai_packed_linear_weight_destroy(ctypes.byref(pw))
