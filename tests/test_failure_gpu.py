"""Failure detection on the GPU, in the forms that fault nothing.

  * A bounded wait that runs out: a GEMV of the cross-GPU exchange waits for
    a signal word that nothing ever raises.  With the peer-wait limit cut to a
    fraction of a second the kernel must give up, return, and report
    kDevErrTimeout through the device error word; the device must stay usable
    (the next GEMV matches the oracle bit for bit).  Once the error word is
    set, every later wait of the step returns at once, so a step whose peers
    died costs one timeout, not one per GEMV.
  * An allocation that fails: the library's allocation hook makes the next
    device allocation fail as cudaMalloc does when the device is out of
    memory, and the entry points return SME_AI_ALLOC_FAILED (-2, the
    reference's sme_ai_ops.h:39-45 code) and leave their outputs empty.

No kernel here traps, asserts, reads out of bounds or spins without a limit.
"""
import ctypes
import time

import numpy as np
import pytest
import torch

import smeai_b200 as S
from smeai_b200 import q2k as Q
from smeai_b200.peer import make_exchange

pytestmark = pytest.mark.gpu
MS = 1_000_000


def _matrix(cuda, rows, k, seed):
    g = torch.Generator(device=cuda).manual_seed(seed)
    blocks = Q.quantize_q2k(torch.randn((rows, k), generator=g, device=cuda) * 0.02)
    return Q.Q2KMatrix(blocks, rows, k), blocks


@pytest.fixture
def short_peer_wait():
    L = S.lib()
    L.smeai_set_wait_timeouts(0, 200 * MS)       # peer waits give up after 200 ms
    yield 200 * MS
    L.smeai_set_wait_timeouts(0, 0)
    torch.cuda.synchronize()
    S.take_device_error()


def _dead_exchange(words):
    """An exchange whose wait can never be satisfied: *wait_sig stays 0 while
    the target is (*epoch + 1) * 1 = 1; nothing is stored or signalled."""
    base = words.data_ptr()
    return make_exchange(wait_sig=base, wait_count=1, epoch=base + 4)


def test_peer_wait_times_out_and_device_recovers(cuda, oracle, short_peer_wait):
    rows, k = 512, 4096
    m, blocks = _matrix(cuda, rows, k, 3)
    x = torch.randn((1, k), generator=torch.Generator(device=cuda).manual_seed(4), device=cuda)
    words = torch.zeros(2, dtype=torch.int32, device=cuda)
    out = torch.full((1, rows), float("nan"), device=cuda)
    assert S.take_device_error() == 0
    t0 = time.perf_counter()
    m.mul_mat_f32_peer(x, 1, out, _dead_exchange(words))
    torch.cuda.synchronize()
    elapsed = time.perf_counter() - t0
    assert S.take_device_error() == 1                  # kDevErrTimeout
    assert 0.15 < elapsed < 5.0, elapsed               # it waited its limit, then returned
    assert torch.isnan(out).all()                      # nothing was computed
    # the context is intact: the same weight's plain GEMV is exact
    y = m.mul_mat_f32(x).cpu().numpy()
    exp = oracle.q2k_mul_mat(blocks.cpu().numpy().reshape(-1).view(oracle.BLOCK_Q2_K), rows, k,
                             oracle.quantize_q8_K(x.cpu().numpy().reshape(-1)), 1)
    assert np.array_equal(y.view(np.uint32), exp.view(np.uint32))
    assert S.take_device_error() == 0


def test_timeout_cascade_ends_after_one_wait(cuda, short_peer_wait):
    """Four GEMVs whose peers never arrive, plus the step-end kernel: the first
    wait runs out its 200 ms, every later one sees the error word and returns
    at once (without that, the step would take 5 x 200 ms)."""
    rows, k = 4096, 4096
    m, _ = _matrix(cuda, rows, k, 5)
    x = torch.randn((1, k), device=cuda)
    words = torch.zeros(2, dtype=torch.int32, device=cuda)
    out = torch.empty((1, rows), device=cuda)
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    for _ in range(4):
        m.mul_mat_f32_peer(x, 1, out, _dead_exchange(words))
    base = words.data_ptr()
    S.check(S.lib().smeai_peer_step_end(ctypes.c_void_p(base), 1, ctypes.c_void_p(base + 4), Q.cur_stream()),
            "peer_step_end")
    torch.cuda.synchronize()
    elapsed = time.perf_counter() - t0
    assert S.take_device_error() == 1
    assert elapsed < 0.6, elapsed
    assert words.cpu().tolist() == [0, 0]             # the step counter did not advance


def test_alloc_failure_returns_alloc_failed(cuda):
    L = S.lib()
    try:
        # workspace
        ws = S.Workspace()
        L.smeai_debug_fail_next_allocs(1)
        assert L.sme_ai_workspace_init(ctypes.byref(ws), 4, 64, 64) == S.SME_AI_ALLOC_FAILED
        assert ws.tmp_f32 is None and ws.b_pack is None and ws.max_batch == 0   # left zeroed
        # packed weight
        w16 = (np.random.default_rng(0).standard_normal(64 * 64) * 0.1).astype(np.float16)
        pw = S.PackedWeight()
        L.smeai_debug_fail_next_allocs(1)
        assert L.sme_ai_packed_linear_weight_init(ctypes.byref(pw), w16.ctypes.data, 64, 64) == \
            S.SME_AI_ALLOC_FAILED
        assert pw.packed_weight is None
        # repacked Q2_K weight (device input: the tile allocation is the one that fails)
        blocks = Q.quantize_q2k(torch.randn((64, 512), device=cuda) * 0.02)
        h = ctypes.c_void_p()
        L.smeai_debug_fail_next_allocs(1)
        assert L.smeai_q2k_repack(ctypes.c_void_p(blocks.data_ptr()), 64, 512, ctypes.byref(h)) == \
            S.SME_AI_ALLOC_FAILED
        assert h.value is None and "failed" in S.last_error()
        # the hook is spent: the same calls now succeed
        assert L.sme_ai_workspace_init(ctypes.byref(ws), 4, 64, 64) == S.SME_AI_OK
        assert L.sme_ai_packed_linear_weight_init(ctypes.byref(pw), w16.ctypes.data, 64, 64) == S.SME_AI_OK
        x16 = (np.random.default_rng(1).standard_normal(4 * 64)).astype(np.float16)
        y = np.zeros(4 * 64, np.float32)
        assert L.sme_ai_linear_sme_packed_f16f32(ctypes.byref(ws), x16.ctypes.data, 4, ctypes.byref(pw), None,
                                                 y.ctypes.data) == S.SME_AI_OK
        exp = x16.astype(np.float32).reshape(4, 64) @ w16.astype(np.float32).reshape(64, 64)
        assert np.allclose(y.reshape(4, 64), exp, rtol=1e-5, atol=1e-5)
        assert L.smeai_q2k_repack(ctypes.c_void_p(blocks.data_ptr()), 64, 512, ctypes.byref(h)) == S.SME_AI_OK
        L.smeai_q2k_free(h)
        L.sme_ai_packed_linear_weight_destroy(ctypes.byref(pw))
        L.sme_ai_workspace_destroy(ctypes.byref(ws))
    finally:
        L.smeai_debug_fail_next_allocs(0)
