"""Q2_K x Q8_K path over torch device memory (thin wrappers of smeai_q2k.h)."""
from __future__ import annotations

import ctypes

import numpy as np
import torch

from . import (EPI_RESIDUAL, EPI_SILU_MUL, EPI_STORE, Q2K_BLOCK_BYTES, Q3K_BLOCK_BYTES, Q6K_BLOCK_BYTES,
               Q8K_BLOCK_BYTES, QK_K, check, lib)


def _ptr(t):
    return ctypes.c_void_p(0 if t is None else t.data_ptr())


def cur_stream() -> ctypes.c_void_p:
    return ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)


def quantize_q8k(x: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
    """fp32 [n, k] (cuda) -> ggml block_q8_K rows, uint8 [n, k/256*292]."""
    x2 = x.reshape(-1, x.shape[-1])
    n, k = x2.shape
    assert x2.dtype == torch.float32 and x2.is_cuda and x2.stride(1) == 1
    if out is None:
        out = torch.empty((n, k // QK_K * Q8K_BLOCK_BYTES), dtype=torch.uint8, device=x.device)
    check(lib().smeai_q8k_quantize(_ptr(x2), x2.stride(0), n, k, _ptr(out), cur_stream()), "q8k_quantize")
    return out


def rms_quantize_q8k(x: torch.Tensor, eps: float, out: torch.Tensor | None = None,
                     norm_w: torch.Tensor | None = None) -> torch.Tensor:
    """RMSNorm of each row (times norm_w when given), then Q8_K."""
    x2 = x.reshape(-1, x.shape[-1])
    n, k = x2.shape
    assert x2.dtype == torch.float32 and x2.is_cuda and x2.stride(1) == 1
    if out is None:
        out = torch.empty((n, k // QK_K * Q8K_BLOCK_BYTES), dtype=torch.uint8, device=x.device)
    if norm_w is None:
        check(lib().smeai_rms_q8k_quantize(_ptr(x2), x2.stride(0), n, k, ctypes.c_float(eps), _ptr(out),
                                            cur_stream()), "rms_q8k_quantize")
    else:
        assert norm_w.dtype == torch.float32 and norm_w.is_cuda and norm_w.numel() == k and norm_w.is_contiguous()
        check(lib().smeai_rms_q8k_quantize_w(_ptr(x2), x2.stride(0), n, k, _ptr(norm_w), ctypes.c_float(eps),
                                              _ptr(out), cur_stream()), "rms_q8k_quantize_w")
    return out


def quantize_q2k(x: torch.Tensor) -> torch.Tensor:
    """fp32 [rows, k] (cuda) -> ggml block_q2_K rows, uint8 [rows, k/256*84]."""
    x2 = x.reshape(-1, x.shape[-1]).contiguous()
    rows, k = x2.shape
    out = torch.empty((rows, k // QK_K * Q2K_BLOCK_BYTES), dtype=torch.uint8, device=x.device)
    check(lib().smeai_q2k_quantize_device(_ptr(x2), x2.numel(), _ptr(out), cur_stream()), "q2k_quantize")
    return out


def dequantize_q2k(blocks: torch.Tensor, k: int) -> torch.Tensor:
    rows = blocks.numel() // (k // QK_K * Q2K_BLOCK_BYTES)
    out = torch.empty((rows, k), dtype=torch.float32, device=blocks.device)
    check(lib().smeai_q2k_dequantize_device(_ptr(blocks), rows * k, _ptr(out), cur_stream()), "q2k_dequantize")
    return out


def as_bytes(blocks) -> np.ndarray:
    """numpy structured blocks / raw bytes -> flat uint8 view."""
    return np.ascontiguousarray(blocks).view(np.uint8).reshape(-1)


class Q2KMatrix:
    """A Q2_K weight [n_rows, k] repacked into the device tile layout."""

    def __init__(self, blocks, n_rows: int, k: int):
        assert k % QK_K == 0
        self.n_rows, self.k, self.nb = n_rows, k, k // QK_K
        handle = ctypes.c_void_p()
        if isinstance(blocks, torch.Tensor):
            src = blocks.contiguous()
            ptr = _ptr(src)
            torch.cuda.current_stream().synchronize() if src.is_cuda else None
        else:
            src = as_bytes(blocks)
            ptr = ctypes.c_void_p(src.ctypes.data)
        assert (src.numel() if isinstance(src, torch.Tensor) else src.size) == n_rows * self.nb * Q2K_BLOCK_BYTES
        check(lib().smeai_q2k_repack(ptr, n_rows, k, ctypes.byref(handle)), "q2k_repack")
        self.handle = handle
        self.bytes = lib().smeai_q2k_weight_bytes(handle)

    @classmethod
    def from_handle(cls, handle: ctypes.c_void_p, n_rows: int, k: int) -> "Q2KMatrix":
        """Wrap a weight already in the device tile layout (e.g. smeai_gguf_load_q2k)."""
        self = cls.__new__(cls)
        self.n_rows, self.k, self.nb = n_rows, k, k // QK_K
        self.handle = handle
        self.bytes = lib().smeai_q2k_weight_bytes(handle)
        return self

    def mul_mat(self, xq: torch.Tensor, n_cols: int, out: torch.Tensor | None = None, epilogue: int = EPI_STORE,
                resid: torch.Tensor | None = None) -> torch.Tensor:
        out_rows = self.n_rows // 2 if epilogue == EPI_SILU_MUL else self.n_rows
        if out is None:
            out = torch.empty((n_cols, out_rows), dtype=torch.float32, device=xq.device)
        ldy = out.stride(0) if out.dim() == 2 else out_rows
        if epilogue == EPI_STORE:
            st = lib().smeai_q2k_mul_mat(self.handle, self.n_rows, self.k, _ptr(xq), n_cols, _ptr(out), ldy,
                                         cur_stream())
        else:
            ldr = 0 if resid is None else (resid.stride(0) if resid.dim() == 2 else out_rows)
            st = lib().smeai_q2k_mul_mat_ex(self.handle, _ptr(xq), n_cols, _ptr(out), ldy, epilogue,
                                            _ptr(resid), ldr, cur_stream())
        check(st, "q2k_mul_mat")
        return out

    def mul_mat_tc(self, xq: torch.Tensor, n_cols: int, out: torch.Tensor | None = None,
                   epilogue: int = EPI_STORE, resid: torch.Tensor | None = None) -> torch.Tensor:
        """The tensor-core GEMM path (any number of activation rows), with the
        GEMV's epilogues."""
        out_rows = self.n_rows // 2 if epilogue == EPI_SILU_MUL else self.n_rows
        if out is None:
            out = torch.empty((n_cols, out_rows), dtype=torch.float32, device=xq.device)
        if epilogue == EPI_STORE:
            check(lib().smeai_q2k_mul_mat_tc(self.handle, _ptr(xq), n_cols, _ptr(out), out.stride(0),
                                             cur_stream()), "q2k_mul_mat_tc")
        else:
            ldr = 0 if resid is None else resid.stride(0)
            check(lib().smeai_q2k_mul_mat_tc_ex(self.handle, _ptr(xq), n_cols, _ptr(out), out.stride(0), epilogue,
                                                _ptr(resid), ldr, cur_stream()), "q2k_mul_mat_tc_ex")
        return out

    def mul_mat_f32(self, x: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
        x2 = x.reshape(-1, self.k).contiguous()
        n_cols = x2.shape[0]
        if out is None:
            out = torch.empty((n_cols, self.n_rows), dtype=torch.float32, device=x.device)
        check(lib().smeai_q2k_mul_mat_f32(self.handle, _ptr(x2), n_cols, _ptr(out), out.stride(0), cur_stream()),
              "q2k_mul_mat_f32")
        return out

    def mul_mat_f32_ex(self, x: torch.Tensor, n_cols: int, out: torch.Tensor | None = None,
                       epilogue: int = EPI_STORE, resid: torch.Tensor | None = None,
                       rms_eps: float | None = None, norm_w: torch.Tensor | None = None) -> torch.Tensor:
        """fp32 activations [n_cols, >=k] (row stride x.stride(0)), quantized to
        Q8_K (after an RMSNorm when rms_eps is given, times norm_w when given)
        inside the GEMV."""
        out_rows = self.n_rows // 2 if epilogue == EPI_SILU_MUL else self.n_rows
        if out is None:
            out = torch.empty((n_cols, out_rows), dtype=torch.float32, device=x.device)
        assert x.dtype == torch.float32 and x.stride(-1) == 1
        ld_x = x.stride(0) if x.dim() == 2 else self.k
        ldy = out.stride(0) if out.dim() == 2 else out_rows
        ldr = 0 if resid is None else (resid.stride(0) if resid.dim() == 2 else out_rows)
        eps = -1.0 if rms_eps is None else float(rms_eps)
        check(lib().smeai_q2k_mul_mat_f32_norm(self.handle, _ptr(x), ld_x, n_cols, _ptr(out), ldy, epilogue,
                                               _ptr(resid), ldr, ctypes.c_float(eps), _ptr(norm_w), cur_stream()),
              "q2k_mul_mat_f32_norm")
        return out

    def mul_mat_f32_peer(self, x: torch.Tensor, n_cols: int, out: torch.Tensor, ex, epilogue: int = EPI_STORE,
                         resid: torch.Tensor | None = None, rms_eps: float | None = None,
                         norm_w: torch.Tensor | None = None) -> torch.Tensor:
        """mul_mat_f32_ex with the fused cross-GPU exchange `ex` (a PeerExchange)."""
        out_rows = self.n_rows // 2 if epilogue == EPI_SILU_MUL else self.n_rows
        assert x.dtype == torch.float32 and x.stride(-1) == 1
        ld_x = x.stride(0) if x.dim() == 2 else self.k
        ldy = out.stride(0) if out.dim() == 2 else out_rows
        ldr = 0 if resid is None else (resid.stride(0) if resid.dim() == 2 else out_rows)
        eps = -1.0 if rms_eps is None else float(rms_eps)
        check(lib().smeai_q2k_mul_mat_f32_peer(self.handle, _ptr(x), ld_x, n_cols, _ptr(out), ldy, epilogue,
                                               _ptr(resid), ldr, ctypes.c_float(eps), _ptr(norm_w),
                                               ctypes.byref(ex), cur_stream()), "q2k_mul_mat_f32_peer")
        return out

    def block_sums(self, xq: torch.Tensor):
        isum = torch.empty((self.n_rows, self.nb), dtype=torch.int32, device=xq.device)
        summs = torch.empty_like(isum)
        check(lib().smeai_q2k_block_sums(self.handle, _ptr(xq), _ptr(isum), _ptr(summs), cur_stream()),
              "q2k_block_sums")
        return isum, summs

    def free(self):
        if self.handle:
            lib().smeai_q2k_free(self.handle)
            self.handle = ctypes.c_void_p()

    def __del__(self):
        try:
            self.free()
        except Exception:
            pass


__all__ = ["quantize_q8k", "rms_quantize_q8k", "quantize_q2k", "dequantize_q2k", "Q2KMatrix", "Q3KMatrix",
           "dequantize_q3k", "Q6KMatrix", "dequantize_q6k", "as_bytes",
           "EPI_STORE", "EPI_RESIDUAL", "EPI_SILU_MUL"]


class Q3KMatrix:
    """A Q3_K weight [n_rows, k] in the device tile layout (smeai_q3k_*)."""

    def __init__(self, blocks, n_rows: int, k: int, handle: ctypes.c_void_p | None = None):
        assert k % QK_K == 0
        self.n_rows, self.k, self.nb = n_rows, k, k // QK_K
        if handle is None:
            handle = ctypes.c_void_p()
            if isinstance(blocks, torch.Tensor):
                src = blocks.contiguous()
                ptr = _ptr(src)
                if src.is_cuda:
                    torch.cuda.current_stream().synchronize()
                n = src.numel()
            else:
                src = as_bytes(blocks)
                ptr = ctypes.c_void_p(src.ctypes.data)
                n = src.size
            assert n == n_rows * self.nb * Q3K_BLOCK_BYTES
            check(lib().smeai_q3k_repack(ptr, n_rows, k, ctypes.byref(handle)), "q3k_repack")
        self.handle = handle
        self.bytes = lib().smeai_q2k_weight_bytes(handle)

    def mul_mat(self, xq: torch.Tensor, n_cols: int, out: torch.Tensor | None = None) -> torch.Tensor:
        if out is None:
            out = torch.empty((n_cols, self.n_rows), dtype=torch.float32, device=xq.device)
        check(lib().smeai_q3k_mul_mat(self.handle, _ptr(xq), n_cols, _ptr(out), out.stride(0), cur_stream()),
              "q3k_mul_mat")
        return out

    def mul_mat_f32(self, x: torch.Tensor, rms_eps: float | None = None,
                    out: torch.Tensor | None = None) -> torch.Tensor:
        x2 = x.reshape(-1, self.k)
        n_cols = x2.shape[0]
        if out is None:
            out = torch.empty((n_cols, self.n_rows), dtype=torch.float32, device=x.device)
        eps = -1.0 if rms_eps is None else rms_eps
        check(lib().smeai_q3k_mul_mat_f32(self.handle, _ptr(x2), x2.stride(0), n_cols, _ptr(out), out.stride(0),
                                          ctypes.c_float(eps), cur_stream()), "q3k_mul_mat_f32")
        return out

    def block_sums(self, xq_row: torch.Tensor):
        isum = torch.empty((self.n_rows, self.nb), dtype=torch.int32, device=xq_row.device)
        summs = torch.empty_like(isum)
        check(lib().smeai_q3k_block_sums(self.handle, _ptr(xq_row), _ptr(isum), _ptr(summs), cur_stream()),
              "q3k_block_sums")
        return isum, summs

    def free(self):
        if getattr(self, "handle", None) and self.handle.value:
            lib().smeai_q3k_free(self.handle)
            self.handle = ctypes.c_void_p()

    def __del__(self):
        try:
            self.free()
        except Exception:
            pass


def dequantize_q3k(blocks: torch.Tensor, k_total: int) -> torch.Tensor:
    out = torch.empty(k_total, dtype=torch.float32, device=blocks.device)
    check(lib().smeai_q3k_dequantize_device(_ptr(blocks), k_total, _ptr(out), cur_stream()), "q3k_dequantize")
    return out


class Q6KMatrix:
    """A Q6_K weight [n_rows, k] in the device tile layout (smeai_q6k_*)."""

    def __init__(self, blocks, n_rows: int, k: int, handle: ctypes.c_void_p | None = None):
        assert k % QK_K == 0
        self.n_rows, self.k, self.nb = n_rows, k, k // QK_K
        if handle is None:
            handle = ctypes.c_void_p()
            if isinstance(blocks, torch.Tensor):
                src = blocks.contiguous()
                ptr = _ptr(src)
                if src.is_cuda:
                    torch.cuda.current_stream().synchronize()
                n = src.numel()
            else:
                src = as_bytes(blocks)
                ptr = ctypes.c_void_p(src.ctypes.data)
                n = src.size
            assert n == n_rows * self.nb * Q6K_BLOCK_BYTES
            check(lib().smeai_q6k_repack(ptr, n_rows, k, ctypes.byref(handle)), "q6k_repack")
        self.handle = handle
        self.bytes = lib().smeai_q2k_weight_bytes(handle)

    def mul_mat(self, xq: torch.Tensor, n_cols: int, out: torch.Tensor | None = None) -> torch.Tensor:
        if out is None:
            out = torch.empty((n_cols, self.n_rows), dtype=torch.float32, device=xq.device)
        check(lib().smeai_q6k_mul_mat(self.handle, _ptr(xq), n_cols, _ptr(out), out.stride(0), cur_stream()),
              "q6k_mul_mat")
        return out

    def mul_mat_f32(self, x: torch.Tensor, rms_eps: float | None = None,
                    out: torch.Tensor | None = None) -> torch.Tensor:
        x2 = x.reshape(-1, self.k)
        n_cols = x2.shape[0]
        if out is None:
            out = torch.empty((n_cols, self.n_rows), dtype=torch.float32, device=x.device)
        eps = -1.0 if rms_eps is None else rms_eps
        check(lib().smeai_q6k_mul_mat_f32(self.handle, _ptr(x2), x2.stride(0), n_cols, _ptr(out), out.stride(0),
                                          ctypes.c_float(eps), cur_stream()), "q6k_mul_mat_f32")
        return out

    def block_sums(self, xq_row: torch.Tensor):
        isum = torch.empty((self.n_rows, self.nb), dtype=torch.int32, device=xq_row.device)
        summs = torch.empty_like(isum)
        check(lib().smeai_q6k_block_sums(self.handle, _ptr(xq_row), _ptr(isum), _ptr(summs), cur_stream()),
              "q6k_block_sums")
        return isum, summs

    def free(self):
        if getattr(self, "handle", None) and self.handle.value:
            lib().smeai_q6k_free(self.handle)
            self.handle = ctypes.c_void_p()

    def __del__(self):
        try:
            self.free()
        except Exception:
            pass


def dequantize_q6k(blocks: torch.Tensor, k_total: int) -> torch.Tensor:
    out = torch.empty(k_total, dtype=torch.float32, device=blocks.device)
    check(lib().smeai_q6k_dequantize_device(_ptr(blocks), k_total, _ptr(out), cur_stream()), "q6k_dequantize")
    return out


class Q2KProgram:
    """A chain of GEMV phases run as one persistent kernel
    (smeai_q2k_program_*).  phases: dicts with keys w (Q2KMatrix), x (tensor),
    input (IN_Q8K / IN_F32 / IN_F32_RMS), y (tensor), epilogue, resid, norm_w
    (the RMSNorm weight of an IN_F32_RMS input).  Phase p
    must read phase p-1's complete output.  The tensors must stay alive (and
    in place) while the program exists."""

    def __init__(self, phases, n_cols: int, rms_eps: float = 1e-5):
        from . import Q2KPhase, IN_Q8K
        arr = (Q2KPhase * len(phases))()
        self._keep = []
        for i, ph in enumerate(phases):
            w, x, y = ph["w"], ph["x"], ph["y"]
            epi = ph.get("epilogue", EPI_STORE)
            resid = ph.get("resid")
            mode = ph.get("input", IN_Q8K)
            out_rows = w.n_rows // 2 if epi == EPI_SILU_MUL else w.n_rows
            arr[i].w = w.handle
            arr[i].input = mode
            arr[i].x = x.data_ptr()
            arr[i].ld_x = 0 if mode == IN_Q8K else (x.stride(0) if x.dim() == 2 else w.k)
            arr[i].y = y.data_ptr()
            arr[i].ldy = y.stride(0) if y.dim() == 2 else out_rows
            arr[i].epilogue = epi
            arr[i].resid = 0 if resid is None else resid.data_ptr()
            arr[i].ld_resid = 0 if resid is None else (resid.stride(0) if resid.dim() == 2 else out_rows)
            nw = ph.get("norm_w")
            arr[i].norm_w = 0 if nw is None else nw.data_ptr()
            self._keep += [w, x, y, resid, nw]
        h = ctypes.c_void_p()
        check(lib().smeai_q2k_program_create(arr, len(phases), n_cols, ctypes.c_float(rms_eps), ctypes.byref(h)),
              "q2k_program_create")
        self.handle = h
        self.n_phases = len(phases)

    def run(self):
        check(lib().smeai_q2k_program_run(self.handle, cur_stream()), "q2k_program_run")

    def reset(self):
        check(lib().smeai_q2k_program_reset(self.handle, cur_stream()), "q2k_program_reset")

    def free(self):
        if getattr(self, "handle", None) and self.handle.value:
            lib().smeai_q2k_program_free(self.handle)
            self.handle = ctypes.c_void_p()

    def __del__(self):
        try:
            self.free()
        except Exception:
            pass


class Q2KMGProgram:
    """The decode program over the row shards of several GPUs
    (smeai_q2k_mg_program_*): one per rank, phases wired explicitly.

    phases: dicts with keys w (this rank's shard, Q2KMatrix), input
    (IN_F32 / IN_F32_RMS), x_src / x_row0 (producing phase and its global
    row) or x (outside input tensor), epilogue, resid_src / resid_row0 or
    resid (outside), norm_w, out_rows (global rows), ex_lo / ex_hi / ex_row0
    (local rows exchanged and their global position), y (local output tensor).
    Construction is collective over `group`: the ranks swap the IPC handles of
    their tagged buffers and map each other's; if any rank fails, every rank
    raises RuntimeError (nobody is left waiting in a collective)."""

    def __init__(self, phases, n_cols: int, rank: int, world: int, rms_eps: float = 1e-5, group=None):
        import torch.distributed as dist
        from . import Q2KMGPhase, IN_F32
        arr = (Q2KMGPhase * len(phases))()
        self._keep = []
        for i, ph in enumerate(phases):
            w, y = ph["w"], ph["y"]
            epi = ph.get("epilogue", EPI_STORE)
            x, resid, nw = ph.get("x"), ph.get("resid"), ph.get("norm_w")
            a = arr[i]
            a.w = w.handle
            a.input = ph.get("input", IN_F32)
            a.x_src = ph.get("x_src", -1)
            a.x_row0 = ph.get("x_row0", 0)
            a.x = 0 if x is None else x.data_ptr()
            a.ld_x = 0 if x is None else (x.stride(0) if x.dim() == 2 else w.k)
            a.epilogue = epi
            a.resid_src = ph.get("resid_src", -1)
            a.resid_row0 = ph.get("resid_row0", 0)
            a.resid = 0 if resid is None else resid.data_ptr()
            a.ld_resid = 0 if resid is None else (resid.stride(0) if resid.dim() == 2 else resid.numel())
            a.norm_w = 0 if nw is None else nw.data_ptr()
            a.out_rows = ph["out_rows"]
            a.ex_lo, a.ex_hi, a.ex_row0 = ph.get("ex_lo", 0), ph["ex_hi"], ph.get("ex_row0", 0)
            a.y = y.data_ptr()
            a.ldy = y.stride(0) if y.dim() == 2 else y.numel()
            self._keep += [w, x, resid, nw, y]
        h = ctypes.c_void_p()
        ok = False
        try:
            ok = lib().smeai_q2k_mg_program_create(arr, len(phases), n_cols, ctypes.c_float(rms_eps), rank, world,
                                                   ctypes.byref(h)) == 0
        except Exception:
            ok = False
        err = "" if ok else str(lib().smeai_last_error().decode(errors="replace"))
        handle = (ctypes.c_ubyte * 64)()
        if ok:
            ok = lib().smeai_q2k_program_ipc_handle(h, handle) == 0
        self.handle = h
        self.n_phases = len(phases)
        handles = [None] * world
        if world == 1:
            handles = [bytes(handle) if ok else None]
        else:
            dist.all_gather_object(handles, bytes(handle) if ok else None, group=group)
        if all(x is not None for x in handles):
            blob = (ctypes.c_ubyte * (64 * world)).from_buffer_copy(b"".join(handles))
            ok = lib().smeai_q2k_program_connect(h, blob, world) == 0
            if not ok:
                err = str(lib().smeai_last_error().decode(errors="replace"))
        else:
            ok = False
        oks = [ok]
        if world > 1:
            oks = [None] * world
            dist.all_gather_object(oks, ok, group=group)
        if not all(oks):
            self.free()
            raise RuntimeError(f"multi-GPU program unavailable on some rank ({err or 'a peer failed'})")

    def run(self):
        check(lib().smeai_q2k_program_run(self.handle, cur_stream()), "q2k_program_run")

    def gather(self, phase: int, out: torch.Tensor):
        """Phase `phase`'s global output of the last run (all ranks' rows) into `out`."""
        check(lib().smeai_q2k_program_gather(self.handle, phase, _ptr(out), out.stride(0), cur_stream()),
              "q2k_program_gather")
        return out

    def reset(self):
        check(lib().smeai_q2k_program_reset(self.handle, cur_stream()), "q2k_program_reset")

    def free(self):
        if getattr(self, "handle", None) and self.handle.value:
            lib().smeai_q2k_program_free(self.handle)
            self.handle = ctypes.c_void_p()

    def __del__(self):
        try:
            self.free()
        except Exception:
            pass
