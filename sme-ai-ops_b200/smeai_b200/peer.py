"""Cross-GPU exchange for the row-sharded decode stack.

Every rank owns one CUDA-IPC-shareable device arena (smeai_ipc_alloc) with the
same layout on all ranks: the replicated activations each row-sharded GEMV
gathers into (v, x, h, logits), the signal words of the fused exchange and
the rank's step counter.  The ranks swap their arena handles once over the
process group and map each other's arenas (smeai_ipc_open), so a GEMV's
finisher can store its rows into every rank's copy and bump every rank's
signal word in the same kernel (smeai_q2k_mul_mat_f32_peer).
"""
from __future__ import annotations

import contextlib
import ctypes
import math

import torch
import torch.distributed as dist

from . import PeerExchange, lib

_ALIGN = 256


class _DeviceSpan:
    """Raw device memory as a __cuda_array_interface__ object (bytes)."""

    def __init__(self, ptr: int, nbytes: int):
        self.__cuda_array_interface__ = {"shape": (nbytes,), "typestr": "|u1", "data": (ptr, False),
                                         "version": 3, "strides": None}


def exchange_groups(rows_per_rank, rows_per_group: int = 32) -> int:
    """Row groups all ranks publish for one exchanged output (the wait count)."""
    return sum(math.ceil(r / rows_per_group) for r in rows_per_rank)


def decode_plan(H: int, F: int, V: int, L: int, rank: int, world: int, shard_range):
    """The fused exchanges of one rank's decode step (pure bookkeeping).

    One entry per GEMV, in step order: (name, dst, ld, row0, sig, wait, count)
      dst    [(rank, buffer, element offset)] the rows are stored to
      ld     the destination's token stride (elements)
      row0   first exchanged local output row
      sig    index of the signal word bumped on every rank
      wait   index of this rank's signal word waited on (None: no wait)
      count  row groups all ranks publish behind `wait` per step (every group of
             the producing GEMV signals, also those whose rows are not stored)
    Signal words: 4 per layer (v, x after o, h, x after down), then logits.
    A final ("end", ..., wait = the logits word) entry closes the step."""
    rows = lambda n: [shard_range(n, q, world)[1] - shard_range(n, q, world)[0] for q in range(world)]
    hs_all, fs_all, vs_all = rows(H), rows(F), rows(V)
    n_h, n_f, n_v = exchange_groups(hs_all), exchange_groups([2 * f for f in fs_all]), exchange_groups(vs_all)
    n_qkv = exchange_groups([3 * h for h in hs_all])   # every group signals, q and k rows included
    h_lo, f_lo, v_lo = shard_range(H, rank, world)[0], shard_range(F, rank, world)[0], shard_range(V, rank, world)[0]
    hs = hs_all[rank]
    others = [q for q in range(world) if q != rank]
    plan = []
    for li in range(L):
        b = 4 * li
        plan += [
            ("qkv", [(q, "v", h_lo) for q in range(world)], H, 2 * hs, b, b - 1 if li else None, n_h),
            ("o", [(q, "x", h_lo) for q in others], H, 0, b + 1, b, n_qkv),
            ("gate_up", [(q, "h", f_lo) for q in others], F, 0, b + 2, b + 1, n_h),
            ("down", [(q, "x", h_lo) for q in others], H, 0, b + 3, b + 2, n_f),
        ]
    plan.append(("lm_head", [(q, "lg", v_lo) for q in others], V, 0, 4 * L, 4 * L - 1, n_h))
    plan.append(("end", [], 0, 0, None, 4 * L, n_v))
    return plan


class PeerUnavailable(RuntimeError):
    """Some rank could not allocate, export or map an arena (all ranks raise it)."""


class PeerArena:
    """`layout`: list of (name, bytes).  After construction, tensor(name, ...)
    views this rank's buffer and addr(q, name, byte_offset) is the address, in
    this process, of rank q's buffer (its own or a peer mapping)."""

    def __init__(self, layout, device, rank: int, world: int, group=None):
        self.rank, self.world, self.device = rank, world, device
        self.off, total = {}, 0
        for name, nbytes in layout:
            self.off[name] = total
            total += (nbytes + _ALIGN - 1) // _ALIGN * _ALIGN
        self.nbytes = total
        L = lib()
        ptr, handle = ctypes.c_void_p(), (ctypes.c_ubyte * 64)()
        on_dev = lambda: torch.cuda.device(device) if device is not None else contextlib.nullcontext()
        # every rank takes part in both exchanges, so a local failure (an error
        # code or an exception) cannot leave the others waiting in a
        # collective; the decision is shared
        try:
            with on_dev():
                ok = L.smeai_ipc_alloc(total, ctypes.byref(ptr), handle) == 0
        except Exception:
            ok = False
        self.local = ptr.value if ok else 0
        self.base, self._opened, self._span = [0] * world, [], None
        handles = [None] * world
        dist.all_gather_object(handles, bytes(handle) if ok else None, group=group)
        if all(h is not None for h in handles):
            for q in range(world):
                if q == rank:
                    self.base[q] = self.local
                    continue
                hq = (ctypes.c_ubyte * 64).from_buffer_copy(handles[q])
                pq = ctypes.c_void_p()
                try:
                    with on_dev():
                        opened = L.smeai_ipc_open(hq, ctypes.byref(pq)) == 0
                except Exception:
                    opened = False
                if not opened:
                    ok = False
                    break
                self.base[q] = pq.value
                self._opened.append(pq.value)
        else:
            ok = False
        oks = [None] * world
        dist.all_gather_object(oks, ok, group=group)
        if not all(oks):
            self.close()
            raise PeerUnavailable("peer memory unavailable on some rank")
        self._span = torch.as_tensor(_DeviceSpan(self.local, total), device=device)

    def tensor(self, name: str, dtype: torch.dtype, shape) -> torch.Tensor:
        n = math.prod(shape) * torch.empty((), dtype=dtype).element_size()
        o = self.off[name]
        return self._span[o:o + n].view(dtype).view(*shape)

    def addr(self, q: int, name: str, byte_offset: int = 0) -> int:
        return self.base[q] + self.off[name] + byte_offset

    def close(self):
        L = lib()
        for p in self._opened:
            L.smeai_ipc_close(ctypes.c_void_p(p))
        self._opened = []
        if self.local:
            self._span = None
            L.smeai_ipc_free(ctypes.c_void_p(self.local))
            self.local = 0


def make_exchange(dst=(), ld_dst: int = 0, row0: int = 0, sig=(), wait_sig: int = 0, wait_count: int = 0,
                  epoch: int = 0) -> PeerExchange:
    assert len(dst) <= 8 and len(sig) <= 8
    ex = PeerExchange()
    ex.n_dst, ex.ld_dst, ex.row0, ex.n_sig = len(dst), ld_dst, row0, len(sig)
    for i, a in enumerate(dst):
        ex.dst[i] = a
    for i, a in enumerate(sig):
        ex.sig[i] = a
    ex.wait_sig = wait_sig or None
    ex.wait_count = wait_count
    ex.epoch = epoch or None
    return ex
