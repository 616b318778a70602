"""Host-side failure handling of the cross-GPU exchange set-up, with real 2-rank
gloo process groups on CPU: when one rank cannot allocate (or export, or map)
its peer arena, every rank must learn it in the same collective steps and
raise PeerUnavailable -- the decode stack then falls back to NCCL all-gathers
on all ranks together -- instead of one rank waiting forever in a collective
the other never joins.  The failure is made on the host (a failing allocation
call), as the GPU is never faulted on purpose."""
import os
import socket

import pytest
import torch.distributed as dist
import torch.multiprocessing as mp


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _install_fakes(L, rank, fail_alloc, fail_open, calls):
    """Host fakes of the four IPC calls: a healthy rank 'allocates' a fake
    arena (address and 64-byte handle derived from its rank) and 'maps' the
    peers' handles, so the collective decision runs exactly as it would on
    GPUs; every call is recorded."""
    def alloc(total, ptr_ref, handle):
        calls.append("alloc")
        if fail_alloc:
            return -2                                   # cudaMalloc failed
        ptr_ref._obj.value = 0x10000000 * (rank + 1)
        for i in range(64):
            handle[i] = (rank * 64 + i) & 0xFF
        return 0

    def open_(handle, ptr_ref):
        calls.append("open")
        if fail_open:
            return -5                                   # the peer mapping failed
        ptr_ref._obj.value = 0x70000000 + handle[0]
        return 0

    L.smeai_ipc_alloc = alloc
    L.smeai_ipc_open = open_
    L.smeai_ipc_close = lambda p: calls.append("close")
    L.smeai_ipc_free = lambda p: calls.append("free")


def _worker(rank, world, port, fail_alloc, fail_open, results):
    import sys
    root = os.path.abspath(os.path.join(os.path.dirname(__file__), ".."))
    for p in (root, os.path.join(root, "sme-ai-ops_b200")):
        if p not in sys.path:
            sys.path.insert(0, p)
    import smeai_b200 as S
    from smeai_b200.peer import PeerArena, PeerUnavailable
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        calls = []
        _install_fakes(S.lib(), rank, rank in fail_alloc, rank in fail_open, calls)
        try:
            PeerArena([("x", 1024), ("sig", 64)], None, rank, world)
            outcome = "ok"
        except PeerUnavailable:
            outcome = "unavailable"
        dist.barrier()                            # the ranks are still in step
        results[rank] = (outcome, tuple(calls))
    finally:
        dist.destroy_process_group()


def _run(fail_alloc=(), fail_open=()):
    world = 2
    results = mp.get_context("spawn").Manager().dict()
    mp.start_processes(_worker, args=(world, _free_port(), fail_alloc, fail_open, results), nprocs=world,
                       start_method="spawn")
    return [results[r] for r in range(world)]


@pytest.mark.parametrize("failing", [(1,), (0,), (0, 1)])
def test_arena_failure_is_shared_by_all_ranks(failing):
    """One rank's allocation fails: every rank raises, and a rank whose own
    allocation succeeded frees it (and maps nothing)."""
    res = _run(fail_alloc=failing)
    for rank, (outcome, calls) in enumerate(res):
        assert outcome == "unavailable", (rank, res)
        if rank in failing:
            assert calls == ("alloc",), (rank, calls)
        else:
            assert calls == ("alloc", "free"), (rank, calls)


def test_peer_mapping_failure_is_shared_by_all_ranks():
    """Every rank allocates, rank 1 cannot map rank 0's arena: both raise,
    rank 0 closes the mapping it did open, and both free their arenas."""
    res = _run(fail_open=(1,))
    (o0, c0), (o1, c1) = res
    assert o0 == o1 == "unavailable", res
    assert c0 == ("alloc", "open", "close", "free"), c0
    assert c1 == ("alloc", "open", "free"), c1
