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


def _worker(rank, world, port, failing, results):
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
        L = S.lib()
        if rank in failing:
            L.smeai_ipc_alloc = lambda *args: -2   # this rank's allocation fails
        try:
            PeerArena([("x", 1024), ("sig", 64)], None, rank, world)
            results[rank] = "ok"
        except PeerUnavailable:
            results[rank] = "unavailable"
        dist.barrier()                            # the ranks are still in step
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("failing", [(1,), (0,), (0, 1)])
def test_arena_failure_is_shared_by_all_ranks(failing):
    world = 2
    results = mp.get_context("spawn").Manager().dict()
    mp.start_processes(_worker, args=(world, _free_port(), failing, results), nprocs=world, start_method="spawn")
    assert [results[r] for r in range(world)] == ["unavailable"] * world
