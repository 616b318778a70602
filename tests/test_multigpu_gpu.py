"""Row-sharded decode stack on 2 (and 4) GPUs against the single-GPU stack,
with NCCL all-gathers ("separate"), with the all-gather fused into each GEMV
over CUDA-IPC peer memory ("peer"), and as one persistent kernel per rank
whose finishers store every row into every rank's copy ("mgprog", the
default on several GPUs): logits must be bit-identical (sharding only moves
rows between GPUs; every row's arithmetic is unchanged), eagerly and from a
CUDA graph replayed twice (2, 4 and 8 ranks).  Skips without enough GPUs."""
import datetime
import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu

DIMS = dict(n_layers=2, hidden=1024, ffn=2816, vocab=4096, seed=11)


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _rank(rank, world, port, quant, results):
    import sys
    root = os.path.abspath(os.path.join(os.path.dirname(__file__), ".."))
    for p in (root, os.path.join(root, "sme-ai-ops_b200")):
        if p not in sys.path:
            sys.path.insert(0, p)
    import torch.distributed as dist
    from smeai_b200.stack import Q2KDecodeStack
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=dev)
    try:
        st = Q2KDecodeStack(rank=rank, world=world, device=dev, quant=quant, **DIMS)
        assert st.quant == quant, st.quant
        eager = st.step().clone()
        stream = torch.cuda.Stream()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=stream):
            st.step()
        graphed = []
        for _ in range(2):
            with torch.cuda.stream(stream):
                g.replay()
            stream.synchronize()
            graphed.append(st.logits.cpu().clone())
        import smeai_b200 as S
        code = S.take_device_error()
        results[rank] = (eager.cpu(), graphed, code)
        del g
        dist.barrier()
        st.free()
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world,quant", [(2, "separate"), (2, "peer"), (2, "mgprog"), (4, "mgprog"), (8, "mgprog")])
def test_sharded_stack_matches_single_gpu(cuda, world, quant):
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    from smeai_b200.stack import Q2KDecodeStack
    ref = Q2KDecodeStack(device=cuda, **DIMS).step().cpu().clone()
    torch.cuda.synchronize()
    results = mp.get_context("spawn").Manager().dict()
    mp.start_processes(_rank, args=(world, _port(), quant, results), nprocs=world, start_method="spawn")
    for r in range(world):
        eager, graphed, code = results[r]
        assert code == 0, (r, code)
        assert torch.equal(eager, ref), r
        for gl in graphed:
            assert torch.equal(gl, ref), r
