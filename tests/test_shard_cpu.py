"""CPU tests of the multi-GPU sharding logic with real 2-rank gloo process
groups: each rank computes its row slice of Q2_K mul_mats with the oracle and
the slices are gathered by the same gather_rows the GPU stack uses; the result
must equal the unsharded computation bit for bit."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _worker(rank, world, port, cases, results):
    import sys
    root = os.path.abspath(os.path.join(os.path.dirname(__file__), ".."))
    for p in (root, os.path.join(root, "sme-ai-ops_b200")):
        if p not in sys.path:
            sys.path.insert(0, p)
    from oracle import oracle as O
    from smeai_b200.stack import gather_rows, shard_range
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        out = []
        for rows, k, cols, seed in cases:
            rng = np.random.default_rng(seed)
            w = O.quantize_q2_K((rng.standard_normal(rows * k) * 0.02).astype(np.float32))
            xq = O.quantize_q8_K(rng.standard_normal(cols * k).astype(np.float32))
            lo, hi = shard_range(rows, rank, world)
            nb = k // 256
            local = O.q2k_mul_mat(w[lo * nb:hi * nb], hi - lo, k, xq, cols) if hi > lo else \
                np.zeros((cols, 0), np.float32)
            full = torch.empty((cols, rows))
            gather_rows(full, torch.from_numpy(np.ascontiguousarray(local)), rows, world)
            out.append(full.numpy().copy())
        results[rank] = out
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2])
def test_sharded_mul_mat_equals_unsharded(oracle, world):
    # (rows, k, cols, seed): even shards with one column (the direct gather),
    # an uneven last shard, several columns (the padded gather), a tiny matrix
    cases = [(128, 512, 1, 1), (100, 256, 1, 2), (96, 512, 3, 3), (40, 256, 2, 4)]
    mgr = mp.get_context("spawn").Manager()
    results = mgr.dict()
    mp.start_processes(_worker, args=(world, _free_port(), cases, results), nprocs=world, start_method="spawn")
    for ci, (rows, k, cols, seed) in enumerate(cases):
        rng = np.random.default_rng(seed)
        w = oracle.quantize_q2_K((rng.standard_normal(rows * k) * 0.02).astype(np.float32))
        xq = oracle.quantize_q8_K(rng.standard_normal(cols * k).astype(np.float32))
        exp = oracle.q2k_mul_mat(w, rows, k, xq, cols)
        for r in range(world):
            assert np.array_equal(results[r][ci].view(np.uint32), exp.view(np.uint32)), (ci, r)


def test_shard_ranges_cover_rows():
    import sys
    sys.path.insert(0, os.path.join(os.path.dirname(__file__), "..", "sme-ai-ops_b200"))
    from smeai_b200.stack import shard_range, shard_stride
    for n in (40, 100, 4096, 11008, 12288, 32000):
        for world in (1, 2, 3, 4, 8):
            spans = [shard_range(n, r, world) for r in range(world)]
            assert spans[0][0] == 0 and spans[-1][1] == n
            assert all(a[1] == b[0] for a, b in zip(spans, spans[1:]))
            assert all(hi - lo <= shard_stride(n, world) for lo, hi in spans)
            assert all(lo % 32 == 0 or lo == hi == n for lo, hi in spans)


def test_token_ranges_partition_tokens():
    """Sequence sharding of a prefill: the ranks' token ranges tile the batch
    in order and differ in size by at most one."""
    import sys
    sys.path.insert(0, os.path.join(os.path.dirname(__file__), "..", "sme-ai-ops_b200"))
    from smeai_b200.stack import token_range
    for n in (8, 130, 512, 513):
        for world in (1, 2, 3, 4, 8):
            spans = [token_range(n, r, world) for r in range(world)]
            assert spans[0][0] == 0 and spans[-1][1] == n
            assert all(a[1] == b[0] for a, b in zip(spans, spans[1:]))
            sizes = [hi - lo for lo, hi in spans]
            assert max(sizes) - min(sizes) <= 1 and min(sizes) >= 1
