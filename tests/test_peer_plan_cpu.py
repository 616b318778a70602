"""CPU check of the fused-exchange plan of the row-sharded decode stack
(smeai_b200.peer.decode_plan): every rank's GEMVs, run in step order with the
plan's destinations, signal words and wait counts, must rebuild on every
rank exactly the activations of the unsharded stack, and each wait must find
its word at exactly the target the kernels compute ((epoch + 1) * count).

The device kernels follow the same rules: the rows of a finished 32-row group
at or past row0 (16 output rows per group for the gate/up pair) are stored to
every destination, and every finished group bumps the signal word on every
rank once."""
import math

import numpy as np
import pytest

from smeai_b200.peer import decode_plan, exchange_groups
from smeai_b200.stack import shard_range

P = 1_000_003  # exact modular arithmetic stands in for the GEMVs


def _mats(H, F, V, L, rng):
    m = lambda r, c: rng.integers(0, 97, size=(r, c), dtype=np.int64)
    layers = [dict(q=m(H, H), k=m(H, H), v=m(H, H), o=m(H, H), g=m(F, H), u=m(F, H), d=m(H, F)) for _ in range(L)]
    return layers, m(V, H)


def _reference(x, layers, lm):
    x = x.copy()
    for w in layers:
        v = w["v"] @ x % P
        x = (x + w["o"] @ v) % P
        h = (w["g"] @ x % P) * (w["u"] @ x % P) % P
        x = (x + w["d"] @ h) % P
    return lm @ x % P


@pytest.mark.parametrize("world", [2, 4])
@pytest.mark.parametrize("steps", [1, 3])
def test_plan_rebuilds_unsharded_activations(world, steps):
    H, F, V, L = 256, 512, 384, 2
    rng = np.random.default_rng(world)
    layers, lm = _mats(H, F, V, L, rng)
    x0 = rng.integers(0, 97, size=H, dtype=np.int64)
    ref = _reference(x0, layers, lm)
    plans = [decode_plan(H, F, V, L, r, world, shard_range) for r in range(world)]
    bufs = [dict(x=np.zeros(H, np.int64), v=np.zeros(H, np.int64), h=np.zeros(F, np.int64),
                 lg=np.zeros(V, np.int64)) for _ in range(world)]
    sig = np.zeros((world, 4 * L + 1), np.int64)
    epoch = [0] * world
    lo = lambda n, r: shard_range(n, r, world)
    for _ in range(steps):
        for r in range(world):
            bufs[r]["x"][:] = x0
        for i in range(len(plans[0])):
            for r in range(world):
                name, dst, ld, row0, s, wait, count = plans[r][i]
                if wait is not None:
                    assert sig[r][wait] == (epoch[r] + 1) * count, (name, r)
                if name == "end":
                    epoch[r] += 1
                    continue
                li = min(i // 4, L - 1)
                w, b = layers[li], bufs[r]
                (h0, h1), (f0, f1), (v0, v1) = lo(H, r), lo(F, r), lo(V, r)
                if name == "qkv":
                    out = np.concatenate([w["q"][h0:h1] @ b["x"], w["k"][h0:h1] @ b["x"], w["v"][h0:h1] @ b["x"]]) % P
                    n_rows, per = out.size, 32
                elif name == "o":
                    out = (b["x"][h0:h1] + w["o"][h0:h1] @ b["v"]) % P
                    b["x"][h0:h1] = out
                    n_rows, per = out.size, 32
                elif name == "gate_up":
                    out = (w["g"][f0:f1] @ b["x"] % P) * (w["u"][f0:f1] @ b["x"] % P) % P
                    b["h"][f0:f1] = out
                    n_rows, per = 2 * out.size, 16      # interleaved pairs: 16 outputs per group
                elif name == "down":
                    out = (b["x"][h0:h1] + w["d"][h0:h1] @ b["h"]) % P
                    b["x"][h0:h1] = out
                    n_rows, per = out.size, 32
                else:
                    out = lm[v0:v1] @ b["x"] % P
                    b["lg"][v0:v1] = out
                    n_rows, per = out.size, 32
                for g in range(math.ceil(n_rows / 32)):       # the finisher, one row group at a time
                    a = g * per
                    if a >= row0:
                        rows = out[a:min(a + per, out.size)]
                        for q, buf, off in dst:
                            bufs[q][buf][off + a - row0:off + a - row0 + rows.size] = rows
                    sig[:, s] += 1                              # every group signals
            # all ranks finish GEMV i before any starts GEMV i + 1 (what the waits enforce)
    for r in range(world):
        assert np.array_equal(bufs[r]["lg"], ref), r
        assert epoch[r] == steps


def test_exchange_group_counts():
    assert exchange_groups([512] * 8) == 128
    assert exchange_groups([2 * 1376] * 8) == 688
    assert exchange_groups([4000] * 8) == 1000
    assert exchange_groups([33, 31]) == 3
