"""A Q2_K tensor loaded from a GGUF file (smeai_gguf_load_q2k) drives the
device GEMV and the tensor-core GEMM to the oracle's result, bit for bit."""
import numpy as np
import pytest
import torch

from gguf_files import write_model

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("rows,k,cols", [(64, 512, 1), (96, 1024, 3), (256, 2048, 40)])
def test_gguf_q2k_weight_matches_oracle(tmp_path, cuda, oracle, rows, k, cols):
    from smeai_b200 import gguf as G
    from smeai_b200 import q2k as Q
    path = tmp_path / "m.gguf"
    ref = write_model(path, oracle, rows=rows, k=k, seed=rows + cols)
    with G.GGUFFile(path) as f:
        m = f.load_q2k("blk.0.attn_q.weight")
    assert (m.n_rows, m.k) == (rows, k)
    rng = np.random.default_rng(cols)
    x = rng.standard_normal((cols, k)).astype(np.float32)
    xq_np = np.concatenate([oracle.quantize_q8_K(x[c]) for c in range(cols)])
    xq = torch.from_numpy(xq_np.view(np.uint8).copy()).to(cuda)
    blocks = ref["q2"].reshape(-1).view(oracle.BLOCK_Q2_K)
    exp = oracle.q2k_mul_mat(blocks, rows, k, xq_np, cols)
    y = m.mul_mat(xq, cols).cpu().numpy()
    assert np.array_equal(y, exp.reshape(cols, rows))
    if cols >= 16:
        assert np.array_equal(m.mul_mat_tc(xq, cols).cpu().numpy(), exp.reshape(cols, rows))
    m.free()
