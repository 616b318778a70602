"""GGUF reader (smeai_gguf.h) against the independent gguf-py 0.19 reader and
writer, on the CPU (the reader is host code; nothing here touches a GPU)."""
import numpy as np
import pytest

from gguf_files import write_model


@pytest.fixture(scope="module")
def G():
    from smeai_b200 import gguf as G
    return G


@pytest.mark.parametrize("alignment", [None, 64])
def test_tensor_table_matches_gguf_py(tmp_path, oracle, G, alignment):
    import gguf
    path = tmp_path / "m.gguf"
    ref = write_model(path, oracle, alignment=alignment)
    r = gguf.GGUFReader(str(path))
    with G.GGUFFile(path) as f:
        assert f.version == 3
        assert f.alignment == (alignment or 32)
        assert [t.name for t in f.tensors] == [t.name for t in r.tensors]
        for mine, theirs in zip(f.tensors, r.tensors):
            assert mine.ggml_type == int(theirs.tensor_type)
            assert mine.shape == tuple(int(v) for v in theirs.shape)
            assert f.data_offset + mine.offset == theirs.data_offset
            assert mine.nbytes == theirs.n_bytes
            assert np.array_equal(f.read(mine.name), np.asarray(theirs.data).view(np.uint8).reshape(-1))
        t = f.by_name["blk.0.attn_q.weight"]
        assert (t.ggml_type, t.shape, t.nbytes) == (G.GGML_Q2_K, (ref["k"], ref["rows"]), ref["q2"].size)
        assert np.array_equal(f.read(t.name), ref["q2"].reshape(-1))
        assert np.array_equal(f.read("blk.0.attn_norm.weight").view(np.float32), ref["norm"])
        assert f.by_name["output.weight"].ggml_type == G.GGML_Q6_K
        assert np.array_equal(f.read("output.weight"), ref["q6"].reshape(-1))
        assert f.find("output.weight") == 2 and f.find("nope") == -1


def test_metadata(tmp_path, oracle, G):
    path = tmp_path / "m.gguf"
    write_model(path, oracle)
    with G.GGUFFile(path) as f:
        assert f.get_int("llama.block_count") == 2
        assert f.get_int("test.big") == 1 << 40
        assert f.get_float("test.neg") == -7.0
        with pytest.raises(G.SmeaiError):
            f.get_int("test.neg")                       # negative: not a u64
        assert f.get_float("llama.rope.freq_base") == 10000.0
        assert f.get_str("general.name") == "smeai-test"
        assert f.get_str("general.architecture") == "llama"
        assert f.key_type("tokenizer.ggml.tokens") == 9   # array
        assert f.get_int("test.flag") == 1
        with pytest.raises(G.SmeaiError):
            f.get_str("missing.key")


def test_malformed_files_are_refused(tmp_path, oracle, G):
    path = tmp_path / "m.gguf"
    write_model(path, oracle)
    data = path.read_bytes()
    cases = {
        "magic": b"GGUX" + data[4:],
        "version1": data[:4] + (1).to_bytes(4, "little") + data[8:],
        "byteswapped": data[:4] + (3).to_bytes(4, "big") + data[8:],
        "truncated_header": data[:40],
        "truncated_data": data[: len(data) - 100],
        "huge_count": data[:8] + (1 << 40).to_bytes(8, "little") + data[16:],
    }
    for name, blob in cases.items():
        bad = tmp_path / f"{name}.gguf"
        bad.write_bytes(blob)
        with pytest.raises(G.SmeaiError):
            G.GGUFFile(bad)
    with pytest.raises(G.SmeaiError):
        G.GGUFFile(tmp_path / "does_not_exist.gguf")


def test_non_q2k_tensor_is_refused_for_q2k_load(tmp_path, oracle, G):
    path = tmp_path / "m.gguf"
    write_model(path, oracle)
    with G.GGUFFile(path) as f:
        with pytest.raises(G.SmeaiError):
            f.load_q2k("output.weight")                  # Q6_K
        with pytest.raises(G.SmeaiError):
            f.load_q2k("blk.0.attn_norm.weight")         # F32, 1-D
