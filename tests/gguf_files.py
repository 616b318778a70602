"""GGUF test files written by the independent gguf-py writer (gguf 0.19):
metadata of several value types, a Q2_K weight (blocks from the oracle's
quantizer), an F32 vector and a Q6_K weight (random block bytes)."""
import numpy as np

QK = 256


def write_model(path, oracle, rows=64, k=512, alignment=None, seed=0):
    import gguf
    rng = np.random.default_rng(seed)
    w = (rng.standard_normal((rows, k)) * 0.02).astype(np.float32)
    q2 = oracle.quantize_q2_K(w.reshape(-1)).view(np.uint8).reshape(rows, k // QK * 84)
    norm = rng.standard_normal(k).astype(np.float32)
    q6 = rng.integers(0, 256, size=(8, 210), dtype=np.uint8)          # one Q6_K row of 256
    wr = gguf.GGUFWriter(str(path), arch="llama")
    wr.add_uint32("llama.block_count", 2)
    wr.add_uint64("test.big", 1 << 40)
    wr.add_int32("test.neg", -7)
    wr.add_float32("llama.rope.freq_base", 10000.0)
    wr.add_string("general.name", "smeai-test")
    wr.add_array("tokenizer.ggml.tokens", ["<s>", "</s>", "hello"])
    wr.add_array("tokenizer.ggml.scores", [0.0, -1.5, 2.25])
    wr.add_bool("test.flag", True)
    if alignment:
        wr.add_custom_alignment(alignment)
    wr.add_tensor("blk.0.attn_q.weight", q2, raw_dtype=gguf.GGMLQuantizationType.Q2_K)
    wr.add_tensor("blk.0.attn_norm.weight", norm)
    wr.add_tensor("output.weight", q6.reshape(8, 210), raw_dtype=gguf.GGMLQuantizationType.Q6_K)
    wr.write_header_to_file()
    wr.write_kv_data_to_file()
    wr.write_tensors_to_file()
    wr.close()
    return dict(q2=q2, norm=norm, q6=q6, rows=rows, k=k)
