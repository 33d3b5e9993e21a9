"""A small GGUF file of MoE expert tensors written with gguf-py, for the tests of the hot
method's GGUF access: E experts, gate / up [E, INTER, row_bytes(K)] and down [E, K,
row_bytes(INTER)] per layer, N(0, 0.02) weights quantized by the package's encoders."""
import numpy as np

from kt_gguf_b200 import synth

E, K, INTER, LAYERS = 6, 512, 512, (0, 1)


def write_gguf(path, types=(12, 12, 14), seed=0):
    """writes the file; returns {(layer, proj): uint8 [E, rows, row_bytes]}"""
    from gguf import GGMLQuantizationType, GGUFWriter

    rng = np.random.default_rng(seed)
    w = GGUFWriter(str(path), "qwen3moe")
    w.add_expert_count(E)
    w.add_embedding_length(K)
    w.add_expert_feed_forward_length(INTER)
    data = {}
    for li in LAYERS:
        for proj, t in zip(("gate", "up", "down"), types):
            rows, cols = (INTER, K) if proj != "down" else (K, INTER)
            b = np.stack([synth.quantize(rng.standard_normal((rows, cols), dtype=np.float32) * 0.02, t)
                          for _ in range(E)])
            w.add_tensor(f"blk.{li}.ffn_{proj}_exps.weight", b, raw_shape=b.shape, raw_dtype=GGMLQuantizationType(t))
            data[(li, proj)] = b
    w.write_header_to_file()
    w.write_kv_data_to_file()
    w.write_tensors_to_file()
    w.close()
    return data
