"""TEST INFRASTRUCTURE: writes a llama.cpp-style GGUF file of the synthetic
GPT-2 (GGUF Q4_K layers, Q6_K tied token_embd, float32 small tensors) with
the gguf package's writer; the same blocks FloatModel('gguf-q4_k') packs."""

import numpy as np


def write_gpt2_gguf(path: str, tensors: dict, n_layer: int = 12, head=None):
    """head: an untied [V, C] output matrix, written as output.weight (Q6_K)."""
    import gguf

    from llm_mojo_b200 import gguf_blocks as G

    w = gguf.GGUFWriter(path, "gpt2")
    w.add_uint32("general.alignment", 32)
    w.add_string("general.name", "synthetic gpt2")

    def quant(name, a, t, qt):
        w.add_tensor(name, G.quantize(np.ascontiguousarray(a), t), raw_dtype=qt)  # byte shape [rows, row bytes]

    Q = gguf.GGMLQuantizationType
    quant("token_embd.weight", tensors["wte.weight"], G.Q6_K, Q.Q6_K)
    w.add_tensor("position_embd.weight", np.ascontiguousarray(tensors["wpe.weight"], dtype=np.float32))
    mats = {"attn_qkv": "attn.c_attn.weight", "attn_output": "attn.c_proj.weight", "ffn_up": "mlp.c_fc.weight",
            "ffn_down": "mlp.c_proj.weight"}
    vecs = {"attn_norm.weight": "ln_1.weight", "attn_norm.bias": "ln_1.bias", "attn_qkv.bias": "attn.c_attn.bias",
            "attn_output.bias": "attn.c_proj.bias", "ffn_norm.weight": "ln_2.weight", "ffn_norm.bias": "ln_2.bias",
            "ffn_up.bias": "mlp.c_fc.bias", "ffn_down.bias": "mlp.c_proj.bias"}
    for l in range(n_layer):
        for g, hf in mats.items():
            quant(f"blk.{l}.{g}.weight", np.ascontiguousarray(tensors[f"h.{l}.{hf}"].T), G.Q4_K, Q.Q4_K)
        for g, hf in vecs.items():
            w.add_tensor(f"blk.{l}.{g}", np.ascontiguousarray(tensors[f"h.{l}.{hf}"], dtype=np.float32))
    if head is not None:
        quant("output.weight", head, G.Q6_K, Q.Q6_K)
    w.add_tensor("output_norm.weight", np.ascontiguousarray(tensors["ln_f.weight"], dtype=np.float32))
    w.add_tensor("output_norm.bias", np.ascontiguousarray(tensors["ln_f.bias"], dtype=np.float32))
    w.write_header_to_file()
    w.write_kv_data_to_file()
    w.write_tensors_to_file()
    w.close()
