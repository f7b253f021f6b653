"""Generates the golden fixtures in this folder from the reference's own
NumPy GPT-2 (tests/reference.py of llm_mojo), run unmodified.

reference.py reads ../gpt2/model.safetensors relative to its own file, so it
is copied into a temporary tree next to a synthetic checkpoint (random-init
GPT-2 124M, seed 0, as llm_mojo_b200.synth writes it) and imported from
there. Nothing of the reference is written into this repository: only its
outputs, as .npz files.

Run (needs the reference checkout; not run by the tests):
    python tests/golden/make_golden.py /path/to/llm_mojo
"""

from __future__ import annotations

import importlib.util
import os
import shutil
import sys
import tempfile

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))

from llm_mojo_b200 import synth  # noqa: E402


def layer0_only(t: dict) -> dict:
    """The seed-0 weights with every matrix of layers 1-11 set to zero: those
    layers then add exactly 0 to the residual stream (their attention and MLP
    outputs are 0), so the model is one layer deep and rounding differences
    are not amplified through depth."""
    t = dict(t)
    for l in range(1, 12):
        for name in synth.MAT_NAMES:
            t[f"h.{l}.{name}"] = np.zeros_like(t[f"h.{l}.{name}"])
    return t


def load_reference(ref_root: str, tmp: str, tensors: dict):
    os.makedirs(os.path.join(tmp, "gpt2"))
    os.makedirs(os.path.join(tmp, "tests"))
    synth.write_safetensors(tensors, os.path.join(tmp, "gpt2", "model.safetensors"))
    shutil.copy(os.path.join(ref_root, "tests", "reference.py"), os.path.join(tmp, "tests", "reference.py"))
    spec = importlib.util.spec_from_file_location("llm_mojo_reference", os.path.join(tmp, "tests", "reference.py"))
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def configure(ref, quant=None, quant_head=None, act16=False, kv=None, gguf_path=None):
    ref.QUANT, ref.QUANT_HEAD, ref.ACT16, ref.KV = quant, quant_head, act16, kv
    if gguf_path is None:
        ref.GGUF = None
    else:
        from gguf import GGUFReader

        ref.GGUF = GGUFReader(gguf_path)
    ref._cache.clear()


def bf16_weights(t: dict) -> dict:
    """The seed-0 weights with the matrices gpt2t's bf16 format stores as
    bfloat16 (the four per-layer matrices and wte) rounded to bfloat16, as
    DenseMatrix[bf16] holds them; the small tensors stay float32."""
    t = dict(t)
    for name in list(t):
        if name == "wte.weight" or any(name.endswith(m) for m in synth.MAT_NAMES):
            b = np.ascontiguousarray(t[name], dtype=np.float32).view(np.uint32).astype(np.uint64)
            b = ((b + 0x7FFF + ((b >> 16) & 1)) >> 16) << 16
            t[name] = b.astype(np.uint32).view(np.float32)
    return t


def model_goldens(ref, out: dict, tag: str, prompt) -> None:
    """Logits after [EOT], after the 24-token prompt, at all positions of its
    first 16 tokens, and 8 greedy ids from [EOT]: top ids / values and the
    largest |logit| (the tolerance's scale)."""
    lg = ref.forward([synth.EOT]).astype(np.float32)
    out[f"{tag}_eot_top_ids"], out[f"{tag}_eot_top_vals"] = topk(lg)
    out[f"{tag}_eot_max"] = np.float32(np.abs(lg).max())
    toks = [synth.EOT]
    for _ in range(8):
        toks.append(int(np.argmax(ref.forward(toks))))
    out[f"{tag}_greedy8"] = np.array(toks[1:], dtype=np.int32)
    lg = ref.forward(list(prompt)).astype(np.float32)
    out[f"{tag}_p24_top_ids"], out[f"{tag}_p24_top_vals"] = topk(lg)
    out[f"{tag}_p24_max"] = np.float32(np.abs(lg).max())
    allp = ref.forward(list(prompt[:16]), all_positions=True).astype(np.float32)
    out[f"{tag}_all16_top_ids"] = np.stack([topk(r, 8)[0] for r in allp])
    out[f"{tag}_all16_top_vals"] = np.stack([topk(r, 8)[1] for r in allp])
    out[f"{tag}_all16_max"] = np.float32(np.abs(allp).max())


def topk(logits, k=32):
    idx = np.argsort(-logits, kind="stable")[:k]
    return idx.astype(np.int32), logits[idx].astype(np.float32)


def main(ref_root: str):
    out = {}
    with tempfile.TemporaryDirectory() as tmp:
        ref = load_reference(ref_root, tmp, layer0_only(synth.gpt2_random_init(0)))
        prompt = np.random.default_rng(2).integers(0, synth.V, size=24).astype(np.int64)
        for tag, cfg in [("l0_f32", {}),
                         ("l0_a16", dict(quant=(4, 32, False), quant_head=(8, 0, False), act16=True, kv="int8"))]:
            configure(ref, **cfg)
            lg = ref.forward([synth.EOT]).astype(np.float32)
            out[f"{tag}_eot_top_ids"], out[f"{tag}_eot_top_vals"] = topk(lg)
            out[f"{tag}_eot_max"] = np.float32(np.abs(lg).max())
            lg = ref.forward(list(prompt)).astype(np.float32)
            out[f"{tag}_p24_top_ids"], out[f"{tag}_p24_top_vals"] = topk(lg)
            out[f"{tag}_p24_max"] = np.float32(np.abs(lg).max())
    with tempfile.TemporaryDirectory() as tmp:
        ref = load_reference(ref_root, tmp, synth.gpt2_random_init(0))

        # 1. The quantizer: reference.fake_quant on a seeded matrix, per format.
        rng = np.random.default_rng(7)
        w = (rng.standard_normal((128, 128), dtype=np.float32) * np.float32(0.02)).astype(np.float32)
        for bits, group, sym in [(4, 32, 0), (4, 32, 1), (4, 64, 0), (4, 128, 0), (4, 0, 1), (8, 0, 0), (8, 32, 0)]:
            out[f"fq_{bits}_{group}_{sym}"] = ref.fake_quant(w, bits, group, bool(sym), reduce_rows=True)
            out[f"fqh_{bits}_{group}_{sym}"] = ref.fake_quant(w, bits, group, bool(sym), reduce_rows=False)
        out["fq_src"] = w

        # 2. Activation (aq) and KV (kvq) fake quantization.
        x = (rng.standard_normal((3, 768), dtype=np.float32) * np.float32(1.5)).astype(np.float32)
        out["aq_src"] = x
        out["aq"] = ref.aq(x, force=True)
        kv = rng.standard_normal((12, 5, 64), dtype=np.float32).astype(np.float32)
        out["kvq_src"] = kv
        configure(ref, kv="int8")
        out["kvq_int8"] = ref.kvq(kv)

        # 3. Whole-model logits and greedy ids: f32; int4-g32-a16 with an
        # int8 head and int8 KV cache (gpt2t --dtype int4-g32-a16 defaults);
        # int4-g32 (W4A32: the same weights, float activations, the int8
        # head, and the float32 cache of gpt2t --dtype int4-g32 --kv f32, so
        # that no int8 KV rounding flips enter the float comparison).
        prompt = np.random.default_rng(2).integers(0, synth.V, size=24).astype(np.int64)
        out["prompt24"] = prompt.astype(np.int32)
        for tag, cfg in [("f32", {}),
                         ("a16", dict(quant=(4, 32, False), quant_head=(8, 0, False), act16=True, kv="int8")),
                         ("wa32", dict(quant=(4, 32, False), quant_head=(8, 0, False), act16=False, kv="f32"))]:
            configure(ref, **cfg)
            model_goldens(ref, out, tag, prompt)

        # 4. A GGUF file of the same weights (Q4_K layers, Q6_K tied head,
        # float32 small tensors; the layout of GPT-2's Q4_K_M files), read
        # by reference.py's --gguf path (gguf-py dequantization, int16 head
        # input), with the int8 KV cache gpt2t uses for GGUF models.
        sys.path.insert(0, os.path.join(os.path.dirname(HERE)))
        from gguf_file import write_gpt2_gguf

        gpath = os.path.join(tmp, "gpt2_q4_k.gguf")
        write_gpt2_gguf(gpath, synth.gpt2_random_init(0))
        configure(ref, kv="int8", gguf_path=gpath)
        model_goldens(ref, out, "gguf", prompt)
    # 5. bf16: the reference model on bfloat16-rounded matrices with the
    # bfloat16 KV cache (kvcache.mojo DenseKV[bf16]).
    with tempfile.TemporaryDirectory() as tmp:
        ref = load_reference(ref_root, tmp, bf16_weights(synth.gpt2_random_init(0)))
        configure(ref, kv="bf16")
        model_goldens(ref, out, "bf16", prompt)
    np.savez_compressed(os.path.join(HERE, "reference_py.npz"), **out)
    print("wrote", os.path.join(HERE, "reference_py.npz"))


if __name__ == "__main__":
    if len(sys.argv) != 2:
        sys.exit("usage: python tests/golden/make_golden.py /path/to/llm_mojo")
    main(sys.argv[1])
