"""Saved weights (.llmm, the reference's --save / --weights layout) and GGUF
files: a model read back must give the same logits and ids as the one
written; the generic one-token decode of the float formats is deterministic
and agrees with the forward pass."""

import os
import struct

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def torch():
    import torch

    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return torch


@pytest.fixture(scope="module")
def ctx(torch):
    from llm_mojo_b200 import build
    from llm_mojo_b200.tensor import Context

    build.build()
    c = Context(0)
    yield c
    c.close()


def _header(path):
    """magic, version, layer format, head format of a saved file (the
    serialize.mojo encoding, read independently of the library)."""
    with open(path, "rb") as f:
        def i64():
            return struct.unpack("<q", f.read(8))[0]

        def s():
            return f.read(i64()).decode()

        return s(), i64(), s(), s()


def test_a16_model_save_load_round_trip(torch, ctx, gpt2_tensors, tmp_path):
    from llm_mojo_b200.model import LoadedModel, Model, save_model

    m = Model(ctx, gpt2_tensors, max_t=128)
    path = str(tmp_path / "gpt2-int4-g32-a16.llmm")
    save_model(m, path)
    assert _header(path) == ("llm_mojo GPT-2 124M weights", 1, "int4-g32-a16", "int8-ch-a16")
    # head (rows, cols, group) comes first
    with open(path, "rb") as f:
        f.seek(8 + 27 + 8 + 8 + 12 + 8 + 11)
        assert struct.unpack("<3q", f.read(24)) == (50257, 768, 768)
    lm = LoadedModel(ctx, path, max_t=128)
    try:
        prompt = [50256, 464, 3290]
        assert list(lm.generate(prompt, 24)) == list(m.generate(prompt, 24))
        a = torch.zeros(50257, dtype=torch.float32, device="cuda")
        b = torch.zeros(50257, dtype=torch.float32, device="cuda")
        m.forward(prompt, 0, a)
        lm.forward(prompt, 0, b)
        assert torch.equal(a, b)
        # and saving the loaded model writes the same bytes
        path2 = str(tmp_path / "again.llmm")
        lm.save(path2)
        assert open(path, "rb").read() == open(path2, "rb").read()
    finally:
        lm.free()
        m.free()


def test_bf16_model_save_load_and_decode(torch, ctx, gpt2_tensors, tmp_path):
    from llm_mojo_b200.model import FloatModel, LoadedModel, save_model

    m = FloatModel(ctx, gpt2_tensors, "bf16", max_t=64)
    path = str(tmp_path / "gpt2-bf16.llmm")
    save_model(m, path)
    assert _header(path)[2:] == ("bf16", "bf16")
    lm = LoadedModel(ctx, path, kv="bf16", max_t=64)
    try:
        toks = [50256, 11, 262, 286, 13]
        a = torch.zeros((5, 50257), dtype=torch.float32, device="cuda")
        b = torch.zeros((5, 50257), dtype=torch.float32, device="cuda")
        m.forward_all(toks, a)
        lm.forward_all(toks, b)
        assert torch.equal(a, b)
        ids = lm.generate(toks, 8)
        assert list(ids) == list(m.generate(toks, 8))
        # the first generated id is the argmax of the prompt's last logits
        assert ids[0] == int(torch.argmax(b[-1]).item())
    finally:
        lm.free()
        m.free()


def test_gguf_file_load(torch, ctx, gpt2_tensors, tmp_path):
    from gguf_file import write_gpt2_gguf
    from llm_mojo_b200.model import FloatModel, LoadedModel

    path = str(tmp_path / "gpt2-q4_k.gguf")
    write_gpt2_gguf(path, gpt2_tensors)
    assert os.path.getsize(path) > 60_000_000
    lm = LoadedModel(ctx, path, kv="int8", max_t=64, gguf=True)
    ref = FloatModel(ctx, gpt2_tensors, "gguf-q4_k", max_t=64)
    try:
        toks = list(np.random.default_rng(3).integers(0, 50257, 12))
        a = torch.zeros((12, 50257), dtype=torch.float32, device="cuda")
        b = torch.zeros((12, 50257), dtype=torch.float32, device="cuda")
        ref.forward_all(toks, a)
        lm.forward_all(toks, b)
        assert torch.equal(a, b)
        ids = lm.generate(toks, 6)
        assert list(ids) == list(lm.generate(toks, 6))
        assert ids[0] == int(torch.argmax(b[-1]).item())
    finally:
        lm.free()
        ref.free()


def test_gguf_untied_output_head(torch, ctx, gpt2_tensors, tmp_path):
    """An untied output.weight (load_gguf, gpt2t.mojo:733-736): embeddings
    come from token_embd, logits from output.weight, equal to the oracle's
    model built the same way."""
    from float_oracle import oracle_float_forward
    from gguf_file import write_gpt2_gguf
    from llm_mojo_b200._lib import LlmqError
    from llm_mojo_b200.model import LoadedModel

    head = (np.random.default_rng(17).standard_normal((50257, 768)) * 0.02).astype(np.float32)
    path = str(tmp_path / "gpt2-q4_k-untied.gguf")
    write_gpt2_gguf(path, gpt2_tensors, head=head)
    lm = LoadedModel(ctx, path, kv="int8", max_t=64, gguf=True)
    try:
        toks = [50256, 464, 3290, 318, 257]
        got = torch.zeros((5, 50257), dtype=torch.float32, device="cuda")
        lm.forward_all(toks, got)
        want = oracle_float_forward(gpt2_tensors, "gguf-q4_k", toks, 12, head=head)
        assert np.array_equal(got.cpu().numpy().view(np.uint32), want.view(np.uint32))
        with pytest.raises(LlmqError):
            lm.save(str(tmp_path / "untied.llmm"))  # the saved format has one tied matrix
    finally:
        lm.free()


def test_load_rejects_bad_files(ctx, tmp_path):
    from llm_mojo_b200._lib import LlmqError
    from llm_mojo_b200.model import LoadedModel

    bad = tmp_path / "bad.llmm"
    bad.write_bytes(b"not a model at all")
    with pytest.raises(LlmqError):
        LoadedModel(ctx, str(bad))
    with pytest.raises(LlmqError):
        LoadedModel(ctx, str(bad), gguf=True)
