"""Batched greedy decode of independent sequences (config 3's workload):
every sequence's ids must equal its own single-sequence decode on the GPU
(itself bit-exact against the oracle) and the oracle's."""

import numpy as np
import pytest

from oracle import oracle as O

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def torch():
    import torch

    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return torch


@pytest.fixture(scope="module")
def gpu_model(torch, gpt2_tensors):
    from llm_mojo_b200 import build
    from llm_mojo_b200.model import Model
    from llm_mojo_b200.tensor import Context

    build.build()
    ctx = Context(0)
    m = Model(ctx, gpt2_tensors, max_t=256)
    yield m
    m.free()
    ctx.close()


@pytest.mark.parametrize("B,P,steps", [(5, 20, 16), (17, 5, 9), (1, 1, 8)])
def test_batch_matches_single_sequence_decode(gpu_model, oracle_a16, B, P, steps):
    from llm_mojo_b200 import synth
    from llm_mojo_b200.model import Batch

    prompts = synth.uniform_ids(B * P, 3 + B).reshape(B, P)
    bt = Batch(gpu_model, 32, 32)
    try:
        got = bt.generate(prompts, steps)
        again = bt.generate(prompts, steps)  # the captured decode graph, replayed
    finally:
        bt.free()
    assert np.array_equal(got, again)
    for b in range(B):
        want = gpu_model.generate(list(prompts[b]), steps)
        assert list(got[b]) == list(want), f"sequence {b}"
    for b in (0, B - 1):
        assert list(got[b]) == list(oracle_a16.generate(list(prompts[b]), steps)), f"sequence {b} (oracle)"


def test_batch_rejects_oversized_calls(gpu_model):
    from llm_mojo_b200._lib import LlmqError
    from llm_mojo_b200.model import Batch

    bt = Batch(gpu_model, 4, 8)
    try:
        with pytest.raises(LlmqError):
            bt.generate(np.zeros((5, 4), dtype=np.int32), 2)
        with pytest.raises(LlmqError):
            bt.generate(np.zeros((2, 9), dtype=np.int32), 2)
        with pytest.raises(LlmqError):
            bt.generate(np.full((2, 4), 50257, dtype=np.int32), 2)
    finally:
        bt.free()


@pytest.mark.parametrize("B,P,steps", [(40, 12, 10), (1, 3, 6), (33, 7, 5)])
def test_batch_tcgen05_matches_cuda_core_and_single_decode(gpu_model, B, P, steps):
    """The lane-mode tcgen05 GEMM (the layers' BLOCKED int4-g32 rows and the
    int8 head as MMAs with one lane per K-step half) and the dp2a batched
    GEMVs give the same ids, equal to each sequence's single decode; counts
    below, at and past one 32-sequence tile."""
    from llm_mojo_b200 import synth
    from llm_mojo_b200.model import Batch

    prompts = synth.uniform_ids(B * P, 11 + B).reshape(B, P)
    bt = Batch(gpu_model, 48, 16)
    try:
        bt.set_kernel("tcgen05")
        tc = bt.generate(prompts, steps)
        bt.set_kernel("cuda_core")
        cc = bt.generate(prompts, steps)
        bt.set_kernel("auto")
        auto = bt.generate(prompts, steps)
    finally:
        bt.free()
    assert np.array_equal(tc, cc)
    assert np.array_equal(auto, tc)
    for b in sorted({0, B // 2, B - 1}):
        assert list(tc[b]) == list(gpu_model.generate(list(prompts[b]), steps)), f"sequence {b}"


def test_config3_shape_batch_matches_oracle(gpu_model, oracle_a16):
    """Config 3's sequence shape: 32 sequences of a 128-token uniform prompt
    (seed 3, the bench's first 32) and 128 greedy tokens through the default
    kernels: every sequence equals its single decode, three equal the CPU
    oracle's."""
    from llm_mojo_b200 import synth
    from llm_mojo_b200.model import Batch

    prompts = synth.uniform_ids(256 * 128, 3).reshape(256, 128)[:32]
    bt = Batch(gpu_model, 32, 128)
    try:
        got = bt.generate(prompts, 128)
    finally:
        bt.free()
    for b in range(32):
        assert list(got[b]) == list(gpu_model.generate(list(prompts[b]), 128)), f"sequence {b}"
    for b in (0, 15, 31):
        assert list(got[b]) == list(oracle_a16.generate(list(prompts[b]), 128)), f"sequence {b} (oracle)"
