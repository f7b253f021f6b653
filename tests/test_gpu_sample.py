"""Top-k / temperature sampling on the device (gpt2t.mojo:775-834) against
the oracle: the top-k id lists, every drawn id and the Rng state after each
draw are identical; sampled generation of the A16 model gives the oracle
model's ids for the same seed in every decode mode."""

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
def ctx(torch):
    from llm_mojo_b200 import build
    from llm_mojo_b200.tensor import Context

    build.build()
    c = Context(0)
    yield c
    c.close()


def _logits(V, seed, ties=True):
    rng = np.random.default_rng(seed)
    x = (rng.standard_normal(V) * 3).astype(np.float32)
    if ties:
        x[: V // 3] = np.round(x[: V // 3] * 2) / 2  # many equal values
        x[rng.integers(0, V, V // 50 + 1)] = -np.inf
        x[rng.integers(0, V, 3)] = -0.0
    return x


@pytest.mark.parametrize("V,k", [(50257, 1), (50257, 5), (50257, 40), (50257, 1024), (50257, 1025),
                                 (50257, 5000), (50257, 0), (1000, 40), (4096, 4096), (4097, 100),
                                 (200000, 40), (200000, 400), (3, 5)])
def test_top_k_matches_oracle(torch, ctx, V, k):
    from llm_mojo_b200.kernels import top_k

    x = _logits(V, V + k)
    ids = top_k(ctx, torch.from_numpy(x).cuda(), k).cpu().numpy()
    n = min(k, V) if k > 0 else V
    want = np.zeros(n, dtype=np.int32)
    assert O.lib().oq_top_k(O.ptr(x), V, n, O.ptr(want)) == n
    assert np.array_equal(ids, want)


@pytest.mark.parametrize("temperature,k,draws", [(0.8, 40, 64), (1.0, 0, 6), (0.05, 10, 32), (2.0, 1024, 24),
                                                 (1.3, 3000, 8), (0.8, 1, 8), (0.0, 40, 4)])
def test_sample_draws_match_oracle(torch, ctx, temperature, k, draws):
    from llm_mojo_b200.kernels import Rng, sample

    V = 50257
    x = _logits(V, 11 + k)
    dx = torch.from_numpy(x).cuda()
    rng = Rng(1337)
    st = np.array([O.lib().oq_rng_init(1337)], dtype=np.uint64)
    for i in range(draws):
        got = int(sample(ctx, dx, temperature, k, rng).item())
        want = O.lib().oq_sample(O.ptr(x), V, temperature, k, O.ptr(st))
        assert got == want, f"draw {i}"
        assert rng.value() == int(st[0])


def test_sample_all_equal_logits(torch, ctx):
    """All weights 1: the walk picks by position in id order."""
    from llm_mojo_b200.kernels import Rng, sample

    V = 50257
    x = np.zeros(V, dtype=np.float32)
    dx = torch.from_numpy(x).cuda()
    rng = Rng(7)
    st = np.array([O.lib().oq_rng_init(7)], dtype=np.uint64)
    for k in (40, 0):
        for _ in range(8):
            assert int(sample(ctx, dx, 0.8, k, rng).item()) == O.lib().oq_sample(O.ptr(x), V, 0.8, k, O.ptr(st))


@pytest.fixture(scope="module")
def models(torch, ctx, gpt2_tensors, oracle_a16):
    from llm_mojo_b200.model import Model

    g = Model(ctx, gpt2_tensors, max_t=256)
    yield g, oracle_a16
    g.free()


@pytest.mark.parametrize("mode", ["persistent", "graph", "eager"])
def test_generate_sampled_matches_oracle(models, mode):
    g, o = models
    g.set_mode(mode)
    try:
        prompt = [50256, 464, 3290, 318]
        got = g.generate_sampled(prompt, 24, 0.8, 40, 1337)
        want = o.generate_sampled(prompt, 24, 0.8, 40, 1337)
        assert list(got) == list(want)
        # one-token prompt: the decode path from the first step
        got = g.generate_sampled([50256], 12, 1.1, 200, 5)
        assert list(got) == list(o.generate_sampled([50256], 12, 1.1, 200, 5))
    finally:
        g.set_mode("persistent")


def test_generate_sampled_all_candidates_and_state(models):
    g, o = models
    st_g = np.array([O.lib().oq_rng_init(99)], dtype=np.uint64)
    got = g.generate_sampled([50256, 11], 4, 1.0, 0, state=st_g)
    st_o = np.array([O.lib().oq_rng_init(99)], dtype=np.uint64)
    p = np.array([50256, 11], dtype=np.int32)
    want = np.zeros(4, dtype=np.int32)
    O.lib().oq_generate_sampled(o.h, O.ptr(p), 2, 4, 1.0, 0, O.ptr(st_o), O.ptr(want))
    assert list(got) == list(want)
    assert int(st_g[0]) == int(st_o[0])


def test_generate_sampled_zero_temperature_is_greedy(models):
    g, _ = models
    assert list(g.generate_sampled([50256], 10, 0.0, 40, 1)) == list(g.generate([50256], 10))


def test_float_model_sampled_decode(torch, ctx, gpt2_tensors):
    """The float formats' generation draws on its own logits: the ids equal a
    host loop of forward + the oracle's sample on the same logits."""
    from llm_mojo_b200.model import FloatModel

    m = FloatModel(ctx, gpt2_tensors, "bf16", max_t=64)
    try:
        prompt = [50256, 40, 588]
        ids = m.generate_sampled(prompt, 6, 0.9, 50, 21)
        st = np.array([O.lib().oq_rng_init(21)], dtype=np.uint64)
        logits = torch.zeros(50257, dtype=torch.float32, device="cuda")
        m.forward(prompt, 0, logits)
        pos = len(prompt)
        want = []
        for i in range(6):
            x = logits.cpu().numpy()
            nxt = O.lib().oq_sample(O.ptr(x), 50257, 0.9, 50, O.ptr(st))
            want.append(nxt)
            if i < 5:
                m.forward([nxt], pos, logits)
                pos += 1
        assert list(ids) == want
    finally:
        m.free()
