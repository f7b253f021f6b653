"""The oracle's sampling (Rng, top_k, sample; gpt2t.mojo:775-834) against a
line-by-line Python transcription of the reference's Mojo code: the list
insertion of top_k with its append-then-pop, float32 weights and the
float32 sum and subtraction walk. The weights use the same exp (lm_expf)."""

import numpy as np
import pytest

from oracle import oracle as O

M64 = (1 << 64) - 1


class PyRng:
    def __init__(self, seed):
        self.state = (seed * 0x9E3779B97F4A7C15 + 1) & M64

    def uniform(self):
        s = self.state
        s ^= s >> 12
        s ^= (s << 25) & M64
        s ^= s >> 27
        self.state = s
        r = ((s * 0x2545F4914F6CDD1D) & M64) >> 40
        return np.float32(r) / np.float32(1 << 24)


def py_top_k(logits, k):
    ids = []
    for v in range(len(logits)):
        lv = logits[v]
        if len(ids) == k and lv <= logits[ids[k - 1]]:
            continue
        pos = len(ids)
        ids.append(v)
        while pos > 0 and logits[ids[pos - 1]] < lv:
            ids[pos] = ids[pos - 1]
            pos -= 1
        ids[pos] = v
        if len(ids) > k:
            ids.pop()
    return ids


def py_sample(logits, temperature, k, rng):
    f32 = np.float32
    if temperature <= 0:
        return int(np.argmax(logits))
    cand = py_top_k(logits, k if k > 0 else len(logits))
    mx = logits[cand[0]]
    probs, total = [], f32(0)
    for i in cand:
        p = f32(O.lib().lm_expf(float(f32(f32(logits[i] - mx) / f32(temperature)))))
        probs.append(p)
        total = f32(total + p)
    r = f32(rng.uniform() * total)
    for i in range(len(cand)):
        r = f32(r - probs[i])
        if r <= 0:
            return cand[i]
    return cand[-1]


def test_rng_sequence_matches_transcription():
    for seed in (0, 1, 1337, -5, 2**62):
        st = np.array([O.lib().oq_rng_init(seed)], dtype=np.uint64)
        py = PyRng(seed)
        assert int(st[0]) == py.state
        for _ in range(50):
            assert O.lib().oq_rng_uniform(O.ptr(st)) == py.uniform()
            assert int(st[0]) == py.state


@pytest.mark.parametrize("V,k", [(1, 1), (7, 3), (300, 1), (300, 40), (300, 300), (300, 500), (1000, 999)])
def test_top_k_matches_insertion(V, k):
    rng = np.random.default_rng(V * 7 + k)
    logits = (np.round(rng.standard_normal(V) * 3) / 2).astype(np.float32)  # many ties
    logits[rng.integers(0, V, V // 10 + 1)] = -np.inf
    ids = np.zeros(min(k, V), dtype=np.int32)
    n = O.lib().oq_top_k(O.ptr(logits), V, k, O.ptr(ids))
    assert n == min(k, V)
    assert list(ids) == py_top_k(list(logits), k)


@pytest.mark.parametrize("temperature,k", [(0.8, 40), (1.0, 0), (0.05, 10), (2.5, 300), (0.0, 40), (-1.0, 5)])
def test_sample_matches_transcription(temperature, k):
    rng = np.random.default_rng(abs(int(temperature * 100)) + k)
    V = 400
    logits = (rng.standard_normal(V) * 4).astype(np.float32)
    logits[:20] = logits[20:40]  # ties
    st = np.array([O.lib().oq_rng_init(1337)], dtype=np.uint64)
    py = PyRng(1337)
    lv = list(logits)
    for _ in range(40):
        got = O.lib().oq_sample(O.ptr(logits), V, temperature, k, O.ptr(st))
        assert got == py_sample(lv, temperature, k, py)
        assert int(st[0]) == py.state
