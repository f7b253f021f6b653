"""IntAttnKV (int_attention.mojo) on the GPU against the CPU oracle.

Everything up to the final float flush is integer fixed point, and the float
flushes follow the reference's order, so the key/value codes, their Q24
scales and the attention outputs must match the oracle bit for bit. The
context grid is the one of the reference's tests/int_attention_check.mojo.
"""

import ctypes as C

import numpy as np
import pytest

from oracle import oracle as O

pytestmark = pytest.mark.gpu

NH, HS, CN, MAXT = 12, 64, 768, 1024


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
    return Context(0)


def dev(torch, a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def _arr(ptr, ctype, n):
    return np.ctypeslib.as_array(C.cast(ptr, C.POINTER(ctype)), shape=(n,)).copy()


@pytest.mark.parametrize("npos0,T", [(0, 1), (0, 5), (15, 1), (16, 1), (17, 1), (99, 1), (255, 2), (256, 1),
                                     (511, 3), (1000, 3), (1023, 1)])
def test_intattn_attention_bit_exact(torch, ctx, npos0, T):
    from llm_mojo_b200.kernels import KVCache

    rng = np.random.default_rng(npos0 * 10 + T + 7)
    n = npos0 + T
    qkv_all = (rng.standard_normal((n, 3 * CN)) * 2).astype(np.float32)
    kv = KVCache(ctx, "intattn", 1, MAXT, NH, HS)
    oc = O.lib().oq_intkv_new(1, MAXT, NH, HS)
    try:
        if npos0:
            kv.store(0, 0, npos0, dev(torch, qkv_all[:npos0]))
        for p in range(n):
            row = qkv_all[p]
            O.lib().oq_intkv_store(oc, 0, p, O.ptr(np.ascontiguousarray(row[CN:2 * CN])),
                                   O.ptr(np.ascontiguousarray(row[2 * CN:])))
        q = np.ascontiguousarray(qkv_all[npos0:])
        kv.store(0, npos0, T, dev(torch, q))
        out = torch.zeros((T, CN), dtype=torch.float32, device="cuda")
        kv.attend(out, dev(torch, q), 0, T, npos0)
        want = np.zeros((T, CN), dtype=np.float32)
        for t in range(T):
            for h in range(NH):
                O.lib().oq_intkv_attend_one(oc, O.ptr(want), O.ptr(q), 0, t, h, npos0)
        got = out.cpu().numpy()
        assert np.array_equal(got.view(np.uint32), want.view(np.uint32)), f"max diff {np.abs(got - want).max()}"
        k, v, kq, vq = kv.read()
        nb = MAXT * NH * HS
        assert np.array_equal(k, _arr(O.lib().oq_intkv_k(oc), C.c_int8, nb))
        assert np.array_equal(v, _arr(O.lib().oq_intkv_v(oc), C.c_int8, nb))
        assert np.array_equal(kq.view(np.int32), _arr(O.lib().oq_intkv_kq(oc), C.c_int32, MAXT * NH))
        assert np.array_equal(vq.view(np.int32), _arr(O.lib().oq_intkv_vq(oc), C.c_int32, MAXT * NH))
    finally:
        O.lib().oq_intkv_free(oc)
        kv.free()


def test_intattn_zero_values_give_zero_output(torch, ctx):
    """vmax == 0 (every value zero): the reference writes zeros."""
    from llm_mojo_b200.kernels import KVCache

    rng = np.random.default_rng(5)
    qkv = rng.standard_normal((4, 3 * CN)).astype(np.float32)
    qkv[:, 2 * CN:] = 0.0
    kv = KVCache(ctx, "intattn", 1, MAXT, NH, HS)
    try:
        kv.store(0, 0, 4, dev(torch, qkv))
        out = torch.full((4, CN), 7.0, dtype=torch.float32, device="cuda")
        kv.attend(out, dev(torch, qkv), 0, 4, 0)
        assert not out.cpu().numpy().any()
    finally:
        kv.free()


def test_intattn_rejects_unaligned_context(ctx):
    from llm_mojo_b200._lib import LlmqError
    from llm_mojo_b200.kernels import KVCache

    with pytest.raises(LlmqError):
        KVCache(ctx, "intattn", 1, 1000, NH, HS)


@pytest.fixture(scope="module")
def intattn_models(torch, ctx, gpt2_tensors):
    from llm_mojo_b200.model import Model

    g = Model(ctx, gpt2_tensors, kv="intattn")
    o = O.Model(gpt2_tensors, kv="intattn")
    yield g, o
    g.free()
    o.close()


def test_intattn_generate_100_ids_match_oracle(intattn_models):
    """Config 0 with --attention int: 100 greedy ids identical."""
    g, o = intattn_models
    assert list(g.generate([50256], 100)) == list(o.generate([50256], 100))


def test_intattn_prompt_logits_bit_exact(torch, intattn_models, golden):
    g, o = intattn_models
    prompt = golden["prompt24"]
    logits = torch.zeros(50257, dtype=torch.float32, device="cuda")
    g.forward(prompt, 0, logits)
    want = o.forward(prompt, 0)
    assert np.array_equal(logits.cpu().numpy().view(np.uint32), want.view(np.uint32))
    assert list(g.generate(prompt, 20)) == list(o.generate(prompt, 20))
