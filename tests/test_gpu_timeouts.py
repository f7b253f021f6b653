"""Bounded device-side waits, made to run out on purpose (the failure
detection of this path, tested without a GPU fault): with a wait limit of a
few cycles the persistent and cluster decode kernels and the row GEMV give up
at their first wait for a copy or an exchange, record an error, wait for
their own copies in flight (a separate, long bound) and return; the call that
synchronises reports LLMQ_ERR_TIMEOUT. The context stays usable: with the
limit restored the same calls give the oracle's results."""

import ctypes as C

import numpy as np
import pytest

from oracle import oracle as O

pytestmark = pytest.mark.gpu

LLMQ_ERR_TIMEOUT = 4


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


@pytest.mark.parametrize("mode", ["persistent", "cluster"])
def test_decode_wait_timeout_is_reported_and_recoverable(ctx, gpt2_tensors, mode):
    from llm_mojo_b200._lib import lib
    from llm_mojo_b200.model import Model

    m = Model(ctx, gpt2_tensors, n_layer=2, max_t=64)
    om = O.Model(gpt2_tensors, n_layer=2, max_t=64)
    try:
        want = list(om.generate([50256], 6))
        m.set_mode(mode)
        prompt = np.array([50256], dtype=np.int32)
        out = np.zeros(6, dtype=np.int32)
        assert lib().llmq_set_wait_limit(ctx.h, 1) == 0
        st = lib().llmq_generate(ctx.h, m.h, prompt.ctypes.data_as(C.c_void_p), 1, 6, out.ctypes.data_as(C.c_void_p))
        assert st == LLMQ_ERR_TIMEOUT, lib().llmq_last_error(ctx.h)
        assert lib().llmq_set_wait_limit(ctx.h, 0) == 0
        assert list(m.generate([50256], 6)) == want
    finally:
        lib().llmq_set_wait_limit(ctx.h, 0)
        m.free()
        om.close()


def test_row_gemv_wait_timeout_is_reported_and_recoverable(torch, ctx):
    from llm_mojo_b200 import gguf_blocks as G
    from llm_mojo_b200._lib import lib
    from llm_mojo_b200.tensor import GGUFMatrix

    IN, OUT = 768, 2304
    rng = np.random.default_rng(3)
    w = (rng.standard_normal((OUT, IN)) * 0.02).astype(np.float32)
    blocks = G.quantize(w, G.Q8_0)
    gw = GGUFMatrix(ctx, G.Q8_0, blocks, OUT, IN)
    x = rng.standard_normal(IN).astype(np.float32)
    xd = torch.from_numpy(x).cuda()
    out = torch.zeros(OUT, dtype=torch.float32, device="cuda")
    torch.cuda.synchronize()
    try:
        assert lib().llmq_set_wait_limit(ctx.h, 1) == 0
        assert lib().llmq_linear(ctx.h, gw.h, C.c_void_p(xd.data_ptr()), None, C.c_void_p(out.data_ptr()), 1, IN,
                                 OUT, 0) == 0
        assert lib().llmq_sync(ctx.h) == LLMQ_ERR_TIMEOUT
        assert lib().llmq_set_wait_limit(ctx.h, 0) == 0
        assert lib().llmq_linear(ctx.h, gw.h, C.c_void_p(xd.data_ptr()), None, C.c_void_p(out.data_ptr()), 1, IN,
                                 OUT, 0) == 0
        assert lib().llmq_sync(ctx.h) == 0
        want = np.array([O.lib().oq_gguf_dot_row(G.Q8_0, O.ptr(np.ascontiguousarray(blocks[o])), IN, O.ptr(x))
                         for o in range(OUT)], dtype=np.float32)
        assert np.array_equal(out.cpu().numpy().view(np.uint32), want.view(np.uint32))
    finally:
        lib().llmq_set_wait_limit(ctx.h, 0)
        gw.free()
