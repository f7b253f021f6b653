"""llmq_head_argmax_noalloc against llmq_head_argmax, through the C ABI.

The no-allocation entry point runs the same head GEMV + argmax kernel with
its scratch in a fixed device array, so its logits must equal the existing
entry point's bit for bit (the tolerance of the head tests: zero) and its
argmax must be the same index. Two calls in a row check that the state the
array carries (the CTA ticket and the id slot) is cleared between calls.
The cases take the three head GEMV kernels: the per-warp cp.async ring
(int8-ch, 50257 rows), the split-K tiles (int4-g32, 2304 rows) and the
whole-row kernel of the other formats from 8192 rows (int4-g128). The first
case is also checked against the CPU oracle. This file is collected last so
that it also runs after every other test.
"""

import ctypes as C

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def torch():
    import torch

    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return torch


def _p(t):
    return C.c_void_p(t.data_ptr())


@pytest.mark.parametrize("fmt,rows", [("int8-ch-a16", 50257), ("int4-g32-a16", 2304), ("int4-g128-a16", 8192)])
def test_head_argmax_noalloc_matches_head_argmax(torch, fmt, rows):
    from llm_mojo_b200 import build
    from llm_mojo_b200._lib import check, lib
    from llm_mojo_b200.tensor import Context, QuantMatrix, parse_dtype

    build.build()
    ctx = Context(0)
    bits, group, sym, a16 = parse_dtype(fmt)
    rng = np.random.default_rng(rows)
    src = rng.normal(0, 0.02, (rows, 768)).astype(np.float32)
    w = QuantMatrix.from_f32(ctx, src, bits, group, sym, a16, False)
    hs = [torch.from_numpy(rng.standard_normal(768).astype(np.float32)).cuda() for _ in range(2)]
    want_l = [torch.zeros(rows, dtype=torch.float32, device="cuda") for _ in range(2)]
    want_a = [torch.full((1,), -1, dtype=torch.int32, device="cuda") for _ in range(2)]
    got_l = [torch.zeros(rows, dtype=torch.float32, device="cuda") for _ in range(2)]
    got_a = [torch.full((1,), -1, dtype=torch.int32, device="cuda") for _ in range(2)]
    torch.cuda.synchronize()
    for i in range(2):
        check(lib().llmq_head_argmax(ctx.h, w.h, _p(hs[i]), _p(want_l[i]), _p(want_a[i])), ctx.h)
    ctx.sync()
    # two calls in a row on the context's stream, no synchronisation between
    for i in range(2):
        check(lib().llmq_head_argmax_noalloc(ctx.h, w.h, _p(hs[i]), _p(got_l[i]), _p(got_a[i])), ctx.h)
    ctx.sync()
    for i in range(2):
        want = want_l[i].cpu().numpy()
        got = got_l[i].cpu().numpy()
        assert np.array_equal(got.view(np.uint32), want.view(np.uint32))
        assert int(got_a[i].item()) == int(want_a[i].item()) == int(np.argmax(want))
    if fmt == "int8-ch-a16":
        from oracle import oracle as O

        ow = O.QuantMatrix(src, bits, group, sym, a16, False)
        for i in range(2):
            ref = O.matmul_rows_a16(hs[i].cpu().numpy()[None, :], ow, None)[0]
            assert np.array_equal(got_l[i].cpu().numpy().view(np.uint32), ref.view(np.uint32))
            assert int(got_a[i].item()) == int(O.lib().oq_argmax(O.ptr(ref), rows))
    w.free()
    ctx.close()
