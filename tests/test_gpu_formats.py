"""One-token matmuls of every config-1 sweep format against the CPU oracle,
bit for bit: affine W4A32/W8A32 (QuantMatrix.dot_row), the six GGUF block
types and GGUF F16/F32 rows (GGUFMatrix.dot_row), dense f32/f16/bf16 layer
matrices (gemv with the reference's 4 parts) and heads (lm_head), and the
integer GGUF heads (Q8_0, Q6_K)."""

import numpy as np
import pytest

from llm_mojo_b200 import gguf_blocks as G
from oracle import oracle as O

pytestmark = pytest.mark.gpu

SHAPES = [(768, 2304), (3072, 768), (768, 70)]  # (IN, OUT)


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


def bits(a):
    return np.ascontiguousarray(a, dtype=np.float32).view(np.uint32)


@pytest.mark.parametrize("t", [G.Q4_0, G.Q4_1, G.Q8_0, G.Q4_K, G.Q5_K, G.Q6_K, G.F16, G.F32])
@pytest.mark.parametrize("IN,OUT", SHAPES)
def test_gguf_dot_rows(torch, ctx, t, IN, OUT):
    from llm_mojo_b200 import kernels
    from llm_mojo_b200.tensor import GGUFMatrix

    if IN % G.BLOCK_SIZE[t]:
        pytest.skip("shape not a multiple of the block")
    rng = np.random.default_rng(IN + OUT + t)
    w = (rng.standard_normal((OUT, IN)) * 0.02).astype(np.float32)
    blocks = G.quantize(w, t)
    gw = GGUFMatrix(ctx, t, blocks, OUT, IN)
    x = rng.standard_normal(IN).astype(np.float32)
    b = rng.standard_normal(OUT).astype(np.float32)
    out = torch.zeros(OUT, dtype=torch.float32, device="cuda")
    kernels.linear(ctx, out, dev(torch, x), gw, dev(torch, b), 1, IN, OUT, gelu=True)
    want = np.array([O.oq_gelu_np(np.float32(O.lib().oq_gguf_dot_row(t, O.ptr(np.ascontiguousarray(blocks[o])), IN, O.ptr(x))
                                   ) + b[o]) for o in range(OUT)], dtype=np.float32)
    assert np.array_equal(bits(out.cpu().numpy()), bits(want))
    gw.free()


@pytest.mark.parametrize("fmt", ["int4-g32", "int4-g128-sym", "int4-ch", "int8-ch", "int8-g64"])
@pytest.mark.parametrize("IN,OUT", SHAPES)
def test_affine_float_rows(torch, ctx, fmt, IN, OUT):
    from llm_mojo_b200 import kernels
    from llm_mojo_b200.tensor import QuantMatrix, parse_dtype

    bits_, group, sym, a16 = parse_dtype(fmt)
    rng = np.random.default_rng(IN * 3 + OUT)
    src = (rng.standard_normal((IN, OUT)) * 0.02).astype(np.float32)
    ow = O.QuantMatrix(src, bits_, group, sym, False, True)
    gw = QuantMatrix.from_f32(ctx, src, bits_, group, sym, False, True)
    x = rng.standard_normal(IN).astype(np.float32)
    resid = rng.standard_normal(OUT).astype(np.float32)
    out = dev(torch, resid)
    kernels.linear(ctx, out, dev(torch, x), gw, None, 1, IN, OUT, resid=True)
    want = np.array([O.lib().oq_dot_row(O.C.byref(ow.q), o, O.ptr(x)) + resid[o] for o in range(OUT)],
                    dtype=np.float32)
    assert np.array_equal(bits(out.cpu().numpy()), bits(want))
    gw.free()


@pytest.mark.parametrize("fmt", ["int4-g32", "int8-g64", "int4-g128", "int8-ch"])
def test_affine_float_head_rows(torch, ctx, fmt):
    """The one-token W4A32 / W8A32 head shape (16 rows per CTA of the grouped
    kernel from 8192 rows; the per-channel kernel for int8-ch): 12,000 rows of
    768, every row against the oracle's dot_row, bit for bit."""
    from llm_mojo_b200 import kernels
    from llm_mojo_b200.tensor import QuantMatrix, parse_dtype

    bits_, group, sym, _ = parse_dtype(fmt)
    V, Cn = 12000, 768
    rng = np.random.default_rng(V + bits_)
    w = (rng.standard_normal((V, Cn)) * 0.02).astype(np.float32)
    ow = O.QuantMatrix(w, bits_, group, sym, False, False)
    gw = QuantMatrix.from_f32(ctx, w, bits_, group, sym, False, False)
    h = rng.standard_normal(Cn).astype(np.float32)
    logits = torch.zeros((1, V), dtype=torch.float32, device="cuda")
    try:
        kernels.head(ctx, logits, dev(torch, h), gw, 1, V, Cn)
        want = np.array([O.lib().oq_dot_row(O.C.byref(ow.q), o, O.ptr(h)) for o in range(V)], dtype=np.float32)
        assert np.array_equal(bits(logits.cpu().numpy()[0]), bits(want))
    finally:
        gw.free()


@pytest.mark.parametrize("dt", ["f32", "f16", "bf16"])
@pytest.mark.parametrize("IN,OUT", SHAPES)
def test_dense_gemv_parts(torch, ctx, dt, IN, OUT):
    check_dense_gemv(torch, ctx, dt, IN, OUT, 4)


@pytest.mark.parametrize("dt", ["f32", "f16", "bf16"])
@pytest.mark.parametrize("IN,OUT,parts", [(770, 72, 4), (3072, 2304, 3), (768, 768, 1), (3072, 768, 1), (100, 40, 8)])
def test_dense_gemv_strips(torch, ctx, dt, IN, OUT, parts):
    """The staged strips (32 columns x one part per CTA): a ragged last strip
    (72 and 40 columns), parts that do not divide the inputs (770 / 4,
    100 / 8), other part counts, and a part too long to stage (3072 rows of
    f32 in one part), which keeps the unstaged kernel. Same bits as the
    oracle."""
    from llm_mojo_b200 import kernels

    kernels.set_dense_parts(ctx, parts)
    try:
        check_dense_gemv(torch, ctx, dt, IN, OUT, parts)
    finally:
        kernels.set_dense_parts(ctx, 4)


def check_dense_gemv(torch, ctx, dt, IN, OUT, parts):
    from llm_mojo_b200 import kernels
    from llm_mojo_b200.tensor import DenseMatrix

    rng = np.random.default_rng(IN + 7 * OUT)
    src = (rng.standard_normal((IN, OUT)) * 0.02).astype(np.float32)
    gw = DenseMatrix(ctx, dt, src)
    x = rng.standard_normal(IN).astype(np.float32)
    b = rng.standard_normal(OUT).astype(np.float32)
    out = torch.zeros(OUT, dtype=torch.float32, device="cuda")
    kernels.linear(ctx, out, dev(torch, x), gw, dev(torch, b), 1, IN, OUT, gelu=True)
    want = np.zeros(OUT, dtype=np.float32)
    O.lib().oq_dense_gemv({"f32": 0, "f16": 1, "bf16": 2}[dt], O.ptr(gw.data), O.ptr(x), O.ptr(b), O.ptr(want), IN,
                          OUT, parts, 0, 1)
    assert np.array_equal(bits(out.cpu().numpy()), bits(want))
    gw.free()


@pytest.mark.parametrize("dt", ["f32", "f16", "bf16"])
def test_dense_head_rows(torch, ctx, dt, gpt2_tensors):
    from llm_mojo_b200 import kernels
    from llm_mojo_b200.tensor import DenseMatrix

    wte = gpt2_tensors["wte.weight"]
    gw = DenseMatrix(ctx, dt, wte)
    h = np.random.default_rng(3).standard_normal((2, 768)).astype(np.float32)
    logits = torch.zeros((2, 50257), dtype=torch.float32, device="cuda")
    kernels.head(ctx, logits, dev(torch, h), gw, 2, 50257, 768)
    got = logits.cpu().numpy()
    dti = {"f32": 0, "f16": 1, "bf16": 2}[dt]
    for t in range(2):
        rows = np.random.default_rng(t).choice(50257, 300, replace=False)
        want = np.array([O.lib().oq_dense_dot_row(dti, O.ptr(gw.data), int(v), 768, O.ptr(h[t])) for v in rows],
                        dtype=np.float32)
        assert np.array_equal(bits(got[t][rows]), bits(want))
    gw.free()


@pytest.mark.parametrize("t", [G.Q8_0, G.Q6_K])
def test_gguf_integer_head(torch, ctx, t):
    """gguf_int_head.mojo: one token and several tokens give identical logits,
    and both equal the oracle's."""
    from llm_mojo_b200 import kernels
    from llm_mojo_b200.tensor import GGUFMatrix

    V, Cn = 4096, 768
    rng = np.random.default_rng(t)
    w = (rng.standard_normal((V, Cn)) * 0.02).astype(np.float32)
    blocks = G.quantize(w, t)
    gw = GGUFMatrix(ctx, t, blocks, V, Cn)
    h = rng.uniform(-3, 3, (5, Cn)).astype(np.float32)
    h[1] = (rng.uniform(0.9, 1.0, Cn) * np.where(np.arange(Cn) % 2 == 0, 1, -1)).astype(np.float32)
    many = torch.zeros((5, V), dtype=torch.float32, device="cuda")
    kernels.head(ctx, many, dev(torch, h), gw, 5, V, Cn)
    for r in range(5):
        one = torch.zeros((1, V), dtype=torch.float32, device="cuda")
        kernels.head(ctx, one, dev(torch, h[r]), gw, 1, V, Cn)
        assert np.array_equal(bits(one.cpu().numpy()[0]), bits(many.cpu().numpy()[r]))
        want = np.zeros(V, dtype=np.float32)
        O.lib().oq_gguf_head_i16(t, O.ptr(np.ascontiguousarray(blocks)), V, Cn, O.ptr(h[r]), O.ptr(want))
        assert np.array_equal(bits(many.cpu().numpy()[r]), bits(want))
    gw.free()
