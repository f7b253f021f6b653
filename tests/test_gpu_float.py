"""Float-activation several-token paths (the perplexity harness's formats)
against the CPU oracle, bit for bit: the dense matmul tile (f32 / bf16), the
dense head for every position, GGUF and affine W4A32 / W8A32 rows for
several tokens, the dense KV caches, a whole float model's forward_all, and
the scores."""

import ctypes as C

import numpy as np
import pytest

from float_oracle import DT, oracle_float_forward
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


def dev(torch, a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def same(got, want):
    bad = np.argwhere(got.view(np.uint32) != want.view(np.uint32))
    assert bad.size == 0, f"{len(bad)} differ, first {bad[:3].tolist()}, max diff {np.abs(got - want).max()}"


@pytest.mark.parametrize("dt", ["f32", "bf16"])
@pytest.mark.parametrize("T,IN,OUT,epi", [(5, 768, 2304, "gelu"), (70, 3072, 768, "resid"), (130, 768, 96, "plain")])
def test_dense_mm_bit_exact(torch, ctx, dt, T, IN, OUT, epi):
    from llm_mojo_b200 import kernels
    from llm_mojo_b200.tensor import DenseMatrix

    rng = np.random.default_rng(T + OUT)
    w = DenseMatrix(ctx, dt, (rng.standard_normal((IN, OUT)) * 0.02).astype(np.float32))
    x = rng.standard_normal((T, IN)).astype(np.float32)
    b = rng.standard_normal(OUT).astype(np.float32)
    resid = rng.standard_normal((T, OUT)).astype(np.float32) if epi == "resid" else None
    want = resid.copy() if resid is not None else np.zeros((T, OUT), np.float32)
    O.lib().oq_dense_mm(DT[dt], O.ptr(w.data), O.ptr(x), O.ptr(b), O.ptr(want), T, IN, OUT, int(epi == "resid"),
                        int(epi == "gelu"))
    out = dev(torch, resid if resid is not None else np.zeros((T, OUT), np.float32))
    kernels.linear(ctx, out, dev(torch, x), w, dev(torch, b), T, IN, OUT, gelu=epi == "gelu", resid=epi == "resid")
    same(out.cpu().numpy(), want)
    w.free()


@pytest.mark.parametrize("dt", ["f32", "bf16"])
def test_dense_head_rows_bit_exact(torch, ctx, dt):
    from llm_mojo_b200 import kernels
    from llm_mojo_b200.tensor import DenseMatrix

    rng = np.random.default_rng(4)
    T, V, Cn = 37, 1000, 768
    w = DenseMatrix(ctx, dt, (rng.standard_normal((V, Cn)) * 0.02).astype(np.float32))
    h = rng.standard_normal((T, Cn)).astype(np.float32)
    want = np.zeros((T, V), np.float32)
    O.lib().oq_dense_head_rows(DT[dt], O.ptr(w.data), O.ptr(h), O.ptr(want), T, V, Cn)
    logits = torch.zeros((T, V), dtype=torch.float32, device="cuda")
    kernels.head(ctx, logits, dev(torch, h), w, T, V, Cn)
    same(logits.cpu().numpy(), want)
    w.free()


@pytest.mark.parametrize("t", ["Q4_K", "Q6_K", "Q8_0", "Q4_0", "Q5_K"])
@pytest.mark.parametrize("T,OUT", [(9, 70), (33, 2304)])
def test_gguf_rows_several_tokens_bit_exact(torch, ctx, t, T, OUT):
    from llm_mojo_b200 import gguf_blocks as G
    from llm_mojo_b200 import kernels
    from llm_mojo_b200.tensor import GGUFMatrix

    typ = getattr(G, t)
    IN = 768
    rng = np.random.default_rng(OUT + T)
    blocks = G.quantize((rng.standard_normal((OUT, IN)) * 0.02).astype(np.float32), typ)
    w = GGUFMatrix(ctx, typ, blocks, OUT, IN)
    x = rng.standard_normal((T, IN)).astype(np.float32)
    b = rng.standard_normal(OUT).astype(np.float32)
    want = np.zeros((T, OUT), np.float32)
    O.lib().oq_gguf_matmul_rows(typ, O.ptr(w.blocks), G.row_bytes(typ, IN), O.ptr(x), O.ptr(b), O.ptr(want), T, IN,
                                OUT, 0, 1)
    out = torch.zeros((T, OUT), dtype=torch.float32, device="cuda")
    kernels.linear(ctx, out, dev(torch, x), w, dev(torch, b), T, IN, OUT, gelu=True)
    same(out.cpu().numpy(), want)
    w.free()


@pytest.mark.parametrize("dt", ["f32", "bf16"])
@pytest.mark.parametrize("npos0,T", [(0, 1), (0, 20), (100, 7), (1000, 24)])
def test_dense_kv_attention_bit_exact(torch, ctx, dt, npos0, T):
    from llm_mojo_b200.kernels import KVCache

    NH, HS, CN, MAXT = 12, 64, 768, 1024
    rng = np.random.default_rng(npos0 + T)
    n = npos0 + T
    qkv_all = (rng.standard_normal((n, 3 * CN)) * 2).astype(np.float32)
    kv = KVCache(ctx, dt, 1, MAXT, NH, HS)
    try:
        kv.store(0, 0, n, dev(torch, qkv_all))
        q = np.ascontiguousarray(qkv_all[npos0:])
        out = torch.zeros((T, CN), dtype=torch.float32, device="cuda")
        kv.attend(out, dev(torch, q), 0, T, npos0)
        k, v, _, _ = kv.read()
        # the stored values are the cache type's (bfloat16: round to nearest even)
        kk = k.reshape(MAXT, CN)[:n]
        if dt == "f32":
            assert np.array_equal(kk, qkv_all[:, CN:2 * CN])
        want = np.zeros((T, CN), np.float32)
        for t in range(T):
            for h in range(NH):
                O.lib().oq_dkv_attend_one(DT[dt], O.ptr(np.ascontiguousarray(k)), O.ptr(np.ascontiguousarray(v)), NH,
                                          HS, O.ptr(want), O.ptr(q), t, h, npos0)
        same(out.cpu().numpy(), want)
    finally:
        kv.free()


@pytest.mark.parametrize("fmt", ["int4-g32", "int4-g128-sym", "int4-ch", "int8-ch", "int8-g64"])
@pytest.mark.parametrize("T,OUT,epi", [(9, 70, "gelu"), (33, 2304, "resid"), (2, 768, "plain")])
def test_affine_rows_several_tokens_bit_exact(torch, ctx, fmt, T, OUT, epi):
    """matmul_rows for T > 1 of the W4A32 / W8A32 formats (kernels.mojo:
    325-397): dequantized rows through the mm_tile chain, the OUT % 32
    leftover rows through rows_dot; the same bits as the oracle."""
    from llm_mojo_b200 import kernels
    from llm_mojo_b200.tensor import QuantMatrix, parse_dtype

    bits_, group, sym, _ = parse_dtype(fmt)
    IN = 768
    rng = np.random.default_rng(OUT * 5 + T)
    src = (rng.standard_normal((IN, OUT)) * 0.02).astype(np.float32)  # [IN, OUT]
    ow = O.QuantMatrix(src, bits_, group, sym, False, True)
    gw = QuantMatrix.from_f32(ctx, src, bits_, group, sym, False, True)
    x = rng.standard_normal((T, IN)).astype(np.float32)
    b = rng.standard_normal(OUT).astype(np.float32)
    resid = rng.standard_normal((T, OUT)).astype(np.float32)
    want = resid.copy() if epi == "resid" else np.zeros((T, OUT), np.float32)
    O.lib().oq_affine_matmul_rows(C.byref(ow.q), O.ptr(x), O.ptr(b), O.ptr(want), T, IN, OUT, int(epi == "resid"),
                                  int(epi == "gelu"))
    out = dev(torch, resid) if epi == "resid" else torch.zeros((T, OUT), dtype=torch.float32, device="cuda")
    try:
        kernels.linear(ctx, out, dev(torch, x), gw, dev(torch, b), T, IN, OUT, resid=epi == "resid",
                       gelu=epi == "gelu")
        same(out.cpu().numpy(), want)
    finally:
        gw.free()


@pytest.mark.parametrize("fmt", ["int8-ch", "int4-g32"])
def test_affine_head_several_tokens_bit_exact(torch, ctx, fmt):
    """head (kernels.mojo:677-689) of an OUT_MAJOR affine matrix for T > 1:
    matmul_rows with no bias (4113 rows: 17 leftover rows on rows_dot), not
    T one-token dots; T = 1 stays the dot_row path."""
    from llm_mojo_b200 import kernels
    from llm_mojo_b200.tensor import QuantMatrix, parse_dtype

    bits_, group, sym, _ = parse_dtype(fmt)
    V, Cn, T = 4113, 768, 3
    rng = np.random.default_rng(21)
    w = (rng.standard_normal((V, Cn)) * 0.02).astype(np.float32)
    ow = O.QuantMatrix(w, bits_, group, sym, False, False)
    gw = QuantMatrix.from_f32(ctx, w, bits_, group, sym, False, False)
    h = rng.standard_normal((T, Cn)).astype(np.float32)
    try:
        for n in (T, 1):
            want = np.zeros((n, V), np.float32)
            O.lib().oq_affine_matmul_rows(C.byref(ow.q), O.ptr(h[:n]), None, O.ptr(want), n, Cn, V, 0, 0)
            logits = torch.zeros((n, V), dtype=torch.float32, device="cuda")
            kernels.head(ctx, logits, dev(torch, h[:n]), gw, n, V, Cn)
            same(logits.cpu().numpy(), want)
    finally:
        gw.free()


@pytest.mark.parametrize("fmt,kv,T", [("f32", "auto", 20), ("bf16", "auto", 20), ("gguf-q4_k", "auto", 20),
                                      ("int4-g32", "auto", 20), ("int4-g32", "f32", 20), ("int8-ch", "auto", 20),
                                      ("int4-g128-sym", "auto", 20), ("gguf-q4_k", "auto", 1),
                                      ("int4-g32", "auto", 1), ("int8-ch", "f32", 1)])
def test_float_model_forward_all_bit_exact(torch, ctx, gpt2_tensors, fmt, kv, T):
    """forward_all of a 2-layer model, bit for bit with the oracle's; the
    affine W4A32 / W8A32 models with the int8 (auto) or float32 cache. One
    token takes every OUT_MAJOR matrix's one-token path (dot_row), as the
    reference's matmul_rows does for T = 1 (the dense formats' T = 1 gemv is
    tested on its own, test_gpu_formats.py)."""
    from llm_mojo_b200.model import FloatModel

    n_layer = 2
    tokens = np.random.default_rng(8).integers(0, 50257, T).astype(np.int32)
    kw = {} if kv == "auto" else {"kv": kv}
    m = FloatModel(ctx, gpt2_tensors, fmt, n_layer=n_layer, max_t=64, **kw)
    try:
        logits = torch.zeros((T, m.V), dtype=torch.float32, device="cuda")
        m.forward_all(tokens, logits)
        got = logits.cpu().numpy()
    finally:
        m.free()
    same(got, oracle_float_forward(gpt2_tensors, fmt, list(tokens), n_layer, **kw))


def test_score_rows_match_oracle(torch, ctx):
    from llm_mojo_b200._lib import check, lib

    rng = np.random.default_rng(11)
    R, V = 9, 50257
    lm = (rng.standard_normal((R, V)) * 3).astype(np.float32)
    lb = (lm + rng.standard_normal((R, V)).astype(np.float32) * 0.1).astype(np.float32)
    lm[4, 7] = lm[4].max() + 1.0  # a row whose top-1 differs from the base's
    targets = rng.integers(0, V, R).astype(np.int32)
    want = np.zeros((6, R - 2), np.float64)
    O.lib().oq_score_rows(O.ptr(lm), O.ptr(lb), O.ptr(targets), V, 2, R, O.ptr(want), R - 2)
    stats = torch.zeros((6, R - 2), dtype=torch.float64, device="cuda")
    lm_d, lb_d, tg = dev(torch, lm), dev(torch, lb), dev(torch, targets)
    torch.cuda.synchronize()
    check(lib().llmq_score_rows(ctx.h, C.c_void_p(lm_d.data_ptr()), C.c_void_p(lb_d.data_ptr()),
                                C.c_void_p(tg.data_ptr()), V, 2, R, C.c_void_p(stats.data_ptr()), R - 2), ctx.h)
    ctx.sync()
    got = stats.cpu().numpy()
    # float64 sums over the vocabulary in another order: agreement to ~1e-12
    np.testing.assert_allclose(got, want, rtol=1e-11, atol=1e-12)


@pytest.mark.parametrize("fmt,tag", [("f32", "f32"), ("bf16", "bf16"), ("gguf-q4_k", "gguf"), ("int4-g32", "wa32")])
def test_float_model_matches_reference_goldens(torch, ctx, gpt2_tensors, golden, fmt, tag):
    """The whole 12-layer device model against the reference's own NumPy
    GPT-2 (golden/reference_py.npz): logits at all 24 prompt positions and
    the 8 greedy ids after [EOT], within north_star's float tolerance
    max |logit - reference| <= 1e-3 * max |logit|, same argmax."""
    from llm_mojo_b200.model import FloatModel

    prompt = np.ascontiguousarray(golden["prompt24"], dtype=np.int32)
    m = FloatModel(ctx, gpt2_tensors, fmt, max_t=64, **({"kv": "f32"} if tag == "wa32" else {}))
    try:
        logits = torch.zeros((24, m.V), dtype=torch.float32, device="cuda")
        m.forward_all(prompt, logits)
        lg = logits.cpu().numpy()
        ids = list(m.generate([50256], 8))
    finally:
        m.free()
    for rows, key in ((lg[23:24], "p24"), (lg[:16], "all16")):
        top = np.atleast_2d(golden[f"{tag}_{key}_top_ids"]).astype(np.int64)
        vals = np.atleast_2d(golden[f"{tag}_{key}_top_vals"])
        got = np.take_along_axis(rows, top, axis=1)
        assert np.abs(got - vals).max() <= 1e-3 * float(golden[f"{tag}_{key}_max"])
        assert np.array_equal(rows.argmax(axis=1), top[:, 0])
    assert ids == [int(v) for v in golden[f"{tag}_greedy8"]]
