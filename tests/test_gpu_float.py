"""Float-activation several-token paths (the perplexity harness's formats)
against the CPU oracle, bit for bit: the dense matmul tile (f32 / bf16), the
dense head for every position, GGUF rows for several tokens, the dense KV
caches, a whole float model's forward_all, and the scores."""

import ctypes as C

import numpy as np
import pytest

from oracle import oracle as O

pytestmark = pytest.mark.gpu

DT = {"f32": 0, "bf16": 2}


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


def _oracle_float_forward(tensors, fmt, tokens, n_layer):
    """The float model's forward_all composed from oracle kernels."""
    from llm_mojo_b200 import gguf_blocks as G
    from llm_mojo_b200 import synth

    T, Cn, NH, HS = len(tokens), 768, 12, 64
    small = synth.small_floats(tensors, n_layer)
    vec = lambda l, k: small[l * 13 * Cn + [0, 1, 2, 5, 6, 7, 8, 12][k] * Cn:][:[1, 1, 3, 1, 1, 1, 4, 1][k] * Cn]  # noqa
    wpe = small[n_layer * 13 * Cn:][:1024 * Cn].reshape(1024, Cn)
    lnf_w = small[n_layer * 13 * Cn + 1024 * Cn:][:Cn]
    lnf_b = small[n_layer * 13 * Cn + 1025 * Cn:][:Cn]

    def bf16(a):
        b = np.ascontiguousarray(a, dtype=np.float32).view(np.uint32).astype(np.uint64)
        return ((b + 0x7FFF + ((b >> 16) & 1)) >> 16).astype(np.uint16)

    def wdata(a):
        return np.ascontiguousarray(a, dtype=np.float32) if fmt == "f32" else bf16(a)

    wte = tensors["wte.weight"]
    dt = DT.get(fmt, 0)
    if fmt == "gguf-q4_k":
        hb = G.quantize(wte, G.Q6_K)
        emb = np.zeros((T, Cn), np.float32)
        for i, tok in enumerate(tokens):
            O.lib().oq_gguf_dequant_row(G.Q6_K, O.ptr(np.ascontiguousarray(hb[tok])), Cn, O.ptr(emb[i]))
    else:
        wd = wdata(wte)
        emb = (wd.astype(np.float32) if fmt == "f32" else (wd.astype(np.uint32) << 16).view(np.float32))[tokens]
    x = (emb + wpe[:T]).astype(np.float32)
    kv8 = O.lib().oq_qkv8_new(n_layer, 1024, NH, HS) if fmt == "gguf-q4_k" else None

    def mm(w, xin, b, OUT, resid=None, gelu=False):
        Tn, IN = xin.shape
        out = resid.copy() if resid is not None else np.zeros((Tn, OUT), np.float32)
        if fmt == "gguf-q4_k":
            blocks = G.quantize(np.ascontiguousarray(w.T), G.Q4_K)
            O.lib().oq_gguf_matmul_rows(G.Q4_K, O.ptr(blocks), G.row_bytes(G.Q4_K, IN), O.ptr(xin),
                                        O.ptr(np.ascontiguousarray(b)), O.ptr(out), Tn, IN, OUT,
                                        int(resid is not None), int(gelu))
        else:
            O.lib().oq_dense_mm(dt, O.ptr(wdata(w)), O.ptr(xin), O.ptr(np.ascontiguousarray(b)), O.ptr(out), Tn, IN,
                                OUT, int(resid is not None), int(gelu))
        return out

    for l in range(n_layer):
        xn = O.layernorm(x, vec(l, 0), vec(l, 1))
        qkv = mm(tensors[f"h.{l}.attn.c_attn.weight"], xn, vec(l, 2), 3 * Cn)
        att = np.zeros((T, Cn), np.float32)
        if kv8 is not None:
            for t in range(T):
                O.lib().oq_qkv8_store(kv8, l, t, O.ptr(np.ascontiguousarray(qkv[t, Cn:2 * Cn])),
                                      O.ptr(np.ascontiguousarray(qkv[t, 2 * Cn:])))
            for t in range(T):
                for h in range(NH):
                    O.lib().oq_qkv8_attend_one(kv8, O.ptr(att), O.ptr(qkv), l, t, h, 0)
        else:
            k = wdata(qkv[:, Cn:2 * Cn])
            v = wdata(qkv[:, 2 * Cn:])
            for t in range(T):
                for h in range(NH):
                    O.lib().oq_dkv_attend_one(dt, O.ptr(k), O.ptr(v), NH, HS, O.ptr(att), O.ptr(qkv), t, h, 0)
        x = mm(tensors[f"h.{l}.attn.c_proj.weight"], att, vec(l, 3), Cn, resid=x)
        xn = O.layernorm(x, vec(l, 4), vec(l, 5))
        fc = mm(tensors[f"h.{l}.mlp.c_fc.weight"], xn, vec(l, 6), 4 * Cn, gelu=True)
        x = mm(tensors[f"h.{l}.mlp.c_proj.weight"], fc, vec(l, 7), Cn, resid=x)
    xn = O.layernorm(x, lnf_w, lnf_b)
    V = wte.shape[0]
    logits = np.zeros((T, V), np.float32)
    if fmt == "gguf-q4_k":
        for t in range(T):
            O.lib().oq_gguf_head_i16(G.Q6_K, O.ptr(hb), V, Cn, O.ptr(np.ascontiguousarray(xn[t])), O.ptr(logits[t]))
        O.lib().oq_qkv8_free(kv8)
    else:
        O.lib().oq_dense_head_rows(dt, O.ptr(wdata(wte)), O.ptr(xn), O.ptr(logits), T, V, Cn)
    return logits


@pytest.mark.parametrize("fmt", ["f32", "bf16", "gguf-q4_k"])
def test_float_model_forward_all_bit_exact(torch, ctx, gpt2_tensors, fmt):
    from llm_mojo_b200.model import FloatModel

    n_layer, T = 2, 20
    tokens = np.random.default_rng(8).integers(0, 50257, T).astype(np.int32)
    m = FloatModel(ctx, gpt2_tensors, fmt, n_layer=n_layer, max_t=64)
    try:
        logits = torch.zeros((T, m.V), dtype=torch.float32, device="cuda")
        m.forward_all(tokens, logits)
        got = logits.cpu().numpy()
    finally:
        m.free()
    same(got, _oracle_float_forward(gpt2_tensors, fmt, list(tokens), n_layer))


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
