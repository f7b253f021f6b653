"""The split-int8 tcgen05 prefill GEMM against the CPU oracle.

tile_i16 (kernels.mojo:512-573) folds exact int32 segment sums into a float
chain; the GEMM computes every segment sum as 256 * D_h + D_l (- zp * sum x)
from two kind::i8 MMAs, so outputs must be bit-identical to the oracle's, for
every affine A16 format, tile-edge token counts, the leftover output rows
and each epilogue.
"""

import numpy as np
import pytest

from oracle import oracle as O

pytestmark = pytest.mark.gpu

FORMATS = ["int4-g32-a16", "int4-g32-sym-a16", "int4-g64-a16", "int4-g128-a16", "int4-ch-a16", "int8-ch-a16",
           "int8-g32-a16", "int8-g128-sym-a16"]


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


def run_case(torch, ctx, fmt, T, IN, OUT, kernel, seed, epi):
    from llm_mojo_b200 import kernels
    from llm_mojo_b200.tensor import QuantMatrix, parse_dtype

    bits, group, sym, a16 = parse_dtype(fmt)
    rng = np.random.default_rng(seed)
    src = (rng.standard_normal((IN, OUT), dtype=np.float32) * np.float32(0.02)).astype(np.float32)
    ow = O.QuantMatrix(src, bits, group, sym, a16, True)
    gw = QuantMatrix.from_f32(ctx, src, bits, group, sym, a16, True)
    x = rng.standard_normal((T, IN)).astype(np.float32)
    # rows of activations near +-max: the largest int32 segment sums
    x[0] = (rng.uniform(0.9, 1.0, IN) * np.where(np.arange(IN) % 2 == 0, 1, -1)).astype(np.float32)
    x[T - 1] = (rng.uniform(0.9, 1.0, IN) * np.where(np.arange(IN) % 3 == 0, -1, 1)).astype(np.float32)
    b = rng.standard_normal(OUT).astype(np.float32)
    resid = rng.standard_normal((T, OUT)).astype(np.float32) if epi == "resid" else None
    want = O.matmul_rows_a16(x, ow, b, resid_into=resid, gelu=epi == "gelu")
    out = dev(torch, resid if resid is not None else np.zeros((T, OUT), np.float32))
    kernels.set_prefill_kernel(ctx, kernel)
    try:
        kernels.linear(ctx, out, dev(torch, x), gw, dev(torch, b), T, IN, OUT, gelu=epi == "gelu",
                       resid=epi == "resid")
    finally:
        kernels.set_prefill_kernel(ctx, "auto")
    got = out.cpu().numpy()
    gw.free()
    bad = np.argwhere(got.view(np.uint32) != want.view(np.uint32))
    assert bad.size == 0, f"{len(bad)} differ, first {bad[:4].tolist()}, max diff {np.abs(got - want).max()}"


@pytest.mark.parametrize("fmt", FORMATS)
@pytest.mark.parametrize("T,IN,OUT", [(37, 768, 2304), (130, 3072, 768), (5, 768, 70)])
def test_tcgen05_linear_bit_exact(torch, ctx, fmt, T, IN, OUT):
    run_case(torch, ctx, fmt, T, IN, OUT, "tcgen05", T * 13 + OUT, "gelu")


@pytest.mark.parametrize("fmt", ["int4-g32-a16", "int8-ch-a16"])
@pytest.mark.parametrize("epi", ["resid", "plain"])
def test_tcgen05_epilogues_and_full_prompt(torch, ctx, fmt, epi):
    """Config 2's 476-token prompt (four 128-row tiles, the last partial)."""
    run_case(torch, ctx, fmt, 476, 768, 768, "tcgen05", 476, epi)


@pytest.mark.parametrize("T", [16, 128, 129, 256])
def test_tcgen05_tile_edges_match_cuda_core(torch, ctx, T):
    """Token counts at the 128-row tile edges, through the automatic choice."""
    run_case(torch, ctx, "int4-g32-a16", T, 768, 3072 + 17, "auto", T, "gelu")


@pytest.mark.parametrize("npos0,T", [(0, 16), (0, 17), (0, 476), (300, 100), (1000, 24)])
def test_quant8_prefill_attention_matches_one_query_kernel(torch, ctx, npos0, T):
    """The several-token attention (queries staged in blocks of 16) against
    the oracle's attend_float_one, bit for bit."""
    from llm_mojo_b200.kernels import KVCache

    NH, HS, CN, MAXT = 12, 64, 768, 1024
    rng = np.random.default_rng(npos0 + 3 * T)
    n = npos0 + T
    qkv_all = (rng.standard_normal((n, 3 * CN)) * 2).astype(np.float32)
    kv = KVCache(ctx, "int8", 1, MAXT, NH, HS)
    oc = O.lib().oq_qkv8_new(1, MAXT, NH, HS)
    try:
        kv.store(0, 0, n, dev(torch, qkv_all))
        for p in range(n):
            row = qkv_all[p]
            O.lib().oq_qkv8_store(oc, 0, p, O.ptr(np.ascontiguousarray(row[CN:2 * CN])),
                                  O.ptr(np.ascontiguousarray(row[2 * CN:])))
        q = np.ascontiguousarray(qkv_all[npos0:])
        out = torch.zeros((T, CN), dtype=torch.float32, device="cuda")
        kv.attend(out, dev(torch, q), 0, T, npos0)
        want = np.zeros((T, CN), dtype=np.float32)
        for t in range(T):
            for h in range(NH):
                O.lib().oq_qkv8_attend_one(oc, O.ptr(want), O.ptr(q), 0, t, h, npos0)
        got = out.cpu().numpy()
        assert np.array_equal(got.view(np.uint32), want.view(np.uint32)), f"max diff {np.abs(got - want).max()}"
    finally:
        O.lib().oq_qkv8_free(oc)
        kv.free()
