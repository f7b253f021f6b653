"""The oracle's GGUF block decoding (gguf.mojo:178-297) against the gguf
package's dequantize, on packed random rows (the reference's own check,
tests/gguf_check.py, compares its dequantized rows to gguf-py the same way),
plus the float dot and integer head against exact float64."""

import numpy as np
import pytest

from llm_mojo_b200 import gguf_blocks as G
from oracle import oracle as O

TYPES = [G.F32, G.F16, G.Q4_0, G.Q4_1, G.Q8_0, G.Q4_K, G.Q5_K, G.Q6_K]


def rows_for(t, rows=8, cols=768, seed=0):
    rng = np.random.default_rng(seed + t)
    w = (rng.standard_normal((rows, cols)) * 0.02).astype(np.float32)
    w[0, :40] = 0.0  # a partly zero row
    return w, G.quantize(w, t)


@pytest.mark.parametrize("t", TYPES)
def test_dequant_matches_gguf_package(t):
    w, blocks = rows_for(t)
    want = G.dequantize_reference(blocks, t, w.shape[1])
    got = np.zeros_like(want)
    for r in range(w.shape[0]):
        row = np.ascontiguousarray(blocks[r])
        out = np.zeros(w.shape[1], dtype=np.float32)
        O.lib().oq_gguf_dequant_row(t, O.ptr(row), w.shape[1], O.ptr(out))
        got[r] = out
    # gguf-py computes in float32 with its own operation order: tolerance of
    # a few ulps of the block scale
    assert np.allclose(got, want, rtol=1e-6, atol=1e-7 * np.abs(want).max())
    # and the packing is a reasonable quantization of w
    assert np.abs(got - w).max() < 0.25 * np.abs(w).max()


@pytest.mark.parametrize("t", TYPES)
def test_dot_row_matches_float64(t):
    w, blocks = rows_for(t)
    x = np.random.default_rng(1).standard_normal(w.shape[1]).astype(np.float32)
    for r in range(w.shape[0]):
        row = np.ascontiguousarray(blocks[r])
        deq = np.zeros(w.shape[1], dtype=np.float32)
        O.lib().oq_gguf_dequant_row(t, O.ptr(row), w.shape[1], O.ptr(deq))
        got = O.lib().oq_gguf_dot_row(t, O.ptr(row), w.shape[1], O.ptr(x))
        want = float(np.dot(deq.astype(np.float64), x.astype(np.float64)))
        assert abs(got - want) <= 1e-5 * (np.abs(deq).astype(np.float64) @ np.abs(x) + 1e-12)


@pytest.mark.parametrize("t", [G.Q8_0, G.Q6_K])
def test_integer_head_matches_float64(t):
    """gguf_int_head.mojo's criterion: rel < 1e-5 against exact float64 of the
    same int16 activations and dequantized weights."""
    V, Cn = 64, 768
    w, blocks = rows_for(t, V, Cn)
    h = np.random.default_rng(2).uniform(-3, 3, Cn).astype(np.float32)
    logits = np.zeros(V, dtype=np.float32)
    O.lib().oq_gguf_head_i16(t, O.ptr(np.ascontiguousarray(blocks)), V, Cn, O.ptr(h), O.ptr(logits))
    xq, sx = O.quantize_rows(h[None])
    deq = G.dequantize_reference(blocks, t, Cn).astype(np.float64)
    want = deq @ xq[0].astype(np.float64) * float(sx[0])
    assert np.abs(logits - want).max() / np.abs(want).max() < 1e-5


@pytest.mark.parametrize("dt", [0, 1, 2])
def test_dense_gemv_matches_float64(dt):
    rng = np.random.default_rng(dt)
    IN, OUT = 96, 48
    w = (rng.standard_normal((IN, OUT)) * 0.1).astype(np.float32)
    if dt == 1:
        wd = w.astype(np.float16)
        wf = wd.astype(np.float32)
    elif dt == 2:
        wd = (w.view(np.uint32) >> 16).astype(np.uint16)
        wf = (wd.astype(np.uint32) << 16).view(np.float32)
    else:
        wd = wf = w
    x = rng.standard_normal(IN).astype(np.float32)
    b = rng.standard_normal(OUT).astype(np.float32)
    out = np.zeros(OUT, dtype=np.float32)
    O.lib().oq_dense_gemv(dt, O.ptr(np.ascontiguousarray(wd)), O.ptr(x), O.ptr(b), O.ptr(out), IN, OUT, 4, 0, 0)
    want = x.astype(np.float64) @ wf.astype(np.float64) + b
    assert np.abs(out - want).max() < 1e-5 * np.abs(want).max()
