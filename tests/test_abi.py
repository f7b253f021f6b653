"""The C ABI library on the CPU: it loads, exports every entry point that
include/llmq.h declares, and its host quantizer (QuantMatrix.from_f32,
tensor.mojo:333-383) gives the oracle's bytes. No GPU is touched."""

import ctypes as C
import os
import re

import numpy as np
import pytest

from llm_mojo_b200 import _lib, build
from llm_mojo_b200.tensor import QuantMatrix, parse_dtype
from oracle import oracle as O

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def header_symbols():
    text = open(os.path.join(ROOT, "include", "llmq.h")).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(llmq_[a-z0-9_]+)\s*\(", text)))


def test_library_exports_every_declared_symbol():
    build.build()
    L = C.CDLL(_lib.LIB_PATH)
    syms = header_symbols()
    assert len(syms) >= 20
    missing = [s for s in syms if not hasattr(L, s)]
    assert not missing, missing


def test_binding_declares_every_symbol():
    assert set(header_symbols()) <= set(_lib.SIGNATURES)


@pytest.mark.parametrize("fmt", ["int4-g32-a16", "int4-g32-sym-a16", "int4-g64-a16", "int4-g128-a16",
                                 "int4-ch-a16", "int8-ch-a16", "int4-ch-sym", "int8-ch-sym", "int4-g32"])
@pytest.mark.parametrize("reduce_rows", [True, False])
def test_host_quantizer_matches_oracle(fmt, reduce_rows):
    bits, group, sym, a16 = parse_dtype(fmt)
    rng = np.random.default_rng(3)
    src = (rng.standard_normal((512, 256), dtype=np.float32) * np.float32(0.02)).astype(np.float32)
    src[:, 7] = 0.0  # an all-zero column: groups with s == 0 when reduced along rows
    n, k, codes, scale, zp = QuantMatrix.quantize(src, bits, group, sym, a16, reduce_rows)
    ref = O.QuantMatrix(src, bits, group, sym, a16, reduce_rows)
    assert (n, k) == (ref.rows, ref.cols)
    assert np.array_equal(codes, ref.codes)
    assert np.array_equal(scale, ref.scale)
    assert np.array_equal(zp, ref.zp)


def test_host_quantizer_rejects_bad_groups():
    src = np.zeros((100, 64), dtype=np.float32)
    with pytest.raises(_lib.LlmqError):
        QuantMatrix.quantize(src, 4, 32, False, False, True)  # 100 rows not a multiple of 32
    with pytest.raises(_lib.LlmqError):
        QuantMatrix.quantize(np.zeros((96, 64), dtype=np.float32), 4, 32, False, True, True)  # BLOCKED needs 256


def test_f16_scales_match_numpy_rounding():
    """The host float16 conversion is IEEE round-to-nearest-even, as numpy's."""
    rng = np.random.default_rng(5)
    vals = np.concatenate([rng.standard_normal(20000).astype(np.float32) * 1e-3,
                           np.float32([6.1e-5, 6.0e-8, 3e-8, 65504, 70000, 1e-9])])
    src = np.repeat(vals[:, None] * np.float32(7.0), 32, axis=1).astype(np.float32)
    src[:, 0] = 0.0
    n, k, codes, scale, zp = QuantMatrix.quantize(src, 8, 0, True, False, False)
    want = (np.abs(src).max(axis=1) / np.float32(127)).astype(np.float32)
    want[want == 0] = 1
    assert np.array_equal(scale, want.astype(np.float16).view(np.uint16))
