"""Weight formats, mirroring the reference's WeightMatrix trait
(tensor.mojo:49-147) for the formats that run on the GPU.

A QuantMatrix[BITS, GROUP, SYMMETRIC, A16] is quantized on the host by the
reference's rules (from_f32, tensor.mojo:333-383; done in C++ by
llmq_quantize_affine) and uploaded once; the handle owns the device copy
and is released with free(), as WeightMatrix values are.
"""

from __future__ import annotations

import ctypes as C

import numpy as np

from ._lib import check, lib


def _ptr(a: np.ndarray):
    return a.ctypes.data_as(C.c_void_p)


class Context:
    """One device, one stream (llmq_init)."""

    def __init__(self, device: int = 0):
        h = C.c_void_p()
        check(lib().llmq_init(device, C.byref(h)))
        self.h = h
        self.device = device

    def sync(self):
        check(lib().llmq_sync(self.h), self.h)

    def set_stream(self, stream_handle: int | None):
        check(lib().llmq_set_stream(self.h, C.c_void_p(stream_handle or 0)), self.h)

    def close(self):
        if self.h:
            lib().llmq_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def parse_dtype(name: str):
    """--dtype names of the reference's affine formats (gpt2t.mojo:1313-1346):
    int8-ch, int4-ch, int4-g128, int4-g64, int4-g32, each optionally -sym,
    optionally -a16. Returns (bits, group, sym, a16)."""
    parts = name.split("-")
    if len(parts) < 2 or parts[0] not in ("int4", "int8"):
        raise ValueError(f"unknown --dtype {name}")
    bits = int(parts[0][3:])
    g = parts[1]
    group = 0 if g == "ch" else int(g[1:])
    rest = parts[2:]
    sym = "sym" in rest
    a16 = "a16" in rest
    if any(r not in ("sym", "a16") for r in rest):
        raise ValueError(f"unknown --dtype {name}")
    return bits, group, sym, a16


class QuantMatrix:
    """QuantMatrix[BITS, GROUP, SYMMETRIC, A16] on the device."""

    def __init__(self, ctx: Context, bits: int, group: int, sym: bool, a16: bool, rows: int, cols: int,
                 codes: np.ndarray, scale: np.ndarray, zp: np.ndarray):
        self.ctx, self.bits, self.group_param, self.sym, self.a16 = ctx, bits, group, sym, a16
        self.rows, self.cols = rows, cols
        self.group = cols if group == 0 else group
        self.blocked = a16 and bits == 4 and group == 32
        self.codes, self.scale, self.zp = codes, scale, zp
        h = C.c_void_p()
        check(lib().llmq_weight_create_affine(ctx.h, bits, group, int(sym), int(a16), rows, cols, _ptr(codes),
                                              _ptr(scale), _ptr(zp), C.byref(h)), ctx.h)
        self.h = h

    @staticmethod
    def quantize(src: np.ndarray, bits: int, group: int, sym: bool, a16: bool, reduce_rows: bool):
        """Host quantization (from_f32): returns (rows, cols, codes, scale, zp)
        of the stored [OUT, IN] (reduce_rows) or [rows, cols] matrix."""
        src = np.ascontiguousarray(src, dtype=np.float32)
        r, c = src.shape
        n, k = (c, r) if reduce_rows else (r, c)
        g = k if group == 0 else group
        codes = np.zeros(n * k * bits // 8, dtype=np.uint8)
        scale = np.zeros(n * (k // g), dtype=np.uint16)
        zp = np.zeros(n * (k // g), dtype=np.uint8)
        check(lib().llmq_quantize_affine(_ptr(src), r, c, int(reduce_rows), bits, group, int(sym), int(a16),
                                         _ptr(codes), _ptr(scale), _ptr(zp)))
        return n, k, codes, scale, zp

    @classmethod
    def from_f32(cls, ctx: Context, src: np.ndarray, bits: int, group: int, sym: bool, a16: bool,
                 reduce_rows: bool) -> "QuantMatrix":
        n, k, codes, scale, zp = cls.quantize(src, bits, group, sym, a16, reduce_rows)
        return cls(ctx, bits, group, sym, a16, n, k, codes, scale, zp)

    def name(self) -> str:
        """QuantMatrix.name (tensor.mojo:325-331)."""
        g = "ch" if self.group_param == 0 else f"g{self.group_param}"
        s = f"int{self.bits}-{g}" + ("-sym" if self.sym else "")
        return s + "-a16" if self.a16 else s

    def nbytes(self) -> int:
        return int(lib().llmq_weight_nbytes(self.h))

    def free(self):
        if self.h:
            lib().llmq_weight_free(self.h)
            self.h = None

    def __del__(self):
        try:
            self.free()
        except Exception:
            pass


class GGUFMatrix:
    """GGUFMatrix (gguf.mojo:344-512): rows of ggml blocks used as stored."""

    def __init__(self, ctx: Context, ggml_type: int, blocks: np.ndarray, rows: int, cols: int):
        self.ctx, self.kind, self.rows, self.cols = ctx, ggml_type, rows, cols
        self.blocks = np.ascontiguousarray(blocks, dtype=np.uint8)
        h = C.c_void_p()
        check(lib().llmq_weight_create_gguf(ctx.h, ggml_type, _ptr(self.blocks), rows, cols, C.byref(h)), ctx.h)
        self.h = h

    @staticmethod
    def name() -> str:
        return "gguf"

    def has_i16(self) -> bool:
        """GGUFMatrix.has_i16 (gguf.mojo:456-457): Q6_K and Q8_0."""
        return self.kind in (14, 8)

    def nbytes(self) -> int:
        return int(lib().llmq_weight_nbytes(self.h))

    def free(self):
        if self.h:
            lib().llmq_weight_free(self.h)
            self.h = None

    def __del__(self):
        try:
            self.free()
        except Exception:
            pass


class DenseMatrix:
    """DenseMatrix[dtype] (tensor.mojo:150-227): f32 / f16 / bf16 values,
    [rows, cols] as given ([IN, OUT] layer matrices, [V, C] wte)."""

    DTYPES = {"f32": 0, "f16": 1, "bf16": 2}

    def __init__(self, ctx: Context, dtype: str, src: np.ndarray):
        src = np.ascontiguousarray(src, dtype=np.float32)
        self.ctx, self.dtype = ctx, dtype
        self.rows, self.cols = src.shape
        if dtype == "f32":
            data = src
        elif dtype == "f16":
            data = src.astype(np.float16)
        else:  # bfloat16: round to nearest even, as .cast[bfloat16]()
            b = src.view(np.uint32).astype(np.uint64)
            b = (b + 0x7FFF + ((b >> 16) & 1)) >> 16
            data = b.astype(np.uint16)
        self.data = np.ascontiguousarray(data)
        h = C.c_void_p()
        check(lib().llmq_weight_create_dense(ctx.h, self.DTYPES[dtype], _ptr(self.data), self.rows, self.cols,
                                             C.byref(h)), ctx.h)
        self.h = h

    def name(self) -> str:
        return self.dtype

    def nbytes(self) -> int:
        return int(lib().llmq_weight_nbytes(self.h))

    def free(self):
        if self.h:
            lib().llmq_weight_free(self.h)
            self.h = None

    def __del__(self):
        try:
            self.free()
        except Exception:
            pass
