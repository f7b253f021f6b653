"""TEST INFRASTRUCTURE ONLY: ctypes bindings for the CPU oracle (oracle.c).

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg import
this module, as the checker. The llm_mojo_b200 package never does.
"""

from __future__ import annotations

import ctypes as C
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "liboracle.so")


def build(force: bool = False) -> str:
    """Compiles liboracle.so with oracle/Makefile (gcc only)."""
    src = os.path.join(HERE, "oracle.c")
    if force or not os.path.exists(LIB_PATH) or os.path.getmtime(LIB_PATH) < os.path.getmtime(src):
        subprocess.run(["make", "-C", HERE, "-s", "liboracle.so"], check=True)
    return LIB_PATH


class QMat(C.Structure):
    """oq_qmat: an affine-quantized [rows, cols] matrix (QuantMatrix)."""

    _fields_ = [
        ("bits", C.c_int), ("group", C.c_int), ("sym", C.c_int), ("a16", C.c_int), ("blocked", C.c_int),
        ("rows", C.c_int), ("cols", C.c_int),
        ("codes", C.c_void_p), ("scale", C.c_void_p), ("zp", C.c_void_p),
    ]


_lib = None


def lib():
    global _lib
    if _lib is None:
        _lib = C.CDLL(build())
        _declare(_lib)
    return _lib


def _declare(L):
    P, I, F, D, V = C.c_void_p, C.c_int, C.c_float, C.c_double, None
    I64 = C.c_int64
    sig = {
        "lm_expf": (F, [F]), "lm_tanhf": (F, [F]), "oq_gelu": (F, [F]),
        "oq_quant_affine": (I, [P, I, I, I, I, I, I, I, P, P, P]),
        "oq_dequant_row": (V, [P, I, P]),
        "oq_dot_row": (F, [P, I, P]),
        "oq_quantize_rows": (V, [P, I, I, P, P]),
        "oq_permute_x_i16": (V, [P, I, P, P]),
        "oq_dot_row_i16": (F, [P, I, P, P]),
        "oq_dot_row_i16_lanes": (F, [P, I, P, P, P]),
        "oq_unpack_row_i16": (V, [P, I, P, P]),
        "oq_matmul_rows_a16": (V, [P, P, P, P, I, I, I, I, I]),
        "oq_tile_segment_sums": (V, [P, P, I, P]),
        "oq_layernorm": (V, [P, P, P, P, I, I]),
        "oq_qkv8_new": (P, [I, I, I, I]), "oq_qkv8_free": (V, [P]),
        "oq_qkv8_k": (P, [P]), "oq_qkv8_v": (P, [P]), "oq_qkv8_ks": (P, [P]), "oq_qkv8_vs": (P, [P]),
        "oq_qkv8_store": (V, [P, I, I, P, P]),
        "oq_qkv8_attend_one": (V, [P, P, P, I, I, I, I]),
        "oq_exp_multiplier": (I64, [D]),
        "oq_masked_exp": (I64, [P, P, I, I64, P]),
        "oq_masked_softmax": (V, [P, P, I, I64, P, P]),
        "oq_intkv_new": (P, [I, I, I, I]), "oq_intkv_free": (V, [P]),
        "oq_intkv_k": (P, [P]), "oq_intkv_v": (P, [P]), "oq_intkv_kq": (P, [P]), "oq_intkv_vq": (P, [P]),
        "oq_intkv_store": (V, [P, I, I, P, P]),
        "oq_intkv_attend_one": (V, [P, P, P, I, I, I, I]),
        "oq_model_new": (P, [I, P, P, P, I, I]), "oq_model_free": (V, [P]),
        "oq_model_forward": (V, [P, P, I, I, P]),
        "oq_model_forward_all": (V, [P, P, I, P]),
        "oq_argmax": (I, [P, I]),
        "oq_generate": (V, [P, P, I, I, P]),
        "oq_rng_init": (C.c_uint64, [C.c_int64]), "oq_rng_uniform": (F, [P]),
        "oq_top_k": (I, [P, I, I, P]), "oq_sample": (I, [P, I, F, I, P]),
        "oq_generate_sampled": (V, [P, P, I, I, F, I, P, P]),
        "oq_gguf_block_size": (I, [I]), "oq_gguf_block_bytes": (I, [I]),
        "oq_gguf_dequant_row": (V, [I, P, I, P]),
        "oq_gguf_dot_row": (F, [I, P, I, P]),
        "oq_gguf_dot_row_i16": (F, [I, P, I, P]),
        "oq_gguf_head_i16": (V, [I, P, I, I, P, P]),
        "oq_dense_dot_row": (F, [I, P, I, I, P]),
        "oq_dense_gemv": (V, [I, P, P, P, P, I, I, I, I, I]),
        "oq_threads": (I, []), "oq_set_vnni": (I, [I]),
        "oq_dense_mm": (V, [I, P, P, P, P, I, I, I, I, I]),
        "oq_dense_head_rows": (V, [I, P, P, P, I, I, I]),
        "oq_gguf_matmul_rows": (V, [I, P, C.c_long, P, P, P, I, I, I, I, I]),
        "oq_affine_matmul_rows": (V, [P, P, P, P, I, I, I, I, I]),
        "oq_dkv_attend_one": (V, [I, P, P, I, I, P, P, I, I, I]),
        "oq_score_rows": (V, [P, P, P, I, I, I, P, I]),
    }
    for name, (res, args) in sig.items():
        f = getattr(L, name)
        f.restype = res
        f.argtypes = args


def oq_gelu_np(v: float) -> np.float32:
    """The oracle's GELU of one float32 value."""
    return np.float32(lib().oq_gelu(float(np.float32(v))))


def ptr(a: np.ndarray):
    return a.ctypes.data_as(C.c_void_p)


class QuantMatrix:
    """Oracle-side QuantMatrix[BITS, GROUP, SYM, A16] built with the
    reference's quantizer (tensor.mojo:333-383). Keeps its arrays alive."""

    def __init__(self, src: np.ndarray, bits: int, group: int, sym: bool, a16: bool, reduce_rows: bool):
        src = np.ascontiguousarray(src, dtype=np.float32)
        rows, cols = src.shape
        n, k = (cols, rows) if reduce_rows else (rows, cols)
        g = k if group == 0 else group
        self.codes = np.zeros(n * k * bits // 8, dtype=np.uint8)
        self.scale = np.zeros(n * (k // g), dtype=np.uint16)
        self.zp = np.zeros(n * (k // g), dtype=np.uint8)
        rc = lib().oq_quant_affine(ptr(src), rows, cols, int(reduce_rows), bits, group, int(sym), int(a16),
                                   ptr(self.codes), ptr(self.scale), ptr(self.zp))
        if rc != 0:
            raise ValueError("group size must divide the reduction axis and be a multiple of 32")
        self.bits, self.group_param, self.sym, self.a16 = bits, group, sym, a16
        self.rows, self.cols, self.group = n, k, g
        self.blocked = a16 and bits == 4 and group == 32
        self.q = QMat(bits, g, int(sym), int(a16), int(self.blocked), n, k,
                      self.codes.ctypes.data, self.scale.ctypes.data, self.zp.ctypes.data)

    def dequant(self) -> np.ndarray:
        out = np.zeros((self.rows, self.cols), dtype=np.float32)
        row = np.zeros(self.cols, dtype=np.float32)
        for r in range(self.rows):
            lib().oq_dequant_row(C.byref(self.q), r, ptr(row))
            out[r] = row
        return out


def quantize_rows(x: np.ndarray):
    x = np.ascontiguousarray(x, dtype=np.float32)
    T, IN = x.shape
    xq = np.zeros((T, IN), dtype=np.int16)
    sx = np.zeros(T, dtype=np.float32)
    lib().oq_quantize_rows(ptr(x), T, IN, ptr(xq), ptr(sx))
    return xq, sx


def permute_x_i16(xq: np.ndarray):
    n = xq.size
    dst = np.zeros(n, dtype=np.int16)
    sums = np.zeros(n // 16, dtype=np.float32)
    lib().oq_permute_x_i16(ptr(np.ascontiguousarray(xq)), n, ptr(dst), ptr(sums))
    return dst, sums


def matmul_rows_a16(x: np.ndarray, w: QuantMatrix, b, resid_into=None, gelu=False) -> np.ndarray:
    """out[T, OUT] = act(x @ w^T + b) (+ resid_into)."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    T, IN = x.shape
    out = np.zeros((T, w.rows), dtype=np.float32) if resid_into is None else resid_into.copy()
    bp = ptr(np.ascontiguousarray(b, dtype=np.float32)) if b is not None else None
    lib().oq_matmul_rows_a16(ptr(out), ptr(x), C.byref(w.q), bp, T, IN, w.rows, int(resid_into is not None),
                             int(gelu))
    return out


def lane_sums(w: QuantMatrix, row: int, x1: np.ndarray, xs) -> np.ndarray:
    """int32 lane sums of dot_row_i16 for one row: [cols/256, 16] BLOCKED,
    else [groups, 16]; x1 is the (permuted, for BLOCKED) int16 vector."""
    n = (w.cols // 256) if w.blocked else (w.cols // w.group)
    out = np.zeros((n, 16), dtype=np.int32)
    xs_p = ptr(xs) if xs is not None else None
    lib().oq_dot_row_i16_lanes(C.byref(w.q), row, ptr(np.ascontiguousarray(x1)), xs_p, ptr(out))
    return out


def layernorm(x: np.ndarray, w: np.ndarray, b: np.ndarray) -> np.ndarray:
    x = np.ascontiguousarray(x, dtype=np.float32)
    T, Cn = x.shape
    out = np.zeros_like(x)
    lib().oq_layernorm(ptr(out), ptr(x), ptr(w), ptr(b), T, Cn)
    return out


class Model:
    """Oracle GPT-2 with A16 layer matrices, an A16 head and a QuantKV[8]
    (kv='int8') or IntAttnKV (kv='intattn') cache."""

    def __init__(self, tensors: dict, layer_fmt=(4, 32, False), head_fmt=(8, 0, False), kv="int8",
                 n_layer=12, max_t=1024):
        from llm_mojo_b200 import synth

        self.n_layer = n_layer
        self.mats = []
        for l in range(n_layer):
            for name in synth.MAT_NAMES:
                bits, group, sym = layer_fmt
                self.mats.append(QuantMatrix(tensors[f"h.{l}.{name}"], bits, group, sym, True, True))
        bits, group, sym = head_fmt
        self.head = QuantMatrix(tensors["wte.weight"], bits, group, sym, True, False)
        self.small = synth.small_floats(tensors, n_layer)
        arr = (QMat * (4 * n_layer))(*[m.q for m in self.mats])
        self._arr = arr
        self.kv_kind = {"int8": 0, "intattn": 1}[kv]
        self.h = lib().oq_model_new(n_layer, C.cast(arr, C.c_void_p), C.byref(self.head.q), ptr(self.small),
                                    self.kv_kind, max_t)
        self.V = self.head.rows

    def forward(self, tokens, pos0: int) -> np.ndarray:
        t = np.ascontiguousarray(tokens, dtype=np.int32)
        logits = np.zeros(self.V, dtype=np.float32)
        lib().oq_model_forward(self.h, ptr(t), t.size, pos0, ptr(logits))
        return logits

    def forward_all(self, tokens) -> np.ndarray:
        t = np.ascontiguousarray(tokens, dtype=np.int32)
        logits = np.zeros((t.size, self.V), dtype=np.float32)
        lib().oq_model_forward_all(self.h, ptr(t), t.size, ptr(logits))
        return logits

    def generate(self, prompt, steps: int) -> np.ndarray:
        p = np.ascontiguousarray(prompt, dtype=np.int32)
        out = np.zeros(steps, dtype=np.int32)
        lib().oq_generate(self.h, ptr(p), p.size, steps, ptr(out))
        return out

    def generate_sampled(self, prompt, steps: int, temperature: float = 0.8, top_k: int = 40,
                         seed: int = 1337) -> np.ndarray:
        p = np.ascontiguousarray(prompt, dtype=np.int32)
        out = np.zeros(steps, dtype=np.int32)
        st = np.array([lib().oq_rng_init(seed)], dtype=np.uint64)
        lib().oq_generate_sampled(self.h, ptr(p), p.size, steps, temperature, top_k, ptr(st), ptr(out))
        return out

    def close(self):
        if self.h:
            lib().oq_model_free(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
