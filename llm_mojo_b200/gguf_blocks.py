"""GGUF (llama.cpp) block formats as the reference reads them (gguf.mojo:15-28,
41-98): packing float32 rows into Q4_0 / Q4_1 / Q8_0 / Q4_K / Q5_K / Q6_K
blocks, for the synthetic GEMV sweep and tests (no .gguf files are
available).

Q4_0, Q4_1 and Q8_0 use the gguf package's own quantizer. The K-quants get
a simple round-to-nearest packer written here (per sub-block scale and min,
scales quantized to 6 or 8 bits): any well-formed block is a valid input
for the dequant-dot kernels, and the packed bytes decode with the gguf
package's dequantize.
"""

from __future__ import annotations

import numpy as np

F32, F16, Q4_0, Q4_1, Q8_0, Q4_K, Q5_K, Q6_K = 0, 1, 2, 3, 8, 12, 13, 14
NAMES = {F32: "F32", F16: "F16", Q4_0: "Q4_0", Q4_1: "Q4_1", Q8_0: "Q8_0", Q4_K: "Q4_K", Q5_K: "Q5_K", Q6_K: "Q6_K"}
BLOCK_SIZE = {F32: 1, F16: 1, Q4_0: 32, Q4_1: 32, Q8_0: 32, Q4_K: 256, Q5_K: 256, Q6_K: 256}
BLOCK_BYTES = {F32: 4, F16: 2, Q4_0: 18, Q4_1: 20, Q8_0: 34, Q4_K: 144, Q5_K: 176, Q6_K: 210}


def row_bytes(t: int, cols: int) -> int:
    return cols // BLOCK_SIZE[t] * BLOCK_BYTES[t]


def _f16(a) -> np.ndarray:
    return np.asarray(a, dtype=np.float32).astype(np.float16)


def _pack_k_scales(sc: np.ndarray, mn: np.ndarray) -> np.ndarray:
    """8 six-bit scales and mins per superblock into 12 bytes, the inverse of
    k_scale_min (gguf.mojo:205-221). sc, mn: [n, 8] ints in [0, 63]."""
    n = sc.shape[0]
    q = np.zeros((n, 12), dtype=np.uint8)
    q[:, 0:4] = (sc[:, 0:4] & 63) | ((sc[:, 4:8] >> 4) << 6)
    q[:, 4:8] = (mn[:, 0:4] & 63) | ((mn[:, 4:8] >> 4) << 6)
    q[:, 8:12] = (sc[:, 4:8] & 0xF) | ((mn[:, 4:8] & 0xF) << 4)
    return q


def _q45k(w: np.ndarray, bits: int) -> np.ndarray:
    """Q4_K (bits 4) or Q5_K (bits 5) superblocks of w [n, 256]."""
    n = w.shape[0]
    sub = w.reshape(n, 8, 32)
    lo = np.minimum(sub.min(axis=2), 0)
    hi = np.maximum(sub.max(axis=2), 0)
    levels = (1 << bits) - 1
    scale = (hi - lo) / levels
    mins = -lo
    d = _f16(np.maximum(scale.max(axis=1), 1e-8) / 63)
    dmin = _f16(np.maximum(mins.max(axis=1), 1e-8) / 63)
    df, dmf = d.astype(np.float32), dmin.astype(np.float32)
    sc = np.clip(np.round(scale / df[:, None]), 1, 63).astype(np.int64)
    mn = np.clip(np.round(mins / dmf[:, None]), 0, 63).astype(np.int64)
    step = (df[:, None] * sc)[:, :, None]
    q = np.clip(np.round((sub + (dmf[:, None] * mn)[:, :, None]) / step), 0, levels).astype(np.uint8)
    q = q.reshape(n, 256)
    out = np.zeros((n, 144 if bits == 4 else 176), dtype=np.uint8)
    out[:, 0:2] = d.view(np.uint8).reshape(n, 2)
    out[:, 2:4] = dmin.view(np.uint8).reshape(n, 2)
    out[:, 4:16] = _pack_k_scales(sc, mn)
    qs = np.zeros((n, 128), dtype=np.uint8)
    qh = np.zeros((n, 32), dtype=np.uint8)
    for j in range(4):
        a = q[:, 64 * j: 64 * j + 32]        # sub-block 2j: low nibbles
        b = q[:, 64 * j + 32: 64 * j + 64]   # sub-block 2j+1: high nibbles
        qs[:, 32 * j: 32 * j + 32] = (a & 0xF) | ((b & 0xF) << 4)
        qh |= ((a >> 4) & 1) << (2 * j)
        qh |= ((b >> 4) & 1) << (2 * j + 1)
    if bits == 4:
        out[:, 16:144] = qs
    else:
        out[:, 16:48] = qh
        out[:, 48:176] = qs
    return out


def _q6k(w: np.ndarray) -> np.ndarray:
    """Q6_K superblocks of w [n, 256]: 16 sub-blocks of 16 with int8 scales."""
    n = w.shape[0]
    # sub-block s covers weights 128*(s//8) + 32*((s%8)//2) + 16*(s%2) .. +16
    idx = np.array([[128 * (s // 8) + 32 * ((s % 8) // 2) + 16 * (s % 2) + i for i in range(16)] for s in range(16)])
    sub = w[:, idx]  # [n, 16, 16]
    amax = np.abs(sub).max(axis=2)
    scale = amax / 31
    d = _f16(np.maximum(scale.max(axis=1), 1e-8) / 127)
    df = d.astype(np.float32)
    sc = np.clip(np.round(scale / df[:, None]), 1, 127).astype(np.int64)
    step = (df[:, None] * sc)[:, :, None]
    qsub = np.clip(np.round(sub / step) + 32, 0, 63).astype(np.uint8)
    q = np.zeros((n, 256), dtype=np.uint8)
    q[:, idx] = qsub
    out = np.zeros((n, 210), dtype=np.uint8)
    for nn in range(2):
        for h in range(2):
            for k in range(4):
                wq = q[:, 128 * nn + 32 * k + 16 * h: 128 * nn + 32 * k + 16 * h + 16]
                lo_byte = 64 * nn + (32 if k % 2 else 0) + 16 * h
                shift = 4 if k >= 2 else 0
                out[:, lo_byte: lo_byte + 16] |= (wq & 0xF) << shift
                hb = 128 + 32 * nn + 16 * h
                out[:, hb: hb + 16] |= ((wq >> 4) & 3) << (2 * k)
    scales = np.zeros((n, 16), dtype=np.int8)
    for s in range(16):
        nn, rest = s // 8, s % 8
        k, h = rest // 2, rest % 2
        scales[:, 8 * nn + h + 2 * k] = sc[:, s]
    out[:, 192:208] = scales.view(np.uint8)
    out[:, 208:210] = d.view(np.uint8).reshape(n, 2)
    return out


def quantize(w: np.ndarray, t: int) -> np.ndarray:
    """Rows of w [rows, cols] (cols a multiple of the block size) as GGUF
    blocks of type t: uint8 [rows, row_bytes(t, cols)]."""
    w = np.ascontiguousarray(w, dtype=np.float32)
    rows, cols = w.shape
    if t == F32:
        return w.view(np.uint8).reshape(rows, cols * 4).copy()
    if t == F16:
        return w.astype(np.float16).view(np.uint8).reshape(rows, cols * 2).copy()
    if t in (Q4_0, Q4_1, Q8_0):
        from gguf import GGMLQuantizationType as Q
        from gguf.quants import quantize as gq

        qt = {Q4_0: Q.Q4_0, Q4_1: Q.Q4_1, Q8_0: Q.Q8_0}[t]
        return np.ascontiguousarray(gq(w, qt)).reshape(rows, row_bytes(t, cols)).astype(np.uint8)
    blocks = w.reshape(rows * cols // 256, 256)
    packed = _q45k(blocks, 4) if t == Q4_K else _q45k(blocks, 5) if t == Q5_K else _q6k(blocks)
    return packed.reshape(rows, row_bytes(t, cols))


def dequantize_reference(blocks: np.ndarray, t: int, cols: int) -> np.ndarray:
    """The gguf package's dequantization of packed rows (third-party check)."""
    from gguf import GGMLQuantizationType as Q
    from gguf.quants import dequantize

    qt = {F32: Q.F32, F16: Q.F16, Q4_0: Q.Q4_0, Q4_1: Q.Q4_1, Q8_0: Q.Q8_0, Q4_K: Q.Q4_K, Q5_K: Q.Q5_K,
          Q6_K: Q.Q6_K}[t]
    return dequantize(blocks, qt).reshape(blocks.shape[0], cols).astype(np.float32)
