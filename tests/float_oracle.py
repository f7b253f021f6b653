"""TEST INFRASTRUCTURE: the float-format model's forward_all composed from
the CPU oracle's kernels (embedding, layernorm, the mm_tile chain or GGUF
matmul_rows, DenseKV or QuantKV[8] attention, lm_head_rows or the GGUF
integer head), for the GPU tests."""

import numpy as np

from oracle import oracle as O

DT = {"f32": 0, "bf16": 2}
_PREP = {}  # (format, id(array), kind) -> converted weights, reused across calls


def _prep(key, make):
    if key not in _PREP:
        _PREP[key] = make()
    return _PREP[key]


def oracle_float_forward(tensors, fmt, tokens, n_layer, head=None, head_fmt="int8", kv="auto"):
    """The float model's forward_all composed from oracle kernels; head (GGUF
    only) is an untied [V, C] output matrix, the logits' Q6_K head. fmt may
    also be an affine W4A32 / W8A32 dtype ('int4-g32', 'int8-ch', ...): its
    layers and head (head_fmt 'int8' = QuantMatrix[8, 0], or 'same') through
    QuantMatrix.dequant_row / dot_row and matmul_rows, the int8 cache (kv
    'auto') or DenseKV[float32] (kv 'f32')."""
    from llm_mojo_b200 import gguf_blocks as G
    from llm_mojo_b200 import synth
    from llm_mojo_b200.model import affine_float_format

    T, Cn, NH, HS = len(tokens), 768, 12, 64
    small = synth.small_floats(tensors, n_layer)
    vec = lambda l, k: small[l * 13 * Cn + [0, 1, 2, 5, 6, 7, 8, 12][k] * Cn:][:[1, 1, 3, 1, 1, 1, 4, 1][k] * Cn]  # noqa
    wpe = small[n_layer * 13 * Cn:][:1024 * Cn].reshape(1024, Cn)
    lnf_w = small[n_layer * 13 * Cn + 1024 * Cn:][:Cn]
    lnf_b = small[n_layer * 13 * Cn + 1025 * Cn:][:Cn]

    def bf16(a):
        b = np.ascontiguousarray(a, dtype=np.float32).view(np.uint32).astype(np.uint64)
        return ((b + 0x7FFF + ((b >> 16) & 1)) >> 16).astype(np.uint16)

    def wdata(a):  # dense weights and DenseKV entries: float32 (dt 0) or bfloat16 (dt 2)
        return np.ascontiguousarray(a, dtype=np.float32) if dt == 0 else bf16(a)

    def wdata_cached(a):
        return _prep((fmt, id(a), "w"), lambda: (a, wdata(a)))[1]

    def q_cached(a, t, transpose):
        return _prep((t, id(a), transpose), lambda: (a, G.quantize(np.ascontiguousarray(a.T if transpose else a,
                                                                                       dtype=np.float32), t)))[1]

    aff = affine_float_format(fmt)
    if aff is not None and kv not in ("auto", "f32"):
        raise ValueError("the oracle's affine model takes the int8 (auto) or float32 cache")

    def aq_cached(a, spec, reduce_rows):
        return _prep((spec, id(a), reduce_rows), lambda: (a, O.QuantMatrix(a, *spec, False, reduce_rows)))[1]

    wte = tensors["wte.weight"]
    dt = DT.get(fmt, 0)
    if aff is not None:
        hq = aq_cached(wte, (8, 0, False) if head_fmt == "int8" else aff, False)
        emb = np.zeros((T, Cn), np.float32)
        for i, tok in enumerate(tokens):
            O.lib().oq_dequant_row(O.C.byref(hq.q), int(tok), O.ptr(emb[i]))
    elif fmt == "gguf-q4_k":
        hb = q_cached(wte, G.Q6_K, False)
        emb = np.zeros((T, Cn), np.float32)
        for i, tok in enumerate(tokens):
            O.lib().oq_gguf_dequant_row(G.Q6_K, O.ptr(np.ascontiguousarray(hb[tok])), Cn, O.ptr(emb[i]))
    else:
        wd = wdata_cached(wte)
        emb = (wd.astype(np.float32) if fmt == "f32" else (wd.astype(np.uint32) << 16).view(np.float32))[tokens]
    x = (emb + wpe[:T]).astype(np.float32)
    kv8 = O.lib().oq_qkv8_new(n_layer, 1024, NH, HS) if fmt == "gguf-q4_k" or (aff is not None and kv == "auto") \
        else None

    def mm(w, xin, b, OUT, resid=None, gelu=False):
        Tn, IN = xin.shape
        out = resid.copy() if resid is not None else np.zeros((Tn, OUT), np.float32)
        if aff is not None:
            O.lib().oq_affine_matmul_rows(O.C.byref(aq_cached(w, aff, True).q), O.ptr(xin),
                                          O.ptr(np.ascontiguousarray(b)), O.ptr(out), Tn, IN, OUT,
                                          int(resid is not None), int(gelu))
        elif fmt == "gguf-q4_k":
            blocks = q_cached(w, G.Q4_K, True)
            O.lib().oq_gguf_matmul_rows(G.Q4_K, O.ptr(blocks), G.row_bytes(G.Q4_K, IN), O.ptr(xin),
                                        O.ptr(np.ascontiguousarray(b)), O.ptr(out), Tn, IN, OUT,
                                        int(resid is not None), int(gelu))
        else:
            O.lib().oq_dense_mm(dt, O.ptr(wdata_cached(w)), O.ptr(xin), O.ptr(np.ascontiguousarray(b)), O.ptr(out), Tn, IN,
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
    if aff is not None:
        O.lib().oq_affine_matmul_rows(O.C.byref(hq.q), O.ptr(np.ascontiguousarray(xn)), None, O.ptr(logits), T, Cn, V,
                                      0, 0)
        if kv8 is not None:
            O.lib().oq_qkv8_free(kv8)
    elif fmt == "gguf-q4_k":
        if head is not None:
            hb = G.quantize(np.ascontiguousarray(head, dtype=np.float32), G.Q6_K)
        for t in range(T):
            O.lib().oq_gguf_head_i16(G.Q6_K, O.ptr(hb), V, Cn, O.ptr(np.ascontiguousarray(xn[t])), O.ptr(logits[t]))
        O.lib().oq_qkv8_free(kv8)
    else:
        O.lib().oq_dense_head_rows(dt, O.ptr(wdata_cached(wte)), O.ptr(xn), O.ptr(logits), T, V, Cn)
    return logits
