"""ctypes binding of libllmq.so (include/llmq.h).

The library is built in-tree (python -m llm_mojo_b200.build). There is no
fallback: if it is missing or fails to load, importing the package's
kernels raises.
"""

from __future__ import annotations

import ctypes as C
import os

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libllmq.so")

OK, ERR_INVALID, ERR_CUDA, ERR_NOMEM, ERR_TIMEOUT, ERR_UNSUPPORTED = 0, 1, 2, 3, 4, 5
BIAS, GELU, RESID = 1, 2, 4
KV_QUANT8, KV_INTATTN, KV_F32, KV_BF16 = 1, 2, 3, 4
MODE_EAGER, MODE_GRAPH, MODE_PERSISTENT, MODE_CLUSTER = 0, 1, 2, 3
PREFILL_AUTO, PREFILL_CUDA_CORE, PREFILL_TCGEN05 = 0, 1, 2


class LlmqError(RuntimeError):
    def __init__(self, status: int, msg: str):
        super().__init__(f"llmq status {status}: {msg}")
        self.status = status


P, I, LL = C.c_void_p, C.c_int, C.c_longlong
PP = C.POINTER(C.c_void_p)

SIGNATURES = {
    "llmq_init": (I, [I, PP]),
    "llmq_destroy": (I, [P]),
    "llmq_last_error": (C.c_char_p, [P]),
    "llmq_set_stream": (I, [P, P]),
    "llmq_sync": (I, [P]),
    "llmq_quantize_affine": (I, [P, I, I, I, I, I, I, I, P, P, P]),
    "llmq_weight_create_affine": (I, [P, I, I, I, I, I, I, P, P, P, PP]),
    "llmq_weight_free": (I, [P]),
    "llmq_weight_create_gguf": (I, [P, I, P, I, I, PP]),
    "llmq_weight_create_dense": (I, [P, I, P, I, I, PP]),
    "llmq_head": (I, [P, P, P, P, I, I, I]),
    "llmq_set_dense_parts": (I, [P, I]),
    "llmq_weight_nbytes": (LL, [P]),
    "llmq_linear": (I, [P, P, P, P, P, I, I, I, I]),
    "llmq_head_argmax": (I, [P, P, P, P, P]),
    "llmq_head_argmax_noalloc": (I, [P, P, P, P, P]),
    "llmq_set_prefill_kernel": (I, [P, I]),
    "llmq_set_wait_limit": (I, [P, LL]),
    "llmq_batch_create": (I, [P, P, I, I, P]),
    "llmq_score_rows": (I, [P, P, P, P, I, I, I, P, I]),
    "llmq_model_save": (I, [P, P, C.c_char_p]),
    "llmq_model_load": (I, [P, C.c_char_p, I, I, P]),
    "llmq_model_load_gguf": (I, [P, C.c_char_p, I, I, P]),
    "llmq_batch_free": (I, [P]),
    "llmq_batch_set_kernel": (I, [P, I]),
    "llmq_batch_generate": (I, [P, P, P, I, I, I, P]),
    "llmq_batch_generate_async": (I, [P, P, P, I, I, I, P]),
    "llmq_layernorm": (I, [P, P, P, P, P, I, I]),
    "llmq_quantize_rows": (I, [P, P, I, I, P, P]),
    "llmq_debug_lane_sums": (I, [P, P, P, P]),
    "llmq_kv_create": (I, [P, I, I, I, I, I, PP]),
    "llmq_kv_free": (I, [P]),
    "llmq_kv_store": (I, [P, P, I, I, I, P]),
    "llmq_kv_attend": (I, [P, P, P, P, I, I, I]),
    "llmq_kv_read": (I, [P, P, P, P, P, P]),
    "llmq_model_create": (I, [P, I, P, P, P, I, I, PP]),
    "llmq_model_free": (I, [P]),
    "llmq_model_forward": (I, [P, P, P, I, I, P, P]),
    "llmq_model_forward_all": (I, [P, P, P, I, P]),
    "llmq_generate": (I, [P, P, P, I, I, P]),
    "llmq_rng_init": (C.c_uint64, [C.c_int64]),
    "llmq_top_k": (I, [P, P, I, I, P]),
    "llmq_sample": (I, [P, P, I, C.c_float, I, P, P]),
    "llmq_generate_sampled": (I, [P, P, P, I, I, C.c_float, I, P, P]),
    "llmq_model_set_mode": (I, [P, I]),
    "llmq_model_mode": (I, [P]),
    "llmq_generate_async": (I, [P, P, P, I, I, P]),
    "llmq_stream": (P, [P]),
    "llmq_model_check": (I, [P, P]),
    "llmq_model_profile": (I, [P, P, I]),
    "llmq_model_profile_read": (I, [P, P, P, I, I]),
}

_lib = None


def lib():
    """Loads libllmq.so; raises if it is not built."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise ImportError(f"{LIB_PATH} is not built; run: python -m llm_mojo_b200.build")
        L = C.CDLL(LIB_PATH)
        for name, (res, args) in SIGNATURES.items():
            f = getattr(L, name)
            f.restype = res
            f.argtypes = args
        _lib = L
    return _lib


def check(status: int, ctx=None):
    if status != OK:
        msg = lib().llmq_last_error(ctx).decode() if ctx else ""
        raise LlmqError(status, msg)
