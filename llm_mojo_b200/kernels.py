"""The kernels layer (kernels.mojo) on device tensors: linear, head with
greedy argmax, layernorm, quantize_rows, and the KV cache's store/attend.

Arguments are torch CUDA tensors (float32 / int16 / int32, contiguous);
torch only provides the device memory. Calls are issued on the context's
stream and synchronised with torch's before and after, so tensors can be
used directly.
"""

from __future__ import annotations

import ctypes as C

from ._lib import (BIAS, GELU, KV_BF16, KV_F32, KV_INTATTN, KV_QUANT8, PREFILL_AUTO, PREFILL_CUDA_CORE,
                   PREFILL_TCGEN05, RESID, check, lib)
from .tensor import Context, QuantMatrix


def _p(t):
    if t is None:
        return None
    assert t.is_cuda and t.is_contiguous()
    return C.c_void_p(t.data_ptr())


def _pre(ctx: Context):
    import torch

    torch.cuda.current_stream().synchronize()


def linear(ctx: Context, out, x, w: QuantMatrix, b, T: int, IN: int, OUT: int, resid=False, gelu=False):
    """out[T, OUT] (+)= act(x[T, IN] @ w^T + b) (kernels.mojo:655-673)."""
    _pre(ctx)
    flags = (BIAS if b is not None else 0) | (GELU if gelu else 0) | (RESID if resid else 0)
    check(lib().llmq_linear(ctx.h, w.h, _p(x), _p(b), _p(out), T, IN, OUT, flags), ctx.h)
    ctx.sync()


def head(ctx: Context, logits, h, w, T: int, V: int, C_: int):
    """logits[T, V] = h[T, C] @ w[V, C]^T with the head kernel of w's format
    (kernels.mojo:676-690)."""
    _pre(ctx)
    check(lib().llmq_head(ctx.h, w.h, _p(h), _p(logits), T, C_, V), ctx.h)
    ctx.sync()


PREFILL_KERNELS = {"auto": PREFILL_AUTO, "cuda_core": PREFILL_CUDA_CORE, "tcgen05": PREFILL_TCGEN05}


def set_prefill_kernel(ctx: Context, kind: str):
    """The kernel of several-token A16 matmuls: 'auto' (tcgen05 from 16
    tokens), 'cuda_core' or 'tcgen05'. Results are identical."""
    check(lib().llmq_set_prefill_kernel(ctx.h, PREFILL_KERNELS[kind]), ctx.h)


def set_dense_parts(ctx: Context, nparts: int):
    check(lib().llmq_set_dense_parts(ctx.h, nparts), ctx.h)


def head_argmax(ctx: Context, w: QuantMatrix, h, logits, argmax):
    """logits[V] = h[C] @ w^T and the greedy argmax (kernels.mojo:676-690,
    gpt2t.mojo:792-797); argmax is a 1-element int32 device tensor."""
    _pre(ctx)
    check(lib().llmq_head_argmax(ctx.h, w.h, _p(h), _p(logits), _p(argmax)), ctx.h)
    ctx.sync()


class Rng:
    """Rng (gpt2t.mojo:775-789) whose xorshift64* state lives on the device
    (a one-element int64 CUDA tensor holding the uint64 bits), advanced by
    every draw of sample()."""

    def __init__(self, seed: int = 1337):
        import torch

        s = int(lib().llmq_rng_init(seed))
        self.state = torch.tensor([s - (1 << 64) if s >= 1 << 63 else s], dtype=torch.int64, device="cuda")

    def value(self) -> int:
        return int(self.state.item()) & ((1 << 64) - 1)


def top_k(ctx: Context, logits, k: int):
    """Ids of the k largest logits in descending order, ties to the lower id
    (gpt2t.mojo:800-815); k <= 0 gives all. Returns an int32 CUDA tensor."""
    import torch

    V = logits.numel()
    n = min(k, V) if k > 0 else V
    ids = torch.empty(n, dtype=torch.int32, device="cuda")
    _pre(ctx)
    check(lib().llmq_top_k(ctx.h, _p(logits), V, k, _p(ids)), ctx.h)
    ctx.sync()
    return ids


def sample(ctx: Context, logits, temperature: float, k: int, rng: Rng, out=None):
    """One draw of sample (gpt2t.mojo:818-834) from logits[V] on the device;
    returns a one-element int32 CUDA tensor (out, if given)."""
    import torch

    if out is None:
        out = torch.empty(1, dtype=torch.int32, device="cuda")
    _pre(ctx)
    check(lib().llmq_sample(ctx.h, _p(logits), logits.numel(), temperature, k, _p(rng.state), _p(out)), ctx.h)
    ctx.sync()
    return out


def layernorm(ctx: Context, out, x, w, b, T: int, C_: int):
    _pre(ctx)
    check(lib().llmq_layernorm(ctx.h, _p(out), _p(x), _p(w), _p(b), T, C_), ctx.h)
    ctx.sync()


def quantize_rows(ctx: Context, x, T: int, IN: int, xq, sx):
    _pre(ctx)
    check(lib().llmq_quantize_rows(ctx.h, _p(x), T, IN, _p(xq), _p(sx)), ctx.h)
    ctx.sync()


def lane_sums(ctx: Context, w: QuantMatrix, x, lanes):
    """int32 lane sums of dot_row_i16 for every row, [OUT][units][16]."""
    _pre(ctx)
    check(lib().llmq_debug_lane_sums(ctx.h, w.h, _p(x), _p(lanes)), ctx.h)
    ctx.sync()


class KVCache:
    """KVCache (kvcache.mojo:31-87): QuantKV[8] ('int8'), IntAttnKV
    ('intattn'), DenseKV[float32] ('f32') or DenseKV[bfloat16] ('bf16')."""

    def __init__(self, ctx: Context, kind: str, n_layer: int, max_t: int, n_head: int, head_dim: int):
        self.ctx = ctx
        self.kind = {"int8": KV_QUANT8, "intattn": KV_INTATTN, "f32": KV_F32, "bf16": KV_BF16}[kind]
        self.elem = {KV_F32: 4, KV_BF16: 2}.get(self.kind, 1)
        self.shape = (n_layer, max_t, n_head, head_dim)
        h = C.c_void_p()
        check(lib().llmq_kv_create(ctx.h, self.kind, n_layer, max_t, n_head, head_dim, C.byref(h)), ctx.h)
        self.h = h

    def store(self, layer: int, pos0: int, T: int, qkv):
        _pre(self.ctx)
        check(lib().llmq_kv_store(self.ctx.h, self.h, layer, pos0, T, _p(qkv)), self.ctx.h)
        self.ctx.sync()

    def attend(self, out, qkv, layer: int, T: int, pos0: int):
        _pre(self.ctx)
        check(lib().llmq_kv_attend(self.ctx.h, self.h, _p(out), _p(qkv), layer, T, pos0), self.ctx.h)
        self.ctx.sync()

    def read(self):
        """(k, v, ks, vs) host copies of the storage: int8 codes, or float32 /
        bfloat16 bits (uint16) for the dense caches, which have no scales."""
        import numpy as np

        L, T, H, D = self.shape
        dt = {1: np.int8, 2: np.uint16, 4: np.float32}[self.elem]
        k = np.zeros(L * T * H * D, dtype=dt)
        v = np.zeros_like(k)
        ks = np.zeros(L * T * H, dtype=np.float32)
        vs = np.zeros_like(ks)
        ptr = lambda a: a.ctypes.data_as(C.c_void_p)  # noqa: E731
        check(lib().llmq_kv_read(self.ctx.h, self.h, ptr(k), ptr(v), ptr(ks), ptr(vs)), self.ctx.h)
        return k, v, ks, vs

    def free(self):
        if self.h:
            lib().llmq_kv_free(self.h)
            self.h = None

    def __del__(self):
        try:
            self.free()
        except Exception:
            pass
