"""GPT-2 124M on the device, mirroring the reference's Model[W, E, KV]
(gpt2t.mojo:198-572): load_model's conversion of the layer matrices and the
tied wte/head, forward / forward_all, and greedy generate.
"""

from __future__ import annotations

import ctypes as C

import numpy as np

from . import synth
from ._lib import KV_INTATTN, KV_QUANT8, MODE_CLUSTER, MODE_EAGER, MODE_GRAPH, MODE_PERSISTENT, check, lib
from .tensor import Context, QuantMatrix, parse_dtype

# HEAD8_A16 (gpt2t.mojo:1231-1235): int8 per vocabulary row, integer path.
HEAD8_A16 = (8, 0, False, True)


class Model:
    """Model[W, E, KV] with an A16 layer format W (e.g. 'int4-g32-a16'), the
    int8 head (head='int8') or the layer format (head='same'), and a
    QuantKV[8] ('int8') or IntAttnKV ('intattn') cache."""

    def __init__(self, ctx: Context, tensors: dict, dtype: str = "int4-g32-a16", head: str = "int8",
                 kv: str = "int8", n_layer: int = synth.N_LAYER, max_t: int = synth.MAX_T):
        bits, group, sym, a16 = parse_dtype(dtype)
        if not a16:
            raise ValueError("the device model runs the -a16 formats")
        self.ctx, self.dtype, self.n_layer = ctx, dtype, n_layer
        self.mats = [QuantMatrix.from_f32(ctx, tensors[f"h.{l}.{name}"], bits, group, sym, a16, True)
                     for l in range(n_layer) for name in synth.MAT_NAMES]
        hfmt = HEAD8_A16 if head == "int8" else (bits, group, sym, a16)
        self.head = QuantMatrix.from_f32(ctx, tensors["wte.weight"], *hfmt, False)
        self.small = synth.small_floats(tensors, n_layer)
        arr = (C.c_void_p * len(self.mats))(*[m.h.value for m in self.mats])
        h = C.c_void_p()
        kind = {"int8": KV_QUANT8, "intattn": KV_INTATTN}[kv]
        check(lib().llmq_model_create(ctx.h, n_layer, C.cast(arr, C.c_void_p), self.head.h,
                                      self.small.ctypes.data_as(C.c_void_p), kind, max_t, C.byref(h)), ctx.h)
        self.h = h
        self.V = self.head.rows

    def weight_bytes(self) -> int:
        """Model.weight_bytes (gpt2t.mojo:312-319)."""
        return self.head.nbytes() + sum(m.nbytes() for m in self.mats) + self.small.size * 4

    MODES = {"eager": MODE_EAGER, "graph": MODE_GRAPH, "persistent": MODE_PERSISTENT, "cluster": MODE_CLUSTER}

    def set_mode(self, mode: str):
        """'cluster' (one launch of 16-CTA clusters per generation, the layers
        in one cluster), 'persistent' (one kernel over all SMs per
        generation), 'graph' (a CUDA graph per decode step) or 'eager' (one
        launch per operation)."""
        check(lib().llmq_model_set_mode(self.h, self.MODES[mode]), self.ctx.h)

    def mode(self) -> str:
        m = lib().llmq_model_mode(self.h)
        return {v: k for k, v in self.MODES.items()}[m]

    PROFILE_NAMES = ("embed", "qkv wait", "qkv", "attention", "proj wait", "proj", "fc wait", "fc",
                     "fcproj wait", "fcproj", "head wait", "head", "argmax", "ring waits", "steps",
                     "in: layernorm", "in: quantize", "in: int dots", "in: float epilogue")

    def profile(self, enable: bool = True):
        """Per-phase cycle counters of the persistent kernel (--profile)."""
        check(lib().llmq_model_profile(self.ctx.h, self.h, int(enable)), self.ctx.h)

    # the cluster kernel's counters: layer rank 0, then head CTA 0
    CLUSTER_PROFILE_NAMES = (("embed", "ln1 + quantize", "qkv", "attention", "att all-gather", "proj",
                              "xmid all-gather", "ln2 + quantize", "fc", "fc all-gather", "fcproj",
                              "xout all-gather", "argmax wait", "ring waits", "steps", "in: gemv", "in: ln/quantize",
                              "in: push", "in: attention"),
                             ("hidden-state wait", "ln_f + quantize", "head rows", "ring waits", "steps"))

    def profile_read(self, reset: bool = True) -> list[dict]:
        """Counters of two CTAs, {category: cycles}: CTA 0 and CTA grid/2 of
        the persistent kernel, or layer rank 0 and head CTA 0 of the cluster
        kernel."""
        n = len(self.PROFILE_NAMES) + 1
        buf = (C.c_longlong * (2 * n))()
        check(lib().llmq_model_profile_read(self.ctx.h, self.h, buf, 2 * n, int(reset)), self.ctx.h)
        if self.mode() == "cluster":
            return [dict(zip(names, buf[n * i:n * i + len(names)]))
                    for i, names in enumerate(self.CLUSTER_PROFILE_NAMES)]
        return [dict(zip(self.PROFILE_NAMES, buf[n * i:n * i + n - 1])) for i in range(2)]

    def forward(self, tokens, pos0: int, logits=None) -> int:
        """Runs tokens at positions pos0..; returns the last token's argmax and
        writes its logits into `logits` (a float32 CUDA tensor [V]) if given."""
        t = np.ascontiguousarray(tokens, dtype=np.int32)
        out = C.c_int(0)
        lp = C.c_void_p(logits.data_ptr()) if logits is not None else None
        check(lib().llmq_model_forward(self.ctx.h, self.h, t.ctypes.data_as(C.c_void_p), t.size, pos0, lp,
                                       C.byref(out)), self.ctx.h)
        return out.value

    def forward_all(self, tokens, logits) -> None:
        t = np.ascontiguousarray(tokens, dtype=np.int32)
        check(lib().llmq_model_forward_all(self.ctx.h, self.h, t.ctypes.data_as(C.c_void_p), t.size,
                                           C.c_void_p(logits.data_ptr())), self.ctx.h)

    def generate(self, prompt, steps: int) -> np.ndarray:
        p = np.ascontiguousarray(prompt, dtype=np.int32)
        out = np.zeros(steps, dtype=np.int32)
        check(lib().llmq_generate(self.ctx.h, self.h, p.ctypes.data_as(C.c_void_p), p.size, steps,
                                  out.ctypes.data_as(C.c_void_p)), self.ctx.h)
        return out

    def generate_sampled(self, prompt, steps: int, temperature: float = 0.8, top_k: int = 40,
                         seed: int = 1337, state=None) -> np.ndarray:
        """generate with sample (gpt2t.mojo:818-834, 965-980; defaults -t 0.8
        -k 40 -s 1337) and no stop at EOT. `state`, a one-element uint64
        numpy array, carries the Rng state across calls (seeded from `seed`
        when None)."""
        p = np.ascontiguousarray(prompt, dtype=np.int32)
        out = np.zeros(steps, dtype=np.int32)
        if state is None:
            state = np.array([lib().llmq_rng_init(seed)], dtype=np.uint64)
        check(lib().llmq_generate_sampled(self.ctx.h, self.h, p.ctypes.data_as(C.c_void_p), p.size, steps,
                                          temperature, top_k, state.ctypes.data_as(C.c_void_p),
                                          out.ctypes.data_as(C.c_void_p)), self.ctx.h)
        return out

    def free(self):
        if getattr(self, "h", None):
            lib().llmq_model_free(self.h)
            self.h = None
        for m in getattr(self, "mats", []):
            m.free()
        if getattr(self, "head", None) is not None:
            self.head.free()

    def __del__(self):
        try:
            self.free()
        except Exception:
            pass


class Batch:
    """Greedy decode of independent sequences together (no counterpart in
    the reference, which decodes one at a time): up to max_seqs sequences
    with prompts of up to max_prompt tokens, each with its own QuantKV[8]
    cache. Each sequence's ids equal Model.generate on it alone."""

    def __init__(self, model: Model, max_seqs: int, max_prompt: int):
        self.model, self.max_seqs, self.max_prompt = model, max_seqs, max_prompt
        h = C.c_void_p()
        check(lib().llmq_batch_create(model.ctx.h, model.h, max_seqs, max_prompt, C.byref(h)), model.ctx.h)
        self.h = h

    KERNELS = {"auto": 0, "cuda_core": 1, "tcgen05": 2}

    def set_kernel(self, kind: str):
        """Which kernel runs the batched one-token matmuls: 'auto' (the
        lane-mode tcgen05 GEMM from 16 sequences on), 'cuda_core' (dp2a
        batched GEMVs) or 'tcgen05' (the GEMM at any count)."""
        check(lib().llmq_batch_set_kernel(self.h, self.KERNELS[kind]), self.model.ctx.h)

    def generate(self, prompts, steps: int) -> np.ndarray:
        """prompts [B, P] token ids (host); returns ids [B, steps]."""
        p = np.ascontiguousarray(prompts, dtype=np.int32)
        B, P = p.shape
        out = np.zeros((B, steps), dtype=np.int32)
        check(lib().llmq_batch_generate(self.model.ctx.h, self.h, p.ctypes.data_as(C.c_void_p), B, P, steps,
                                        out.ctypes.data_as(C.c_void_p)), self.model.ctx.h)
        return out

    def generate_async(self, prompts_dev, steps: int, ids_dev):
        """Device prompts (int32 CUDA tensor [B, P]) and ids ([B, steps]),
        enqueued on the context's stream."""
        B, P = prompts_dev.shape
        check(lib().llmq_batch_generate_async(self.model.ctx.h, self.h, C.c_void_p(prompts_dev.data_ptr()), B, P,
                                              steps, C.c_void_p(ids_dev.data_ptr())), self.model.ctx.h)

    def free(self):
        if getattr(self, "h", None):
            lib().llmq_batch_free(self.h)
            self.h = None

    def __del__(self):
        try:
            self.free()
        except Exception:
            pass


# Float formats of the perplexity harness (gpt2t.mojo:1180-1270): the layer
# format, its head and the cache that default_kv picks for it. The affine
# W4A32 / W8A32 formats (an int --dtype without -a16, e.g. 'int4-g32') are
# accepted besides these.
FLOAT_FORMATS = ("f32", "bf16", "gguf-q4_k")


def affine_float_format(fmt: str):
    """(bits, group, sym) of an affine dtype without -a16, else None."""
    try:
        bits, group, sym, a16 = parse_dtype(fmt)
    except ValueError:
        return None
    return None if a16 else (bits, group, sym)


class FloatModel:
    """Model[W, E, KV] for the float-activation formats, run through
    forward_all (evaluation): 'f32' (DenseMatrix[float32] layers and head,
    DenseKV[float32]), 'bf16' (DenseMatrix[bfloat16], DenseKV[bfloat16]),
    'gguf-q4_k' (GGUF Q4_K layers, Q6_K head, the int8 cache: the layout of a
    Q4_K_M file), and the affine W4A32 / W8A32 formats such as 'int4-g32'
    (QuantMatrix layers without -a16, the int8 cache, and head='int8' for
    HEAD8 = QuantMatrix[8, 0] or 'same' for the layer format: run_quantized,
    gpt2t.mojo:1280-1292). Weights are converted from float32 tensors as the
    reference's loaders do."""

    def __init__(self, ctx: Context, tensors: dict, fmt: str, n_layer: int = synth.N_LAYER,
                 max_t: int = synth.MAX_T, head: str = "int8", kv: str = "auto"):
        from . import gguf_blocks as G
        from ._lib import KV_BF16, KV_F32
        from .tensor import DenseMatrix, GGUFMatrix

        aff = affine_float_format(fmt)
        if fmt not in FLOAT_FORMATS and aff is None:
            raise ValueError(f"unknown float format {fmt}")
        self.ctx, self.fmt, self.n_layer = ctx, fmt, n_layer
        self.mats = []
        for l in range(n_layer):
            for name in synth.MAT_NAMES:
                w = tensors[f"h.{l}.{name}"]  # [IN, OUT]
                if aff is not None:
                    self.mats.append(QuantMatrix.from_f32(ctx, w, *aff, False, True))
                elif fmt == "gguf-q4_k":
                    self.mats.append(GGUFMatrix(ctx, G.Q4_K, G.quantize(np.ascontiguousarray(w.T), G.Q4_K),
                                                w.shape[1], w.shape[0]))
                else:
                    self.mats.append(DenseMatrix(ctx, fmt, w))
        wte = tensors["wte.weight"]
        if aff is not None:
            hfmt = (8, 0, False) if head == "int8" else aff
            self.head = QuantMatrix.from_f32(ctx, wte, *hfmt, False, False)
            # default_kv of a quantized format is int8; --kv f32 / bf16 also run
            kind = {"auto": KV_QUANT8, "int8": KV_QUANT8, "f32": KV_F32, "bf16": KV_BF16}[kv]
        elif fmt == "gguf-q4_k":
            self.head = GGUFMatrix(ctx, G.Q6_K, G.quantize(wte, G.Q6_K), wte.shape[0], wte.shape[1])
            kind = KV_QUANT8
        else:
            self.head = DenseMatrix(ctx, fmt, wte)
            kind = KV_F32 if fmt == "f32" else KV_BF16
        self.small = synth.small_floats(tensors, n_layer)
        arr = (C.c_void_p * len(self.mats))(*[m.h.value for m in self.mats])
        h = C.c_void_p()
        check(lib().llmq_model_create(ctx.h, n_layer, C.cast(arr, C.c_void_p), self.head.h,
                                      self.small.ctypes.data_as(C.c_void_p), kind, max_t, C.byref(h)), ctx.h)
        self.h = h
        self.V = self.head.rows

    def forward_all(self, tokens, logits):
        """logits [T, V] (float32 CUDA tensor) for every position of tokens."""
        t = np.ascontiguousarray(tokens, dtype=np.int32)
        check(lib().llmq_model_forward_all(self.ctx.h, self.h, t.ctypes.data_as(C.c_void_p), t.size,
                                           C.c_void_p(logits.data_ptr())), self.ctx.h)

    def forward(self, tokens, pos0: int, logits=None) -> int:
        """The blocks for tokens at pos0.., the last token's logits and argmax
        (the one-token paths for later tokens, as generate uses them)."""
        return Model.forward(self, tokens, pos0, logits)

    def generate(self, prompt, steps: int) -> np.ndarray:
        return Model.generate(self, prompt, steps)

    def generate_sampled(self, prompt, steps: int, temperature: float = 0.8, top_k: int = 40,
                         seed: int = 1337, state=None) -> np.ndarray:
        return Model.generate_sampled(self, prompt, steps, temperature, top_k, seed, state)

    def free(self):
        if getattr(self, "h", None):
            lib().llmq_model_free(self.h)
            self.h = None
        for m in getattr(self, "mats", []):
            m.free()
        if getattr(self, "head", None) is not None:
            self.head.free()

    def __del__(self):
        try:
            self.free()
        except Exception:
            pass


class LoadedModel:
    """A model read from a saved-weights file (load_saved, gpt2t.mojo:667-698)
    or a GGUF file (load_gguf, gpt2t.mojo:728-760); the library owns its
    weights. kv: 'int8', 'intattn', 'f32' or 'bf16'."""

    V = 50257

    def __init__(self, ctx: Context, path: str, kv: str = "int8", max_t: int = synth.MAX_T, gguf: bool = False):
        from ._lib import KV_BF16, KV_F32

        kind = {"int8": KV_QUANT8, "intattn": KV_INTATTN, "f32": KV_F32, "bf16": KV_BF16}[kv]
        self.ctx = ctx
        h = C.c_void_p()
        fn = lib().llmq_model_load_gguf if gguf else lib().llmq_model_load
        check(fn(ctx.h, path.encode(), kind, max_t, C.byref(h)), ctx.h)
        self.h = h

    def forward(self, tokens, pos0: int, logits=None) -> int:
        return Model.forward(self, tokens, pos0, logits)

    def forward_all(self, tokens, logits) -> None:
        return Model.forward_all(self, tokens, logits)

    def generate(self, prompt, steps: int) -> np.ndarray:
        return Model.generate(self, prompt, steps)

    def generate_sampled(self, prompt, steps: int, temperature: float = 0.8, top_k: int = 40,
                         seed: int = 1337, state=None) -> np.ndarray:
        return Model.generate_sampled(self, prompt, steps, temperature, top_k, seed, state)

    def save(self, path: str):
        check(lib().llmq_model_save(self.ctx.h, self.h, path.encode()), self.ctx.h)

    def free(self):
        if getattr(self, "h", None):
            lib().llmq_model_free(self.h)
            self.h = None

    def __del__(self):
        try:
            self.free()
        except Exception:
            pass


def save_model(model, path: str):
    """save_model (gpt2t.mojo:617-643): the model's converted weights to path."""
    check(lib().llmq_model_save(model.ctx.h, model.h, path.encode()), model.ctx.h)
