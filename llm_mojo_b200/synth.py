"""Synthetic GPT-2 124M weights and token streams for the benchmark configs.

The reference reads Hugging Face GPT-2 safetensors (gpt2t.mojo:150-187, names
and shapes at gpt2t.mojo:89-118 and :586-604). No real checkpoint is available,
so every config runs on random-init weights: matrices N(0, 0.02), biases 0,
LayerNorm gamma 1 and beta 0, drawn from numpy's PCG64 generator in a fixed
tensor order, so the same seed gives the same bytes on every machine.
"""

from __future__ import annotations

import json
import struct

import numpy as np

N_LAYER = 12
N_HEAD = 12
C = 768
HS = C // N_HEAD
MAX_T = 1024
V = 50257
EOT = 50256

# Per-layer tensors in the order the reference's Model keeps them
# (gpt2t.mojo:84-118): four matrices, then eight float32 vectors.
MAT_NAMES = ("attn.c_attn.weight", "attn.c_proj.weight", "mlp.c_fc.weight", "mlp.c_proj.weight")
MAT_SHAPES = ((C, 3 * C), (C, C), (C, 4 * C), (4 * C, C))  # Hugging Face Conv1D [IN, OUT]
VEC_NAMES = (
    "ln_1.weight", "ln_1.bias", "attn.c_attn.bias", "attn.c_proj.bias",
    "ln_2.weight", "ln_2.bias", "mlp.c_fc.bias", "mlp.c_proj.bias",
)
VEC_LENS = (C, C, 3 * C, C, C, C, 4 * C, C)


def gpt2_random_init(seed: int = 0, n_layer: int = N_LAYER) -> dict[str, np.ndarray]:
    """Returns Hugging Face-named float32 tensors of a random-init GPT-2 124M."""
    rng = np.random.default_rng(seed)

    def normal(shape):
        return (rng.standard_normal(shape, dtype=np.float32) * np.float32(0.02)).astype(np.float32)

    t: dict[str, np.ndarray] = {}
    t["wte.weight"] = normal((V, C))
    t["wpe.weight"] = normal((MAX_T, C))
    for l in range(n_layer):
        p = f"h.{l}."
        for name, shape in zip(MAT_NAMES, MAT_SHAPES):
            t[p + name] = normal(shape)
        for name, n in zip(VEC_NAMES, VEC_LENS):
            fill = 1.0 if name.endswith("ln_1.weight") or name.endswith("ln_2.weight") else 0.0
            t[p + name] = np.full(n, fill, dtype=np.float32)
    t["ln_f.weight"] = np.ones(C, dtype=np.float32)
    t["ln_f.bias"] = np.zeros(C, dtype=np.float32)
    return t


def small_floats(t: dict[str, np.ndarray], n_layer: int = N_LAYER) -> np.ndarray:
    """The float32 parameters in the reference's Model.small order
    (gpt2t.mojo:255-267, SMALL_FLOATS at :576): per layer the eight vectors,
    then wpe, ln_f.weight, ln_f.bias."""
    parts = []
    for l in range(n_layer):
        for name in VEC_NAMES:
            parts.append(t[f"h.{l}.{name}"])
    parts += [t["wpe.weight"].reshape(-1), t["ln_f.weight"], t["ln_f.bias"]]
    return np.ascontiguousarray(np.concatenate(parts).astype(np.float32))


def write_safetensors(t: dict[str, np.ndarray], path: str) -> None:
    """Writes float32 tensors as safetensors. Each header entry lists dtype
    and shape before data_offsets, which the reference's header scan
    (gpt2t.mojo:150-157) finds after the tensor's name."""
    header = {}
    off = 0
    for name, a in t.items():
        n = a.size * 4
        header[name] = {"dtype": "F32", "shape": list(a.shape), "data_offsets": [off, off + n]}
        off += n
    hb = json.dumps(header, separators=(",", ":")).encode()
    hb += b" " * ((8 - len(hb) % 8) % 8)
    with open(path, "wb") as f:
        f.write(struct.pack("<Q", len(hb)))
        f.write(hb)
        for a in t.values():
            f.write(np.ascontiguousarray(a, dtype=np.float32).tobytes())


def uniform_ids(n: int, seed: int) -> np.ndarray:
    """n token ids uniform over [0, V) (configs 2 and 3)."""
    return np.random.default_rng(seed).integers(0, V, size=n, dtype=np.int64).astype(np.int32)


def zipf_ids(n: int, seed: int, s: float = 1.1) -> np.ndarray:
    """n token ids from a Zipf(s) law over [0, V) (config 4): rank r has
    probability proportional to r^-s, ranks mapped to ids by a seeded
    permutation of the vocabulary."""
    rng = np.random.default_rng(seed)
    ranks = np.arange(1, V + 1, dtype=np.float64)
    p = ranks ** -s
    p /= p.sum()
    perm = rng.permutation(V)
    draws = rng.choice(V, size=n, p=p)
    return perm[draws].astype(np.int32)
