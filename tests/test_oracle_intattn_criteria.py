"""The reference's own acceptance criteria for its integer softmax and
integer attention, applied to the CPU oracle's restatements (which the GPU
matches bit for bit, tests/test_gpu_intattn.py):

- tests/int_softmax.mojo: masked_softmax must equal the one-element-at-a-time
  masked_softmax_ref (intmath.mojo:143-172) exactly, give padding positions
  probability 0, and stay within 1e-4 (absolute) and 2e-3 (KL) of float64
  softmax, over lengths 1..1024, three spreads, with and without masks;
- tests/int_attention_check.mojo: IntAttnKV.attend against exact float64
  attention on the same quantized keys, values and query, over its grid of
  (positions before, tokens) and two spreads: max error below 5e-3 of the
  largest output.

The reference draws its inputs from Mojo's random generator, which cannot
run here; the same distributions are drawn with NumPy's, seeded."""

import ctypes as C

import numpy as np
import pytest

from oracle import oracle as O

# intmath.mojo:31-43
FB, MB = 16, 24
MASKED = -(2**31)
D_CAP = 1 << 31
C0, C1, C2, C3 = 1073741824, -742598100, 248207216, -42480028


def masked_softmax_ref(x, mask, has_mask, n, mult):
    """A transcription of masked_softmax_ref (intmath.mojo:143-172), Python
    integers (unbounded, as Mojo's Int does not overflow here)."""
    m = None
    for i in range(n):
        if not has_mask or mask[i] != MASKED:
            v = int(x[i]) + (int(mask[i]) if has_mask else 0)
            m = v if m is None else max(m, v)
    e = [0] * n
    total = 0
    for i in range(n):
        if not has_mask or mask[i] != MASKED:
            v = int(x[i]) + (int(mask[i]) if has_mask else 0)
            y = (min(m - v, D_CAP) * mult) >> MB
            q = y >> FB
            r = y & ((1 << FB) - 1)
            p = C3
            p = ((p * r) >> FB) + C2
            p = ((p * r) >> FB) + C1
            p = ((p * r) >> FB) + C0
            e[i] = 0 if q >= 31 else p >> q
            total += e[i]
    inv = (1 << 61) // total if total > 0 else 0
    return np.array([((ei * inv + (1 << 45)) >> 46) & 0xFFFF for ei in e], dtype=np.uint16)


def test_masked_softmax_matches_scalar_and_float64():
    rng = np.random.default_rng(11)
    scale = 1.0 / 65536  # scores with 16 fraction bits, as the integer attention uses
    mult = int(O.lib().oq_exp_multiplier(scale))
    worst_abs, worst_kl, mismatches, cases = 0.0, 0.0, 0, 0
    for n in [1, 7, 16, 33, 100, 511, 1024]:
        for spread in [1.0, 4.0, 10.0]:
            for use_mask in [False, True]:
                nr = (n + 15) // 16 * 16
                x = (rng.standard_normal(nr) * spread / scale).astype(np.int64).astype(np.int32)
                mask = np.zeros(nr, np.int32)
                if use_mask:
                    mask = (rng.standard_normal(nr) * 0.5 / scale).astype(np.int64).astype(np.int32)
                    drop = (rng.random(nr) < 0.3) & (np.arange(nr) > 0)
                    mask[drop] = MASKED
                e = np.zeros(nr, np.int32)
                p = np.zeros(nr, np.uint16)
                O.lib().oq_masked_softmax(O.ptr(x), O.ptr(mask) if use_mask else None, n, mult, O.ptr(e), O.ptr(p))
                pr = masked_softmax_ref(x, mask, use_mask, n, mult)
                mismatches += int((p[:n] != pr).sum()) + int((p[n:] != 0).sum())
                valid = (mask[:n] != MASKED) if use_mask else np.ones(n, bool)
                v = (x[:n].astype(np.float64) + (mask[:n].astype(np.float64) if use_mask else 0.0)) * scale
                mx = v[valid].max()
                ex = np.where(valid, np.exp(np.where(valid, v - mx, 0.0)), 0.0)
                want = ex / ex.sum()
                got = p[:n].astype(np.float64) / 32768
                worst_abs = max(worst_abs, float(np.abs(got - want).max()))
                pos = want > 0
                kl = float((want[pos] * (np.log(want[pos]) - np.log(np.maximum(got[pos], 0.5 / 32768)))).sum())
                worst_kl = max(worst_kl, kl)
                cases += 1
    assert cases == 42
    assert mismatches == 0
    assert worst_abs < 1e-4, worst_abs
    assert worst_kl < 2e-3, worst_kl


def _round_away(v):
    return np.sign(v) * np.floor(np.abs(v) + 0.5)


def _q(x, qmax):
    """Per-row symmetric quantization in the reference test's float order:
    s = float32(max|x|) / qmax (float32), codes round(x * (1 / s)) with
    float32 products (int_attention_check.mojo:59-83)."""
    x = x.astype(np.float32)
    s = (np.abs(x).max(axis=-1, keepdims=True).astype(np.float32) / np.float32(qmax)).astype(np.float32)
    s = np.where(s == 0, np.float32(1), s).astype(np.float32)
    codes = _round_away((x * (np.float32(1) / s)).astype(np.float32).astype(np.float64))
    return codes, s.astype(np.float64)


GRID = [(0, 1), (0, 5), (15, 1), (16, 1), (99, 1), (200, 7), (511, 1), (1000, 3)]


@pytest.mark.parametrize("npos0,T", GRID)
@pytest.mark.parametrize("spread", [0.5, 2.0])
def test_int_attention_close_to_float64(npos0, T, spread):
    NH, HS, MAXT = 12, 64, 1024
    Cn = NH * HS
    rng = np.random.default_rng(5 + 7 * npos0 + T + int(spread * 10))
    n = npos0 + T
    kf = (rng.standard_normal((n, Cn)) * spread).astype(np.float32)
    vf = rng.standard_normal((n, Cn)).astype(np.float32)
    qkv = (rng.standard_normal((T, 3 * Cn)) * spread).astype(np.float32)
    c = O.lib().oq_intkv_new(1, MAXT, NH, HS)
    try:
        for pos in range(n):
            O.lib().oq_intkv_store(c, 0, pos, O.ptr(np.ascontiguousarray(kf[pos])), O.ptr(np.ascontiguousarray(vf[pos])))
        out = np.zeros((T, Cn), np.float32)
        for t in range(T):
            for h in range(NH):
                O.lib().oq_intkv_attend_one(c, O.ptr(out), O.ptr(qkv), 0, t, h, npos0)
    finally:
        O.lib().oq_intkv_free(c)
    worst, biggest = 0.0, 0.0
    for h in range(NH):
        sl = slice(h * HS, (h + 1) * HS)
        ki, sk = _q(kf[:, sl], 127)
        vi, sv = _q(vf[:, sl], 127)
        qi, sq = _q(qkv[:, sl], 32767)
        for t in range(T):
            npos = npos0 + t + 1
            sc = (ki[:npos] @ qi[t]) * sq[t, 0] * sk[:npos, 0] / np.sqrt(HS)
            w = np.exp(sc - sc.max())
            w = w / w.sum()
            want = (w[:, None] * vi[:npos] * sv[:npos]).sum(axis=0)
            worst = max(worst, float(np.abs(out[t, sl].astype(np.float64) - want).max()))
            biggest = max(biggest, float(np.abs(want).max()))
    assert worst / biggest < 5e-3, worst / biggest


def test_oracle_exports_used_here():
    for name in ("oq_masked_softmax", "oq_exp_multiplier", "oq_intkv_new", "oq_intkv_store", "oq_intkv_attend_one"):
        assert isinstance(getattr(O.lib(), name), C._CFuncPtr)
