"""The CPU oracle against golden vectors made by the reference's own NumPy
GPT-2 (tests/reference.py of llm_mojo, see golden/make_golden.py).

reference.py rounds with np.round (half to even) where the reference's Mojo
code rounds half away from zero (PLAN.md:397), so quantized values may differ
at exact ties only. The int16 activation quantization is discontinuous, so
two correct restatements whose float sums differ by one ulp flip a few codes
per row; through 12 random-init layers that grows to ~5e-3 of the largest
logit. So the model is pinned on a one-layer checkpoint (layers 1-11
zeroed, see golden/make_golden.py) to 1e-4 of the largest logit (the
reference's own --act16 tolerance, PLAN.md:194), and the
12-layer model by identical greedy ids and logits within 1e-2."""

import numpy as np
import pytest

from oracle import oracle as O

FORMATS = [(4, 32, 0), (4, 32, 1), (4, 64, 0), (4, 128, 0), (4, 0, 1), (8, 0, 0), (8, 32, 0)]


def _tie_positions(src_groups, sf):
    q = (src_groups / sf).astype(np.float32)
    return np.abs(q - np.trunc(q)) == 0.5


@pytest.mark.parametrize("bits,group,sym", FORMATS)
@pytest.mark.parametrize("reduce_rows", [True, False])
def test_quantizer_matches_fake_quant(golden, bits, group, sym, reduce_rows):
    src = golden["fq_src"]
    want = golden[("fq" if reduce_rows else "fqh") + f"_{bits}_{group}_{sym}"]
    m = O.QuantMatrix(src, bits, group, bool(sym), False, reduce_rows)
    got = m.dequant()  # stored [n, k]
    got = got.T if reduce_rows else got
    diff = got != want
    # Any difference must be one quantization step at an exact rounding tie.
    if diff.any():
        g = m.group
        scale = np.array([np.float16(0)] * 0)
        sf = m.scale.view(np.float16).astype(np.float32).reshape(m.rows, m.cols // g)
        sf_full = np.repeat(sf, g, axis=1)
        sf_full = sf_full.T if reduce_rows else sf_full
        ties = _tie_positions(src, sf_full)
        assert np.all(ties[diff]), "a value differs away from a rounding tie"
        assert np.allclose(np.abs(got - want)[diff], sf_full[diff], rtol=1e-6)
    assert diff.mean() < 1e-3


def test_quantize_rows_matches_aq(golden):
    xq, sx = O.quantize_rows(golden["aq_src"])
    got = (xq.astype(np.float32) * sx[:, None]).astype(np.float32)
    want = golden["aq"]
    diff = got != want
    assert diff.mean() < 1e-3
    if diff.any():
        q = golden["aq_src"] * (np.float32(1) / sx[:, None])
        assert np.all(np.abs(q - np.trunc(q))[diff] == 0.5)


def test_kv_int8_matches_kvq(golden):
    src = golden["kvq_src"]  # [heads, T, 64]
    H, T, D = src.shape
    c = O.lib().oq_qkv8_new(1, 16, H, D)
    try:
        import ctypes as C

        for t in range(T):
            k = np.ascontiguousarray(src[:, t, :].reshape(-1))
            O.lib().oq_qkv8_store(c, 0, t, O.ptr(k), O.ptr(k))
        codes = np.ctypeslib.as_array(C.cast(O.lib().oq_qkv8_k(c), C.POINTER(C.c_int8)), shape=(16 * H * D,))
        scales = np.ctypeslib.as_array(C.cast(O.lib().oq_qkv8_ks(c), C.POINTER(C.c_float)), shape=(16 * H,))
        codes = codes.reshape(16, H, D)[:T].astype(np.float32)
        sc = scales.reshape(16, H)[:T]
        got = (codes * sc[:, :, None]).transpose(1, 0, 2).astype(np.float32)
    finally:
        O.lib().oq_qkv8_free(c)
    want = golden["kvq_int8"]
    assert (got != want).mean() < 1e-3


def _check_top(got_logits, ids, vals, mx, tol=1e-4):
    assert np.max(np.abs(got_logits[ids] - vals)) <= tol * mx
    # the reference's top ids are the oracle's top ids, up to near-ties
    order = np.argsort(-got_logits, kind="stable")[: len(ids)]
    gap = np.abs(got_logits[order] - got_logits[ids])
    assert np.all((order == ids) | (gap <= 2 * tol * mx))


@pytest.fixture(scope="module")
def oracle_l0(gpt2_tensors):
    t = dict(gpt2_tensors)
    for l in range(1, 12):
        for name in ("attn.c_attn.weight", "attn.c_proj.weight", "mlp.c_fc.weight", "mlp.c_proj.weight"):
            t[f"h.{l}.{name}"] = np.zeros_like(t[f"h.{l}.{name}"])
    return O.Model(t)


def test_one_layer_a16_eot_logits(golden, oracle_l0):
    lg = oracle_l0.forward([50256], 0)
    _check_top(lg, golden["l0_a16_eot_top_ids"], golden["l0_a16_eot_top_vals"], float(golden["l0_a16_eot_max"]),
               tol=1e-4)


def test_one_layer_a16_prefill_logits(golden, oracle_l0):
    lg = oracle_l0.forward(golden["prompt24"], 0)
    _check_top(lg, golden["l0_a16_p24_top_ids"], golden["l0_a16_p24_top_vals"], float(golden["l0_a16_p24_max"]),
               tol=1e-4)


def test_model_a16_eot_logits(golden, oracle_a16):
    lg = oracle_a16.forward([50256], 0)
    _check_top(lg, golden["a16_eot_top_ids"], golden["a16_eot_top_vals"], float(golden["a16_eot_max"]), tol=1e-2)


def test_model_a16_greedy(golden, oracle_a16):
    ids = oracle_a16.generate([50256], 8)
    assert list(ids) == list(golden["a16_greedy8"])


def test_model_a16_prefill_logits(golden, oracle_a16):
    lg = oracle_a16.forward(golden["prompt24"], 0)
    _check_top(lg, golden["a16_p24_top_ids"], golden["a16_p24_top_vals"], float(golden["a16_p24_max"]), tol=1e-2)


def test_model_a16_all_positions(golden, oracle_a16):
    lg = oracle_a16.forward_all(golden["prompt24"][:16])
    mx = float(golden["a16_all16_max"])
    for r in range(16):
        ids, vals = golden["a16_all16_top_ids"][r], golden["a16_all16_top_vals"][r]
        assert np.max(np.abs(lg[r][ids] - vals)) <= 1e-2 * mx


@pytest.mark.parametrize("bits,group", [(4, 32), (8, 0)])
def test_vnni_dots_match_scalar(bits, group):
    """The VNNI integer dots (used where the CPU has AVX-512 VNNI) give the
    scalar lane sums exactly."""
    if not O.lib().oq_set_vnni(1):
        pytest.skip("no AVX-512 VNNI on this CPU")
    rng = np.random.default_rng(3)
    w = O.QuantMatrix(rng.normal(0, 0.02, (768, 96)).astype(np.float32), bits, group, False, True, True)
    xq = rng.integers(-32767, 32768, 768, dtype=np.int16)
    x1, xs = O.permute_x_i16(xq) if w.blocked else (xq, None)
    try:
        fast = [O.lane_sums(w, r, x1, xs) for r in range(w.rows)]
        O.lib().oq_set_vnni(0)
        slow = [O.lane_sums(w, r, x1, xs) for r in range(w.rows)]
    finally:
        O.lib().oq_set_vnni(1)
    assert all(np.array_equal(a, b) for a, b in zip(fast, slow))
