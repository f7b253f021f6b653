"""The CPU oracle's float-format models against the reference's own NumPy
GPT-2 (tests/reference.py of llm_mojo, outputs in golden/reference_py.npz,
made by golden/make_golden.py):

- f32: the seed-0 weights as float32 (DenseMatrix[float32], DenseKV[f32]);
- bf16: the layer matrices and wte rounded to bfloat16, bfloat16 KV cache
  (reference.py on bfloat16-rounded weights with --kv bf16);
- gguf: a GGUF file of the weights, Q4_K layers and a Q6_K tied head,
  int8 KV cache (reference.py --gguf, which dequantizes with gguf-py and
  gives the Q6_K head int16 inputs, as gpt2t computes it);
- wa32: int4-g32 W4A32 (reference.py's fake-quantized int4-g32 layers and
  int8-ch head with float activations, float32 KV cache: gpt2t --dtype
  int4-g32 --kv f32; with the int8 cache, rounding flips of single cache
  entries move the first positions' logits by up to 2e-3 of the largest).

The tolerance is north_star's for float formats: max |logit - reference| <=
1e-3 * max |logit| (checked at the reference's top logits), and the same
argmax. The reference sums in float64 / NumPy order and rounds half to even,
so bit equality is not expected; the GPU equals the oracle bit for bit
(tests/test_gpu_float.py, tests/test_gpu_eval.py)."""

import numpy as np
import pytest

from float_oracle import oracle_float_forward

TOL = 1e-3
FORMATS = [("f32", "f32"), ("bf16", "bf16"), ("gguf-q4_k", "gguf"), ("int4-g32", "wa32")]
KW = {"int4-g32": {"kv": "f32"}}  # the cache the golden was made with


@pytest.fixture(scope="module")
def p24_logits(gpt2_tensors, golden):
    """Each format's logits at all 24 prompt positions (rows 0-15 are the
    all-positions logits of the prompt's first 16 tokens: the model is
    causal and every row's arithmetic is independent of later rows)."""
    prompt = [int(v) for v in golden["prompt24"]]
    return {fmt: oracle_float_forward(gpt2_tensors, fmt, prompt, 12, **KW.get(fmt, {})) for fmt, _ in FORMATS}


def _check_rows(logits, ids, vals, scale):
    got = np.take_along_axis(np.atleast_2d(logits), np.atleast_2d(ids).astype(np.int64), axis=1)
    err = float(np.abs(got - np.atleast_2d(vals)).max())
    assert err <= TOL * float(scale), f"max |diff| {err} > {TOL} * {float(scale)}"
    assert np.array_equal(np.atleast_2d(logits).argmax(axis=1), np.atleast_2d(ids)[:, 0])


@pytest.mark.parametrize("fmt,tag", FORMATS)
def test_float_model_prompt_logits_match_reference(p24_logits, golden, fmt, tag):
    lg = p24_logits[fmt]
    _check_rows(lg[23], golden[f"{tag}_p24_top_ids"], golden[f"{tag}_p24_top_vals"], golden[f"{tag}_p24_max"])
    _check_rows(lg[:16], golden[f"{tag}_all16_top_ids"], golden[f"{tag}_all16_top_vals"],
                golden[f"{tag}_all16_max"])


@pytest.mark.parametrize("fmt,tag", FORMATS)
def test_float_model_greedy_ids_match_reference(gpt2_tensors, golden, fmt, tag):
    """[EOT] then 8 greedy tokens, recomputing the whole prefix each step as
    reference.py's greedy mode does; the first step's logits are checked
    against the reference's at the tolerance."""
    toks = [50256]
    for i in range(8):
        lg = oracle_float_forward(gpt2_tensors, fmt, toks, 12, **KW.get(fmt, {}))[-1]
        if i == 0:
            _check_rows(lg, golden[f"{tag}_eot_top_ids"], golden[f"{tag}_eot_top_vals"], golden[f"{tag}_eot_max"])
        toks.append(int(np.argmax(lg)))
    assert toks[1:] == [int(v) for v in golden[f"{tag}_greedy8"]]
