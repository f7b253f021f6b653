"""The perplexity / KL harness (config 4) against the CPU oracle: on a
2-layer model and a short Zipf stream with small windows, every format's
totals (perplexity, f32 perplexity, top-1 agreement, KL, logit differences)
must match the oracle's forward_all + score_rows to float64 rounding."""

import math

import numpy as np
import pytest

from float_oracle import oracle_float_forward
from oracle import oracle as O

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def torch():
    import torch

    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return torch


def test_harness_matches_oracle(torch, gpt2_tensors):
    from llm_mojo_b200 import build, synth
    from llm_mojo_b200.evaluate import Harness, schedule
    from llm_mojo_b200.model import FloatModel, Model
    from llm_mojo_b200.tensor import Context

    build.build()
    ctx = Context(0)
    n_layer, W, S = 2, 64, 32
    ids = synth.zipf_ids(150, 4)
    base = FloatModel(ctx, gpt2_tensors, "f32", n_layer=n_layer, max_t=W)
    models = {"int4-g32-a16": Model(ctx, gpt2_tensors, n_layer=n_layer, max_t=W),
              "bf16": FloatModel(ctx, gpt2_tensors, "bf16", n_layer=n_layer, max_t=W)}
    h = Harness(ctx, models, base, window=W)
    wins = schedule(len(ids), W, S)
    for begin, end, r0, r1 in wins:
        h.score_window(ids, begin, end, r0, r1)
    got = h.report()
    # the oracle
    om = O.Model(gpt2_tensors, n_layer=n_layer, max_t=W)
    V = 50257
    for name in models:
        tot = np.zeros(6)
        dmax, cnt = 0.0, 0
        for begin, end, r0, r1 in wins:
            win = list(ids[begin:end])
            targets = np.array([ids[i + 1] if i + 1 < len(ids) else 0 for i in range(begin, end)], dtype=np.int32)
            lb = oracle_float_forward(gpt2_tensors, "f32", win, n_layer)
            lm = om.forward_all(win) if name == "int4-g32-a16" else oracle_float_forward(gpt2_tensors, "bf16", win,
                                                                                            n_layer)
            st = np.zeros((6, r1 - r0))
            O.lib().oq_score_rows(O.ptr(np.ascontiguousarray(lm)), O.ptr(np.ascontiguousarray(lb)), O.ptr(targets),
                                  V, r0, r1, O.ptr(st), r1 - r0)
            tot += st.sum(axis=1)
            dmax = max(dmax, st[4].max())
            cnt += r1 - r0
        g = got[name]
        assert g["tokens_scored"] == cnt == len(ids) - 1
        assert math.isclose(g["perplexity"], math.exp(tot[0] / cnt), rel_tol=1e-9)
        assert math.isclose(g["f32_perplexity"], math.exp(tot[1] / cnt), rel_tol=1e-9)
        assert math.isclose(g["top1_agreement"], tot[2] / cnt, rel_tol=1e-12)
        assert math.isclose(g["mean_kl"], tot[3] / cnt, rel_tol=1e-7, abs_tol=1e-12)
        assert math.isclose(g["mean_abs_logit_diff"], tot[5] / (cnt * V), rel_tol=1e-9)
        assert g["max_abs_logit_diff"] == dmax
    om.close()
    for m in list(models.values()) + [base]:
        m.free()
    ctx.close()
