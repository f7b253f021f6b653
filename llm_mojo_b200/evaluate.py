"""The perplexity / KL harness (--ppl FILE --compare, gpt2t.mojo:1016-1176)
on the GPU: sliding windows over a token stream, every token after the first
scored once, each format's predictions compared with float32's on the same
windows. Windows are independent, so they split over the ranks of a node; the
totals meet in one all-reduce at the end.
"""

from __future__ import annotations

import ctypes as C
import math

import numpy as np

from ._lib import check, lib

WINDOW, STRIDE = 1024, 512
NLL, NLL_BASE, AGREE, KL, DIFF_MAX, DIFF_SUM = range(6)


def schedule(n: int, window: int = WINDOW, stride: int = STRIDE):
    """eval_loop's windows (gpt2t.mojo:1119-1149): [(begin, end, r0, r1)];
    row r of a window predicts ids[begin + r + 1], and rows [r0, r1) are the
    ones not scored by an earlier window."""
    out, scored_until, begin = [], 0, 0
    while True:
        end = min(begin + window, n)
        out.append((begin, end, max(0, scored_until - begin), end - begin - 1))
        scored_until = end - 1
        if end == n:
            return out
        begin += stride


def rank_windows(windows: list, world: int, rank: int) -> list:
    """This rank's windows: round-robin over the ranks (every window scored
    by exactly one rank; the scoring ranges depend only on the window)."""
    return windows[rank::world]


def accumulate(total, s, n_rows: int) -> None:
    """Adds one window's per-row statistics s [6, n_rows] (score_rows'
    layout) into a format's totals [7]: sums of NLL, NLL_BASE, AGREE, KL and
    DIFF_SUM, the max of DIFF_MAX, and the row count."""
    import torch

    total[0:4] += s[[NLL, NLL_BASE, AGREE, KL]].sum(dim=1)
    total[4] += s[DIFF_SUM].sum()
    total[5] = torch.maximum(total[5], s[DIFF_MAX].max())
    total[6] += n_rows


def reduce_totals(totals: dict, world: int) -> None:
    """Combines every rank's totals in place (eval_loop's sums over all
    windows, gpt2t.mojo:1120-1176): one all-reduce SUM of each format's
    totals, then one all-reduce MAX of its largest logit difference, in the
    same order on every rank."""
    if world <= 1:
        return
    import torch.distributed as dist

    for name in totals:
        t = totals[name]
        mx = t[5:6].clone()
        dist.all_reduce(t)
        dist.all_reduce(mx, op=dist.ReduceOp.MAX)
        t[5] = mx[0]


def report_totals(totals: dict, V: int, compared: bool) -> dict:
    """The harness's figures from the combined totals (gpt2t.mojo:1150-1176):
    perplexity and mean NLL, and against float32 its perplexity, top-1
    agreement, mean KL and the mean / max absolute logit difference."""
    out = {}
    for name, t in totals.items():
        t = t.cpu().numpy()
        cnt = t[6]
        r = {"tokens_scored": int(cnt), "perplexity": math.exp(t[0] / cnt), "mean_nll": t[0] / cnt}
        if compared:
            r.update({"f32_perplexity": math.exp(t[1] / cnt), "top1_agreement": t[2] / cnt,
                      "mean_kl": t[3] / cnt, "mean_abs_logit_diff": t[4] / (cnt * V),
                      "max_abs_logit_diff": float(t[5])})
        out[name] = r
    return out


class Harness:
    """Scores formats against a float32 base model. models: {name: model}
    with forward_all(tokens, logits) and V; base: the float32 model (or None
    to score without comparing)."""

    def __init__(self, ctx, models: dict, base=None, window: int = WINDOW):
        import torch

        self.ctx, self.models, self.base, self.window = ctx, models, base, window
        V = next(iter(models.values())).V
        self.V = V
        self.logits = torch.empty((window, V), dtype=torch.float32, device="cuda")
        self.base_logits = torch.empty((window, V), dtype=torch.float32, device="cuda") if base else None
        self.stats = torch.zeros((6, window), dtype=torch.float64, device="cuda")
        self.targets = torch.zeros(window, dtype=torch.int32, device="cuda")
        # per format: sums of NLL, NLL_BASE, AGREE, KL, DIFF_SUM; the max of DIFF_MAX; the count
        self.totals = {name: torch.zeros(7, dtype=torch.float64, device="cuda") for name in models}

    def score_window(self, ids: np.ndarray, begin: int, end: int, r0: int, r1: int):
        import torch

        window = np.ascontiguousarray(ids[begin:end], dtype=np.int32)
        n = len(ids)
        targets = np.array([ids[i + 1] if i + 1 < n else 0 for i in range(begin, end)], dtype=np.int32)
        self.targets[: end - begin].copy_(torch.from_numpy(targets))
        if r1 <= r0:
            return
        base_ptr = None
        if self.base is not None:
            self.base.forward_all(window, self.base_logits)
            base_ptr = C.c_void_p(self.base_logits.data_ptr())
        for name, m in self.models.items():
            m.forward_all(window, self.logits)
            check(lib().llmq_score_rows(self.ctx.h, C.c_void_p(self.logits.data_ptr()), base_ptr,
                                        C.c_void_p(self.targets.data_ptr()), self.V, r0, r1,
                                        C.c_void_p(self.stats.data_ptr()), self.window), self.ctx.h)
            self.ctx.sync()
            accumulate(self.totals[name], self.stats[:, : r1 - r0], r1 - r0)

    def reduce(self, world: int):
        """Sums (and the max) over the ranks (reduce_totals)."""
        reduce_totals(self.totals, world)

    def report(self) -> dict:
        return report_totals(self.totals, self.V, self.base is not None)
