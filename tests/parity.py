"""Parity rules between the CUDA engine and the CPU oracle.

* fp32 logits: |gpu - ref| <= 1e-3 + 1e-4 * |ref| at every step (teacher-forced: the oracle scores
  the windows the GPU actually produced), and max-abs <= 1e-3.
* Greedy tokens: the GPU's token must be the oracle's argmax, except at steps where the oracle's
  top-2 gap is below the logit tolerance; such steps are reported.
* Sampled tokens: the GPU's token must be the oracle's draw() with the same generator state,
  except where the draw's target lies within a relative 1e-4 of a cumulative boundary
  (a near-boundary draw, where fp32 logit noise may legitimately flip it); reported likewise.
"""
from __future__ import annotations

from dataclasses import dataclass, field

import numpy as np

from oracle import oracle as orc

ATOL = 1e-3
RTOL = 1e-4
BOUNDARY_RTOL = 1e-4
# Relative slack for the double-precision weights and sums of a draw (CUDA's exp and the host's may
# differ by an ulp per weight, over up to 8192 weights).
DOUBLE_SUM_SLACK = 1e-10


@dataclass
class Report:
    steps: int = 0
    max_abs: float = 0.0
    near_ties: list = field(default_factory=list)
    mismatches: list = field(default_factory=list)


def contexts_along(prefix: np.ndarray, produced: np.ndarray, window: int) -> list:
    """The window the engine scored at each step: tail of prefix + produced[:step]."""
    full = np.concatenate([np.asarray(prefix, np.int64), np.asarray(produced, np.int64)])
    n = len(prefix)
    return [full[step:n + step][-window:] for step in range(len(produced))]


def compare_logits(gpu: np.ndarray, ref: np.ndarray, atol=ATOL, rtol=RTOL, where=""):
    diff = np.abs(gpu.astype(np.float64) - ref.astype(np.float64))
    bound = atol + rtol * np.abs(ref.astype(np.float64))
    worst = float(diff.max()) if diff.size else 0.0
    if np.any(diff > bound):
        i = np.unravel_index(int(np.argmax(diff - bound)), diff.shape)
        raise AssertionError(f"{where}: logits differ by {diff[i]:.3g} at {i} "
                             f"(gpu {gpu[i]!r}, ref {ref[i]!r}, bound {bound[i]:.3g})")
    return worst


def top2_gap(row: np.ndarray) -> float:
    s = np.sort(row.astype(np.float64))
    return float(s[-1] - s[-2]) if s.size > 1 else np.inf


def check_greedy_row(oracle, context, gpu_tokens, gpu_logits, report: Report, where="",
                     atol=ATOL, rtol=RTOL):
    """Teacher-forced comparison of one row's greedy decode."""
    ref = oracle.forced_scores(context, gpu_tokens)
    report.max_abs = max(report.max_abs, compare_logits(gpu_logits, ref, atol, rtol, where))
    report.steps += len(gpu_tokens)
    for step, token in enumerate(gpu_tokens):
        want = int(np.argmax(ref[step]))  # first maximum, as TextEngine.argmax
        if want != int(token):
            if top2_gap(ref[step]) < atol:
                report.near_ties.append((where, step, int(token), want))
            else:
                report.mismatches.append((where, step, int(token), want))
    return ref


def draw_margin(scores: np.ndarray, temperature: float, top_k: int, state: int):
    """Replays TextEngine.draw (TextEngine.java:403-427) on `scores` with generator state `state`.

    The stable descending sort is a lexicographic sort on (-score, index); ``total`` and the
    running sum are sequential double sums in sorted order (np.cumsum adds left to right, as the
    Java loop does). Returns (token, distance of the target to the nearest cumulative boundary
    around it relative to the total, state after the draw)."""
    scores = np.asarray(scores, dtype=np.float64)
    order = np.lexsort((np.arange(scores.size), -scores))[:top_k]
    t = np.float64(np.float32(temperature))
    w = np.exp((scores[order] - scores[order[0]]) / t)
    running = np.cumsum(w)
    total = running[-1]
    state = orc.lcg_advance(state, 1)
    hi = state >> (48 - 26)
    state = orc.lcg_advance(state, 1)
    lo = state >> (48 - 27)
    target = float(((hi << 27) + lo) * 2.0 ** -53) * total
    i = int(np.searchsorted(running, target, side="left"))
    i = min(i, top_k - 1)
    below = running[i - 1] if i > 0 else 0.0
    margin = float(min(abs(running[i] - target), abs(target - below)) / total)
    return int(order[i]), margin, state


def check_sampled_row(oracle, context, gpu_tokens, gpu_logits, temperature, top_k, state,
                      report: Report, where="", atol=ATOL, rtol=RTOL):
    """Teacher-forced comparison of one sampled row starting from generator `state`."""
    ref = oracle.forced_scores(context, gpu_tokens)
    report.max_abs = max(report.max_abs, compare_logits(gpu_logits, ref, atol, rtol, where))
    report.steps += len(gpu_tokens)
    for step, token in enumerate(gpu_tokens):
        want, margin, state = draw_margin(ref[step], temperature, top_k, state)
        if want != int(token):
            if margin < BOUNDARY_RTOL:
                report.near_ties.append((where, step, int(token), want))
                continue  # teacher forcing keeps both sides on the GPU's window
            report.mismatches.append((where, step, int(token), want))
    return state


def draw_undecided(scores: np.ndarray, temperature: float, top_k: int, state: int, delta: float):
    """The tokens TextEngine.draw could return on `scores` moved by at most `delta` each.

    A logit move of <= delta scales every weight exp((s - max) / T) by a factor within
    exp(+-2 delta / T), so each cumulative boundary over the total moves by at most ~4 delta / T
    (plus the double sums' rounding); and tokens whose scores lie within 2 delta of each other may
    trade places in the sorted order. Returns the set of tokens whose buckets meet the target's
    uncertainty interval, widened by those near-equal scores."""
    scores = np.asarray(scores, dtype=np.float64)
    order = np.lexsort((np.arange(scores.size), -scores))[:top_k]
    t = np.float64(np.float32(temperature))
    w = np.exp((scores[order] - scores[order[0]]) / t)
    running = np.cumsum(w)
    total = running[-1]
    state = orc.lcg_advance(state, 1)
    hi = state >> (48 - 26)
    state = orc.lcg_advance(state, 1)
    lo = state >> (48 - 27)
    target = float(((hi << 27) + lo) * 2.0 ** -53) * total
    eps = (4.0 * delta / t * 1.01 + DOUBLE_SUM_SLACK) * total
    k0 = min(int(np.searchsorted(running, target - eps, side="left")), top_k - 1)
    k1 = min(int(np.searchsorted(running, target + eps, side="left")), top_k - 1)
    picked = scores[order[k0:k1 + 1]]
    near = (scores[order] >= picked.min() - 2 * delta) & (scores[order] <= picked.max() + 2 * delta)
    return set(int(x) for x in order[near])


def check_rows(oracle, contexts, rows, gpu_tokens, gpu_logits, report: Report, where="",
               atol=ATOL, rtol=RTOL, sampled=None):
    """Teacher-forced comparison of several rows at once (oracle.forced_scores_rows).

    gpu_tokens: [len(rows), steps]; gpu_logits: [len(rows), steps, V]. For sampled decoding pass
    ``sampled=(temperature, top_k, states)`` with each row's generator state before its first
    draw. Returns the oracle's logits and the per-step agreement of the GPU's tokens with the
    oracle's choice."""
    contexts = np.asarray(contexts)
    ref = oracle.forced_scores_rows(contexts[list(rows)], gpu_tokens)
    agree = []
    for i, r in enumerate(rows):
        here = f"{where} row {r}"
        report.max_abs = max(report.max_abs,
                             compare_logits(gpu_logits[i], ref[i], atol, rtol, here))
        report.steps += gpu_tokens.shape[1]
        state = sampled[2][i] if sampled else None
        for step, token in enumerate(gpu_tokens[i]):
            if sampled:
                # The GPU's draw replayed on its own logits must be exact (the sampler: sort order,
                # double sums, target); against the oracle's logits a draw may differ only where
                # the step's logit difference leaves the draw undecided (draw_undecided).
                own, _, _ = draw_margin(gpu_logits[i, step], sampled[0], sampled[1], state)
                if own != int(token):
                    report.mismatches.append((here + " (sampler)", step, int(token), own))
                delta = float(np.max(np.abs(gpu_logits[i, step].astype(np.float64) -
                                            ref[i, step].astype(np.float64))))
                undecided = draw_undecided(ref[i, step], sampled[0], sampled[1], state, delta)
                want, _, state = draw_margin(ref[i, step], sampled[0], sampled[1], state)
                near = int(token) in undecided
            else:
                want = int(np.argmax(ref[i, step]))
                near = top2_gap(ref[i, step]) < atol
            agree.append(want == int(token))
            if want != int(token):
                (report.near_ties if near else report.mismatches).append(
                    (here, step, int(token), want))
    return ref, float(np.mean(agree)) if agree else 1.0
