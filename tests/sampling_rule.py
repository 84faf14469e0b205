"""When may a sampled id differ from the reference's?

The reference draws one number r per sampled token (Sampler::sample,
src/base/sampler.cpp:52-117): it sorts the top-k logits, takes their softmax,
cuts at top-p (and min-p), takes the temperature softmax of the kept prefix
and returns the first candidate whose cumulative probability reaches r. Under
teacher forcing the runtime draws the same r at every step, so its id can
differ from the reference's only if the logit differences move a cumulative
probability across r (or move the top-p cut).

Each logit differs from the reference's by at most delta, so every
unnormalised weight exp((l - top)/T) moves by a factor within
exp(+-delta/T) and its normalised probability within exp(+-2 delta/T): a
cumulative probability C moves by at most C (exp(2 delta/T) - 1). A flip is
explained when r lies that close to a boundary between the two ids' buckets,
or the top-p cumulative (temperature 1) lies within exp(2 delta) - 1 of
top_p. `flip_distance` measures both distances.
"""
from __future__ import annotations

import numpy as np


def sampling_cdf(logits_sorted, temp: float, top_p: float, min_p: float):
    """(cdf over the kept prefix, top-p cumulative, kept count) as the
    reference computes them from the sorted top-k logits (float32)."""
    lg = np.asarray(logits_sorted, np.float32)
    top = lg[0]
    p = np.exp(lg - top).astype(np.float32)
    p = p / np.float32(p.sum(dtype=np.float32))
    acc = np.cumsum(p, dtype=np.float32)
    cut = len(lg)
    hit = np.nonzero(acc >= np.float32(top_p))[0]
    if hit.size:
        cut = int(hit[0]) + 1
    if min_p > 0:
        thr = top + np.float32(np.log(np.float32(min_p)))
        below = np.nonzero(lg[:cut] < thr)[0]
        if below.size:
            cut = int(below[0])
    q = np.exp((lg[:cut] - top) / np.float32(temp)).astype(np.float32)
    q = q / np.float32(q.sum(dtype=np.float32))
    return np.cumsum(q, dtype=np.float32), acc, cut


def pick(cand_ids, cdf, r: float) -> int:
    hit = np.nonzero(cdf >= np.float32(r))[0]
    return int(cand_ids[hit[0]] if hit.size else cand_ids[len(cdf) - 1])


def flip_distance(cand_ids, cand_logits, temp, top_p, min_p, r, id_ref, id_got):
    """(distance of r to the nearest cumulative boundary between the buckets
    of id_ref and id_got, distance of the top-p cumulative to top_p)."""
    cdf, acc, cut = sampling_cdf(cand_logits, temp, top_p, min_p)
    pos = {int(c): i for i, c in enumerate(cand_ids)}
    a = pos.get(int(id_ref), len(cand_ids))
    b = pos.get(int(id_got), len(cand_ids))
    lo, hi = min(a, b), min(max(a, b), cut)
    d_r = min((abs(float(r) - float(cdf[j])) for j in range(lo, min(hi, cut))), default=float("inf"))
    d_p = float(np.min(np.abs(acc.astype(np.float64) - top_p)))
    return d_r, d_p


def explained(delta: float, temp: float, d_r: float, d_p: float) -> bool:
    slack = 1e-6  # float32 rounding of the cumulative sums themselves
    return d_r <= np.expm1(2 * delta / temp) + slack or d_p <= np.expm1(2 * delta) + slack


def check_sampled(got, ref, ref_cands, gpu_rows, top_k: int, temp: float, top_p: float, min_p: float, r,
                  what: str = "") -> list:
    """Asserts that every id of `got` equals `ref` or that the flip rule
    explains it; returns the flips as (step, distance to boundary, top-p
    distance, logit error) and prints each. ref_cands[i] = (ids, logits): the
    reference's top_k + 1 largest logits of step i, largest first; gpu_rows[i]
    = the runtime's logits of step i."""
    flips = []
    for i, (a, b) in enumerate(zip(got, ref)):
        if int(a) == int(b):
            continue
        cid = np.asarray(ref_cands[i][0])
        clg = np.asarray(ref_cands[i][1], np.float32)
        delta = float(np.abs(np.asarray(gpu_rows[i])[cid] - clg).max())
        if int(a) not in cid[:top_k].tolist():
            # the top-k set itself changed: the k-th and next logits lie within 2 delta
            gap = float(clg[top_k - 1] - clg[top_k])
            print(f"{what} flip at step {i}: {a} vs {b} outside the top-k, gap {gap:.3g}, logit error {delta:.3g}")
            assert gap <= 2 * delta + 1e-6, f"{what} step {i}: id {a} outside the reference's top-k (gap {gap})"
            flips.append((i, None, None, delta))
            continue
        d_r, d_p = flip_distance(cid[:top_k], clg[:top_k], temp, top_p, min_p, r[i], b, a)
        print(f"{what} flip at step {i}: {a} vs {b}, r {float(r[i]):.7f}, distance to boundary {d_r:.3g}, "
              f"top-p distance {d_p:.3g}, logit error {delta:.3g}")
        assert explained(delta, temp, d_r, d_p), f"{what} step {i}: flip not explained by the logit error"
        flips.append((i, d_r, d_p, delta))
    return flips


def top_candidates(row, n: int):
    """(ids, logits) of the n largest entries of a logits row, largest first."""
    row = np.asarray(row, np.float32)
    top = np.argsort(-row, kind="stable")[:n]
    return top, row[top]
