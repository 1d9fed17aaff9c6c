"""numpy restatement of the token-reuse index logic (test infrastructure only).

Follows WAMInfer/approximation.py: the RGB mandatory mask and capacity bucket
of ``TokenReuse.begin`` (:18-47) and the score / stable top-k of
``select_tokens`` (:55-67).
"""

from __future__ import annotations

import math

import numpy as np


def capacities(buckets, n):
    """Buckets below n, then n itself (approximation.py:18-19)."""
    return tuple(b for b in sorted(set(buckets)) if b < n) + (n,)


def mandatory_mask(rgb_now, rgb_before, h: int, w: int) -> np.ndarray:
    """Patches whose float32 mean absolute RGB change exceeds 5.0 (approximation.py:32-36)."""
    diff = np.abs(np.subtract(rgb_now, rgb_before, dtype=np.float32))
    H, W = diff.shape[0], diff.shape[1]
    blocks = diff.reshape(h, H // h, w, W // w, 3)
    return blocks.mean(axis=(1, 3, 4)).reshape(-1) > 5.0


def refresh_count(mandatory: np.ndarray, buckets, n: int) -> int:
    """mandatory + ceil(25% of the rest), rounded up to a capacity (approximation.py:37-39)."""
    required = int(mandatory.sum())
    required += math.ceil(0.25 * (n - required))
    return next(b for b in capacities(buckets, n) if b >= required)


LANES = 32   # the device kernel's reduction width (one warp per row)
CHUNK = 8    # elements per lane per step (one 16-byte bf16 vector)


def _row_sums_fixed_order(terms: np.ndarray) -> np.ndarray:
    """Per-row sum of fp32 `terms` [rows, dim] in the device kernel's order,
    accumulated in float64 and rounded once to float32: lane l adds the
    8-element chunks l, l + 32, l + 64, ... element by element, then the 32
    lane sums combine by the xor butterfly with offsets 16, 8, 4, 2, 1
    (waminfer_b200/csrc/select.cuh).  For activations of magnitude >= 2^-30
    (or 0) every float64 partial sum is exact, so the result is the correctly
    rounded exact sum whatever the order."""
    rows, dim = terms.shape
    if dim % CHUNK:
        raise ValueError("dim must be a multiple of 8")
    chunks = dim // CHUNK
    rounds = -(-chunks // LANES)
    padded = np.zeros((rows, rounds * LANES * CHUNK), dtype=np.float64)
    padded[:, :dim] = terms.astype(np.float64)  # widening is exact; padding adds +0.0 (exact)
    blocks = padded.reshape(rows, rounds, LANES, CHUNK)
    acc = np.zeros((rows, LANES), dtype=np.float64)
    for j in range(rounds):
        for i in range(CHUNK):
            acc = acc + blocks[:, j, :, i]
    lane = np.arange(LANES)
    for offset in (16, 8, 4, 2, 1):
        acc = acc + acc[:, lane ^ offset]
    return acc[:, 0].astype(np.float32)


def scores(now: np.ndarray, before: np.ndarray) -> np.ndarray:
    """2 * sum|now - before| / max(sum(|now| + |before|), 1e-6), float32, per
    row (approximation.py:61).  The terms are formed in float32 as the
    reference forms them; the sums follow the fixed order above."""
    now = now.astype(np.float32)
    before = before.astype(np.float32)
    num = _row_sums_fixed_order(np.abs(now - before))
    den = _row_sums_fixed_order(np.abs(now) + np.abs(before))
    return (np.float32(2) * num / np.maximum(den, np.float32(1e-6))).astype(np.float32)


def select_rows(score: np.ndarray, mandatory: np.ndarray, count: int) -> np.ndarray:
    """Mandatory rows first (score +inf), then by descending score; ties keep
    the smaller index; the chosen rows are returned ascending (approximation.py:64-65)."""
    s = np.where(mandatory, np.float32(np.inf), score.astype(np.float32))
    order = sorted(range(s.shape[0]), key=lambda i: (-float(s[i]), i))
    return np.sort(np.asarray(order[:count], dtype=np.int64))


def token_indices(now, before, mandatory, count: int, n: int, seq: int) -> np.ndarray:
    """Selected current rows followed by every future row n..seq-1 (approximation.py:66-67)."""
    chosen = select_rows(scores(now, before), mandatory, count)
    return np.concatenate([chosen, np.arange(n, seq, dtype=np.int64)])
