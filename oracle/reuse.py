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


def scores(now: np.ndarray, before: np.ndarray) -> np.ndarray:
    """2 * sum|now - before| / max(sum(|now| + |before|), 1e-6), float32, per row."""
    now = now.astype(np.float32)
    before = before.astype(np.float32)
    num = np.float32(2) * np.abs(now - before).sum(-1, dtype=np.float32)
    den = np.maximum((np.abs(now) + np.abs(before)).sum(-1, dtype=np.float32), np.float32(1e-6))
    return (num / den).astype(np.float32)


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
