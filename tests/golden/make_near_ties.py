"""Generates ``near_ties.pt``: ``select_tokens`` (WAMInfer/approximation.py:55-67)
run by the reference's own code on constructed near-ties.

    PYTHONDONTWRITEBYTECODE=1 python tests/golden/make_near_ties.py /path/to/WAMInfer-checkout

Every feature value is k/16 with |k| <= 64 (exact in bf16), and in each
element ``now`` and ``before`` share a sign with |before| <= |now|, so each
row's sums of |now - before| and |now| + |before| are multiples of 1/16 below
2^15: exact in float32 whatever order a reduction adds them in.  The scores
2N/D of a row with sums N/16 and D/16 are then the correctly rounded float32
quotients in the reference and in any correct implementation, so the expected
indices do not depend on torch's reduction order, and rows can be placed a
chosen number of float32 ulps apart:

* a group of rows whose scores are the same float32 value s0 although their
  exact ratios differ (ties: the smaller index wins);
* rows at s0 + 1 ulp, s0 + 2 ulp and s0 - 1 ulp;
* rows far above and below, all-zero rows (score 0, denominator clamped to
  1e-6) and mandatory rows;

with `count` placing the cut inside the tie group, between the 1-ulp groups,
and on a group edge.  Nothing here runs at test time.
"""

from __future__ import annotations

import sys
import types
from pathlib import Path
from types import SimpleNamespace

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
DIM = 3072
N = 120
UNIT = 16          # values are k / UNIT
K_MAX = 64         # |k| <= 64: values up to 4.0


def import_reference(checkout: str):
    stub = types.ModuleType("WAMInfer")
    stub.__path__ = [str(Path(checkout) / "WAMInfer")]
    sys.modules["WAMInfer"] = stub
    import WAMInfer.approximation as approx
    return approx


def f32_score(n_units: int, d_units: int) -> np.float32:
    """The float32 score of a row whose sums are n_units / 16 and d_units / 16."""
    num = np.float32(n_units / UNIT)
    den = np.maximum(np.float32(d_units / UNIT), np.float32(1e-6))
    return np.float32(np.float32(2) * num / den)


def find_pairs(target: np.float32, want: int, rng, used: set) -> list[tuple[int, int]]:
    """(N, D) in 1/16 units with N + D even whose float32 score equals `target`."""
    found = []
    for d in rng.permutation(np.arange(150_000, 280_000)):
        d = int(d)
        n = int(round(float(target) * d / 2))
        for cand in (n - 1, n, n + 1):
            if (cand + d) % 2 or cand <= 0 or cand > d or (cand, d) in used:
                continue
            if f32_score(cand, d) == target:
                found.append((cand, d))
                used.add((cand, d))
                break
        if len(found) == want:
            return found
    raise RuntimeError(f"not enough pairs for {target}")


def realise(n_units: int, d_units: int, rng) -> tuple[np.ndarray, np.ndarray]:
    """now, before [DIM] (k / 16 values) with sum|now - before| = N / 16 and
    sum(|now| + |before|) = D / 16."""
    a_total, b_total = (n_units + d_units) // 2, (d_units - n_units) // 2
    if a_total > DIM * K_MAX:
        raise ValueError("row sums too large")
    a = np.zeros(DIM, dtype=np.int64)
    b = np.zeros(DIM, dtype=np.int64)
    # spread |now| over the elements, then |before| <= |now| element-wise
    base, extra = divmod(a_total, DIM)
    a[:] = base
    a[:extra] += 1
    assert a.min() >= 0 and a.max() <= K_MAX and a.sum() == a_total
    remaining = b_total
    for i in rng.permutation(DIM):
        take = min(int(a[i]), remaining)
        b[i] = take
        remaining -= take
        if remaining == 0:
            break
    assert remaining == 0
    sign = np.where(rng.random(DIM) < 0.5, -1, 1)
    perm = rng.permutation(DIM)
    return (sign * a)[perm] / UNIT, (sign * b)[perm] / UNIT


def make_cases(approx) -> dict:
    rng = np.random.default_rng(2024)
    s0 = f32_score(70_001, 200_000)  # about 0.7
    ulp = np.spacing(s0)
    used: set = set()
    groups = {
        "tie": find_pairs(s0, 10, rng, used),
        "plus1": find_pairs(np.float32(s0 + ulp), 5, rng, used),
        "plus2": find_pairs(np.float32(s0 + 2 * ulp), 5, rng, used),
        "minus1": find_pairs(np.float32(s0 - ulp), 5, rng, used),
    }
    specs = [(g, nd) for g, pairs in groups.items() for nd in pairs]
    specs += [("high", (int(d * 0.45) * 2, d)) for d in (180_000, 190_000, 200_000)]     # score 1.8
    specs += [("low", (int(d * 0.1) * 2, d)) for d in (200_000, 205_000, 215_000, 225_000)]  # score 0.4
    specs += [("zero", (0, 0))] * 2
    while len(specs) < N:  # rows well below s0 (score 0.1 .. 0.6)
        d = int(rng.integers(75_000, 125_000)) * 2
        specs.append(("fill", (int(d * float(rng.uniform(0.05, 0.3))) // 2 * 2, d)))
    order = rng.permutation(N)  # spread the groups over the row indices
    rows = [specs[i] for i in order]
    now = np.zeros((N, DIM))
    before = np.zeros((N, DIM))
    for r, (_, (n_units, d_units)) in enumerate(rows):
        if d_units:
            now[r], before[r] = realise(n_units, d_units, rng)
    now_t = torch.from_numpy(now).to(torch.bfloat16)
    before_t = torch.from_numpy(before).to(torch.bfloat16)
    assert torch.equal(now_t.double(), torch.from_numpy(now)) and torch.equal(before_t.double(), torch.from_numpy(before))
    # the float32 sums are exact: a float64 sum gives the same values
    num32 = (now_t.float() - before_t.float()).abs().sum(-1)
    num64 = (now_t.double() - before_t.double()).abs().sum(-1)
    assert torch.equal(num32.double(), num64)
    labels = [g for g, _ in rows]
    above = sum(1 for g in labels if g in ("high", "plus1", "plus2"))
    n_mand = 3
    mandatory_rows = [i for i, g in enumerate(labels) if g == "fill"][:n_mand]
    counts = {
        "cut_in_tie_group": above + n_mand + 4,
        "cut_after_plus1": n_mand + labels.count("high") + labels.count("plus2") + labels.count("plus1"),
        "cut_inside_plus1": n_mand + labels.count("high") + labels.count("plus2") + 2,
        "cut_after_tie_group": above + n_mand + labels.count("tie"),
        "cut_inside_minus1": above + n_mand + labels.count("tie") + 3,
    }
    cases = []
    for name, count in counts.items():
        for use_mandatory in (True, False):
            mandatory = torch.zeros(N, dtype=torch.bool)
            if use_mandatory:
                mandatory[mandatory_rows] = True
            c = count if use_mandatory else count - n_mand
            seq = 392
            features = torch.cat((now_t[None], torch.zeros(1, seq - N, DIM, dtype=torch.bfloat16)), dim=1)
            reuse = dict(n=N, count=c, mandatory=mandatory, features=before_t[None])
            state = SimpleNamespace(extras=dict(token_reuse=reuse))
            approx.select_tokens(state, features)
            cases.append(dict(name=f"{name}{'' if use_mandatory else '_no_mandatory'}", count=c, seq=seq,
                              mandatory=mandatory, indices=state.extras["token_indices"].clone()))
    scores = (2 * num32 / (now_t.float().abs() + before_t.float().abs()).sum(-1).clamp_min(1e-6))
    return dict(now=now_t, before=before_t, labels=labels, scores=scores, s0=float(s0), ulp=float(ulp), cases=cases)


def main(checkout: str) -> None:
    approx = import_reference(checkout)
    out = make_cases(approx)
    torch.save(out, HERE / "near_ties.pt")
    print("near_ties.pt", (HERE / "near_ties.pt").stat().st_size, [c["name"] for c in out["cases"]])


if __name__ == "__main__":
    if len(sys.argv) != 2:
        raise SystemExit("usage: make_near_ties.py <directory holding the WAMInfer package>")
    main(sys.argv[1])
