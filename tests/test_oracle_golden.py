"""CPU: the oracle reproduces the reference's own outputs (golden fixtures).

The fixtures were produced by running the reference code (tests/golden/make_golden.py):
the ``_modulated_norm`` Triton kernel, ``VideoAdapter.ffn_at_layer_for_compile``
with the native FFN, ``TokenReuse`` / ``select_tokens`` / ``MotionRefinement``.
"""

import numpy as np
import pytest
import torch

from oracle import ffn as offn
from oracle import reuse as oreuse


def _rows(t):
    return t[0].float() if t.dim() == 3 else t.float()


def test_modulated_norm_matches_reference_kernel(golden):
    cases = golden("modulated_norm.pt")
    assert len(cases) == 12
    for c in cases:
        time = c["time"][0].float() if c["per_token"] else c["time"][0].float()
        y, n = offn.modulated_norm(_rows(c["x"]), _rows(c["update"]), c["mod"][0].float(), c["previous"][0].float(),
                                   time, c["weight"].float(), c["bias"].float(), c["mode"], c["eps"])
        ref_y, ref_n = _rows(c["y"]), _rows(c["norm"])
        # The residual is elementwise bf16 arithmetic: identical.
        assert torch.equal(y, ref_y), (c["dim"], c["mode"])
        # The normalised row differs only through fp32 reduction order (interpreter
        # numpy sum vs torch sum), which can flip one bf16 rounding of an
        # intermediate (|n * scale| < 8): at most 2^-5, on at most 1% of elements.
        diff = (n - ref_n).abs()
        assert float(diff.max()) <= 2.0**-5, (c["dim"], c["mode"], float(diff.max()))
        assert float((diff > 0).float().mean()) <= 0.01, (c["dim"], c["mode"])


def test_ffn_phase_matches_reference_adapter(golden):
    cases = golden("ffn_phase.pt")
    for c in cases:
        x, normalized = _rows(c["x"]), _rows(c["normalized"])
        time = c["time_mod"][0].float()
        mod = c["modulation"][0].float()
        n = c["n"]
        reuse = n > 0 and c["layer_id"] > 0
        indices = c["indices"] if reuse else None
        cache = _rows(c["cache"]) if (reuse and indices is not None) else None
        x_next, output, clean, _ = offn.ffn_block(
            x, None, normalized, mod, time, c["w_up"], c["b_up"], c["w_down"], c["b_down"], indices, cache,
            n if reuse else 0, 1e-6, ffn=offn.native_ffn)
        last = c["layer_id"] == c["num_layers"] - 1
        if last:
            # Last layer: the reference applies x + gate * output itself.
            assert torch.equal(x_next, _rows(c["hidden_states"])), "last-layer gate"
        else:
            # Middle layer: the residual is deferred; the golden output is the FFN output.
            assert torch.equal(_rows(c["hidden_states"]), x)
            ref_out = _rows(c["output"])
            assert torch.allclose(output, ref_out, atol=2e-2, rtol=2e-2)
            # Rows served from the cache are bit-exact copies.
            if cache is not None:
                kept = [r for r in range(n) if r not in set(indices.tolist())]
                assert torch.equal(output[kept], ref_out[kept])
        if c["token_outputs"] is not None and reuse:
            ref_clean = _rows(c["token_outputs"][0])
            assert clean.shape == ref_clean.shape
            assert torch.allclose(clean, ref_clean, atol=2e-2, rtol=2e-2)


def test_ffn_native_vs_prepared_semantics(golden):
    """The prepared (fused-epilogue) contract stays within the reference test's
    tolerance of the native path (WAMInfer/tests/test_prepared_ffn.py:32)."""
    for c in golden("ffn_phase.pt"):
        a = _rows(c["normalized"])
        native = offn.native_ffn(a, c["w_up"], c["b_up"], c["w_down"], c["b_down"])
        prepared = offn.prepared_ffn(a, c["w_up"], c["b_up"], c["w_down"], c["b_down"])
        torch.testing.assert_close(prepared, native, atol=5e-3, rtol=3e-2)


def test_token_reuse_known_answers(golden):
    g = golden("token_reuse.pt")
    assert g["small_first_count"] == 4
    assert g["small_second_count"] == 2
    assert g["small_indices"].tolist() == [1, 2, *range(4, 12)]
    # Restate the small case with the oracle.
    before = np.zeros((8, 8, 3), np.uint8)
    now = before.copy()
    now[:4, 4:] = 30
    mandatory = oreuse.mandatory_mask(now, before, 2, 2)
    assert mandatory.tolist() == g["small_second_mandatory"].tolist()
    assert oreuse.refresh_count(mandatory, (1, 2, 3, 4), 4) == 2
    current = np.ones((12, 8), np.float32)
    current[2:4] = 5
    idx = oreuse.token_indices(current[:4], np.ones((4, 8), np.float32), mandatory, 2, 4, 12)
    assert idx.tolist() == [1, 2, *range(4, 12)]


def test_rgb_threshold_boundary(golden):
    g = golden("token_reuse.pt")
    base = g["rgb_base"].numpy()
    for (dtype, change), (mask, count) in g["rgb_masks"].items():
        before = base.astype(dtype)
        current = (base.astype(np.float64) + change).astype(dtype)
        mandatory = oreuse.mandatory_mask(current, before, 12, 10)
        assert mandatory.tolist() == mask.tolist(), (dtype, change)
        assert oreuse.refresh_count(mandatory, (32, 64, 96, 120), 120) == count
    mandatory = oreuse.mandatory_mask(g["patch_change_image"].numpy(), base, 12, 10)
    assert mandatory.tolist() == g["patch_change_mandatory"].tolist()
    assert oreuse.refresh_count(mandatory, (32, 64, 96, 120), 120) == g["patch_change_count"]


def test_select_tokens_indices_bit_exact(golden):
    for s in golden("token_reuse.pt")["selections"]:
        now = s["features"][0].float().numpy()
        before = s["before"][0].float().numpy()
        idx = oreuse.token_indices(now, before, s["mandatory"].numpy(), s["count"], 120, s["seq"])
        assert idx.tolist() == s["indices"].tolist()


def test_motion_schedule(golden):
    full = golden("token_reuse.pt")["motion_full_steps"]
    for motion, steps in full.items():
        expected = [0, 3] if motion > 0.08 else [0, 3, 6, 9]
        assert steps == expected, motion


def test_select_tokens_near_ties(golden):
    """Constructed near-ties (tests/golden/make_near_ties.py): a group of rows
    with one float32 score but different exact ratios, rows 1 and 2 ulps above
    and 1 ulp below it, zero rows, mandatory rows; the cut placed inside each
    group.  The restated fixed-order sums give the reference's indices."""
    g = golden("near_ties.pt")
    now, before = g["now"].float().numpy(), g["before"].float().numpy()
    got_scores = oreuse.scores(now, before)
    assert got_scores.tolist() == g["scores"].tolist()
    labels = g["labels"]
    tie = [i for i, lab in enumerate(labels) if lab == "tie"]
    assert len({float(got_scores[i]) for i in tie}) == 1 and len(tie) == 10
    for lab, steps in (("plus1", 1), ("plus2", 2), ("minus1", -1)):
        rows = [i for i, x in enumerate(labels) if x == lab]
        assert all(got_scores[i] == np.float32(g["s0"] + steps * g["ulp"]) for i in rows), lab
    for case in g["cases"]:
        idx = oreuse.token_indices(now, before, case["mandatory"].numpy(), case["count"], 120, case["seq"])
        assert idx.tolist() == case["indices"].tolist(), case["name"]


def test_fixed_order_sum_is_exact_for_bf16_rows():
    """The fixed-order float64 accumulation equals the exact (math.fsum) sum
    rounded to float32 for bf16 rows of the benchmark's dimension."""
    import math

    rng = np.random.default_rng(5)
    for scale in (1e-3, 1.0, 100.0):
        a = torch.from_numpy(rng.standard_normal((8, 3072)) * scale).to(torch.bfloat16).float().numpy()
        b = torch.from_numpy(rng.standard_normal((8, 3072)) * scale).to(torch.bfloat16).float().numpy()
        terms = np.abs(a - b)
        got = oreuse._row_sums_fixed_order(terms)
        exact = np.array([math.fsum(map(float, row)) for row in terms]).astype(np.float32)
        assert got.tolist() == exact.tolist(), scale
