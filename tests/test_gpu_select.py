"""GPU: device token selection reproduces the reference's indices bit-exactly."""

from types import SimpleNamespace

import pytest
import torch

from oracle import reuse as oreuse

pytestmark = pytest.mark.gpu


def test_select_tokens_matches_reference_golden(cuda_device, golden):
    from waminfer_b200.approximation import select_tokens

    for s in golden("token_reuse.pt")["selections"]:
        n = 120
        features = torch.zeros(1, s["seq"], s["features"].shape[-1], dtype=torch.bfloat16, device=cuda_device)
        features[:, :n] = s["features"].to(cuda_device)
        reuse = dict(n=n, count=s["count"], mandatory=s["mandatory"].to(cuda_device),
                     features=s["before"].to(cuda_device))
        state = SimpleNamespace(extras=dict(token_reuse=reuse))
        select_tokens(state, features)
        assert state.extras["token_indices"].cpu().tolist() == s["indices"].tolist()
        assert torch.equal(state.extras["token_features"].cpu(), s["features"])


def test_select_tokens_known_answer(cuda_device):
    """WAMInfer/tests/test_approximation.py:12-29: mandatory row wins, equal
    scores resolve to the smaller index -> [1, 2, 4..11]."""
    from waminfer_b200.approximation import select_tokens

    previous = torch.ones(1, 4, 8, dtype=torch.bfloat16, device=cuda_device)
    current = torch.ones(1, 12, 8, dtype=torch.bfloat16, device=cuda_device)
    current[:, 2:4] = 5
    mandatory = torch.tensor([False, True, False, False], device=cuda_device)
    state = SimpleNamespace(extras=dict(token_reuse=dict(n=4, count=2, mandatory=mandatory, features=previous)))
    select_tokens(state, current)
    assert state.extras["token_indices"].tolist() == [1, 2, *range(4, 12)]


@pytest.mark.parametrize("count,seed", [(32, 0), (64, 1), (96, 2), (1, 3), (119, 4)])
def test_select_tokens_random_vs_oracle(cuda_device, count, seed):
    from waminfer_b200.approximation import select_rows

    g = torch.Generator().manual_seed(seed)
    before = torch.randn(120, 3072, generator=g).to(torch.bfloat16)
    now = (before.float() + torch.randn(120, 3072, generator=g) * torch.rand(120, 1, generator=g)).to(torch.bfloat16)
    mandatory = torch.rand(120, generator=g) < 0.05
    got = select_rows(now.to(cuda_device), before.to(cuda_device), mandatory, count, 392).cpu()
    ref = oreuse.token_indices(now.float().numpy(), before.float().numpy(), mandatory.numpy(), count, 120, 392)
    assert got.tolist() == ref.tolist()


def _lat():
    return dict(latents=torch.zeros(1, 4, 3, 24, 20))


def test_rgb_mandatory_device_matches_reference_golden(cuda_device, golden):
    """TokenReuse.begin with uint8 CUDA observations (device change test,
    wamffn_rgb_mandatory) gives the reference's masks and counts: the threshold
    boundary (+4.999999 / +5.0 / +5.000001 / +9 truncated to uint8), a partial
    patch change, and the reference's small known-answer case."""
    from waminfer_b200.approximation import TokenReuse

    g = golden("token_reuse.pt")
    base = g["rgb_base"]
    for change in (4.999999, 5.0, 5.000001, 9.0):
        history = TokenReuse((32, 64, 96, 120))
        _, observation = history.begin(base.to(cuda_device), _lat(), "task", (1, 2, 2))
        history.commit(observation, torch.empty(1, 120, 1), torch.empty(1, 1, 120, 1))
        current = (base.double() + change).to(torch.uint8).to(cuda_device)
        reuse, _ = history.begin(current, _lat(), "task", (1, 2, 2))
        mask, count = g["rgb_masks"][("uint8", change)]
        assert torch.equal(reuse["mandatory"].cpu(), mask), change
        assert reuse["count"] == count, change

    history = TokenReuse((32, 64, 96, 120))
    _, observation = history.begin(base.to(cuda_device), _lat(), "task", (1, 2, 2))
    history.commit(observation, torch.empty(1, 120, 1), torch.empty(1, 1, 120, 1))
    reuse, _ = history.begin(g["patch_change_image"].to(cuda_device), _lat(), "task", (1, 2, 2))
    assert torch.equal(reuse["mandatory"].cpu(), g["patch_change_mandatory"])
    assert reuse["count"] == g["patch_change_count"]

    history = TokenReuse((1, 2, 3, 4))
    inputs = dict(latents=torch.zeros(1, 4, 3, 4, 4))
    image = torch.zeros(8, 8, 3, dtype=torch.uint8, device=cuda_device)
    reuse, observation = history.begin(image, inputs, "task", (1, 2, 2))
    assert reuse["count"] == g["small_first_count"]
    history.commit(observation, torch.ones(1, 4, 8), torch.ones(1, 1, 4, 8))
    image[:4, 4:] = 30
    reuse, _ = history.begin(image, inputs, "task", (1, 2, 2))
    assert reuse["count"] == g["small_second_count"]
    assert torch.equal(reuse["mandatory"].cpu(), g["small_second_mandatory"])


def test_rgb_mandatory_device_threshold_and_random(cuda_device):
    """Patch sums of exactly 5 x 3072 - 1, 5 x 3072 and 5 x 3072 + 1 (means
    just below, at and above the threshold) and random observations against
    the oracle's float32 numpy test."""
    import numpy as np

    from waminfer_b200.approximation import TokenReuse

    before = np.zeros((384, 320, 3), dtype=np.uint8)
    now = np.full((384, 320, 3), 5, dtype=np.uint8)
    now[0, 0, 0] = 6      # patch 0: 15361 -> mandatory
    now[0, 32, 0] = 4     # patch 1: 15359 -> not
    now[32, 0, :] = 0     # patch 10: below
    now[33, 0, :] = 10    # patch 10: back to exactly 15360 -> not
    rng = np.random.default_rng(3)
    cases = [(now, before)]
    for scale in (3, 8, 12, 40):
        a = rng.integers(0, 256, (384, 320, 3), dtype=np.uint8)
        b = np.clip(a.astype(np.int32) + rng.integers(-scale, scale + 1, a.shape), 0, 255).astype(np.uint8)
        cases.append((a, b))
    for a, b in cases:
        got = TokenReuse.mandatory_rows_device(torch.from_numpy(a).to(cuda_device),
                                               torch.from_numpy(b).to(cuda_device), 12, 10)
        ref = oreuse.mandatory_mask(a, b, 12, 10)
        assert got.cpu().numpy().tolist() == ref.tolist()
    first = TokenReuse.mandatory_rows_device(torch.from_numpy(now).to(cuda_device),
                                             torch.from_numpy(before).to(cuda_device), 12, 10).cpu()
    assert first[0] and not first[1] and not first[10]
    with pytest.raises(ValueError, match="split"):
        TokenReuse.mandatory_rows_device(torch.zeros(385, 320, 3, dtype=torch.uint8, device=cuda_device),
                                         torch.zeros(385, 320, 3, dtype=torch.uint8, device=cuda_device), 12, 10)


def test_select_tokens_near_ties(cuda_device, golden):
    """Constructed near-ties (equal float32 scores with different exact
    ratios, rows 1-2 ulps apart, zero rows, mandatory rows; cut inside each
    group): the device indices equal the reference's (fixture made by its own
    select_tokens) and the oracle's."""
    from waminfer_b200.approximation import select_tokens

    g = golden("near_ties.pt")
    n = 120
    for case in g["cases"]:
        features = torch.zeros(1, case["seq"], g["now"].shape[-1], dtype=torch.bfloat16, device=cuda_device)
        features[0, :n] = g["now"].to(cuda_device)
        reuse = dict(n=n, count=case["count"], mandatory=case["mandatory"].to(cuda_device),
                     features=g["before"][None].to(cuda_device))
        state = SimpleNamespace(extras=dict(token_reuse=reuse))
        select_tokens(state, features)
        got = state.extras["token_indices"].cpu().tolist()
        assert got == case["indices"].tolist(), case["name"]
        ref = oreuse.token_indices(g["now"].float().numpy(), g["before"].float().numpy(), case["mandatory"].numpy(),
                                   case["count"], n, case["seq"])
        assert got == ref.tolist(), case["name"]


def test_select_tokens_vs_installed_reference_on_gpu(cuda_device, golden):
    """The reference's own select_tokens (the unmodified package in
    baseline/_ref) run on this GPU against the device kernel: the near-tie
    fixture and seeded random features at the capacity buckets."""
    import sys
    from pathlib import Path

    sys.path.insert(0, str(Path(__file__).resolve().parents[1] / "baseline"))
    import reference_phase as rp

    if rp.missing(cuda=False):
        pytest.skip(rp.missing(cuda=False))
    ref = rp.import_reference(cuda=False)
    from waminfer_b200.approximation import select_tokens

    g = golden("near_ties.pt")
    cases = [(g["now"], g["before"], c["mandatory"], c["count"], c["seq"]) for c in g["cases"]]
    gen = torch.Generator().manual_seed(77)
    for count in (32, 64, 96, 1, 119):
        before = torch.randn(120, 3072, generator=gen).to(torch.bfloat16)
        now = (before.float() + torch.randn(120, 3072, generator=gen) * torch.rand(120, 1, generator=gen)).to(
            torch.bfloat16)
        cases.append((now, before, torch.rand(120, generator=gen) < 0.05, count, 392))
    for now, before, mandatory, count, seq in cases:
        results = []
        for fn in (ref.approximation.select_tokens, select_tokens):
            features = torch.zeros(1, seq, now.shape[-1], dtype=torch.bfloat16, device=cuda_device)
            features[0, :120] = now.to(cuda_device)
            reuse = dict(n=120, count=count, mandatory=mandatory.to(cuda_device), features=before[None].to(cuda_device))
            state = SimpleNamespace(extras=dict(token_reuse=reuse))
            fn(state, features)
            results.append(state.extras["token_indices"].cpu().tolist())
        assert results[0] == results[1], count
