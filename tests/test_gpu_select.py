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
