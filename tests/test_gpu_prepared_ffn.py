"""GPU: the PreparedFFN / VideoFFN drop-ins keep the reference's contract.

Re-expresses WAMInfer/tests/test_prepared_ffn.py:12-58 (plan ownership,
native fallback for an unprepared row count, prepared vs native tolerance,
bit-exact CUDA graph replay, weight mutation -> re-prepare, close releases
plans) and WAMInfer/tests/test_approximation.py:139-165 (the reuse FFN runs
length - n + count rows, non-selected cache rows are kept bit-exactly and the
residual is x + gate * output).
"""

from types import SimpleNamespace

import pytest
import torch

pytestmark = pytest.mark.gpu


@torch.no_grad()
def test_prepared_ffn_contract(cuda_device):
    from waminfer_b200.ffn import _PLANS, PreparedFFN

    torch.manual_seed(24)
    ffn = (
        torch.nn.Sequential(torch.nn.Linear(128, 512), torch.nn.GELU(approximate="tanh"), torch.nn.Linear(512, 128))
        .to(cuda_device)
        .bfloat16()
        .eval()
    )
    backbone = SimpleNamespace(training=False, dit=SimpleNamespace(blocks=[SimpleNamespace(ffn=ffn)]))
    before = set(_PLANS)
    first, second = PreparedFFN(backbone), PreparedFFN(backbone)
    try:
        assert first.prepare((16,))
        second.prepare((16,))
        assert set(first.keys.values()).isdisjoint(second.keys.values())
        x = torch.randn(16, 128, device=cuda_device, dtype=torch.bfloat16)
        merged = torch.cat((x, x), dim=0)
        torch.testing.assert_close(first.forward(0, merged), ffn(merged), atol=0, rtol=0)  # native fallback
        expected = ffn(x)
        actual = first.forward(0, x)
        torch.testing.assert_close(actual, expected, atol=0.005, rtol=0.03)
        torch.testing.assert_close(second.forward(0, x), expected, atol=0.005, rtol=0.03)
        stream = torch.cuda.Stream()
        stream.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(stream):
            for _ in range(3):
                first.forward(0, x)
        torch.cuda.current_stream().wait_stream(stream)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            captured = first.forward(0, x)
        graph.replay()
        torch.testing.assert_close(captured, actual, atol=0, rtol=0)
        graph.reset()
        ffn[0].weight.add_(0.1)
        assert first.prepare((16,))
        updated = first.forward(0, x)
        assert not torch.equal(updated, actual)
        torch.testing.assert_close(updated, ffn(x), atol=0.01, rtol=0.04)
        assert not first.prepare((16,))
        # An empty input is an unprepared row count: the native FFN, like the reference.
        empty = torch.empty(1, 0, 128, device=cuda_device, dtype=torch.bfloat16)
        assert first.forward(0, empty).shape == (1, 0, 128)
        first.close()
        assert set(_PLANS) == before | set(second.keys.values())
    finally:
        torch.cuda.synchronize()
        first.close()
        second.close()
    assert set(_PLANS) == before


@torch.no_grad()
def test_prepared_ffn_full_size_graph_replay(cuda_device):
    """The d=3072 / h=14336 geometry at every reference row bucket, captured in
    one CUDA graph and replayed bit-exactly."""
    from waminfer_b200.ffn import PreparedFFN

    torch.manual_seed(3)
    ffn = (
        torch.nn.Sequential(torch.nn.Linear(3072, 14336), torch.nn.GELU(approximate="tanh"), torch.nn.Linear(14336, 3072))
        .to(cuda_device)
        .bfloat16()
        .eval()
    )
    backbone = SimpleNamespace(training=False, dit=SimpleNamespace(blocks=[SimpleNamespace(ffn=ffn)]))
    rows = (360, 240, 272, 304, 336)
    prepared = PreparedFFN(backbone)
    try:
        prepared.prepare(rows)
        xs = [torch.randn(1, m, 3072, device=cuda_device, dtype=torch.bfloat16) for m in rows]
        eager = [prepared.forward(0, x) for x in xs]
        for x, out in zip(xs, eager):
            ref = ffn(x)  # native path: rounds before GELU, so compare with the reference test's tolerance
            torch.testing.assert_close(out, ref, atol=0.02, rtol=0.05)
        stream = torch.cuda.Stream()
        stream.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(stream):
            for x in xs:
                prepared.forward(0, x)
        torch.cuda.current_stream().wait_stream(stream)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            captured = [prepared.forward(0, x) for x in xs]
        graph.replay()
        torch.cuda.synchronize()
        for a, b in zip(captured, eager):
            assert torch.equal(a, b)
        graph.reset()
    finally:
        torch.cuda.synchronize()
        prepared.close()


def _backbone(device, layers=3, d=256, h=1024):
    blocks = []
    for _ in range(layers):
        ffn = torch.nn.Sequential(torch.nn.Linear(d, h), torch.nn.GELU(approximate="tanh"), torch.nn.Linear(h, d))
        ffn = ffn.to(device).bfloat16().eval()
        modulation = (torch.randn(1, 6, d, device=device) * 0.1).bfloat16()
        blocks.append(SimpleNamespace(ffn=ffn, modulation=modulation,
                                      norm2=SimpleNamespace(eps=1e-6)))
    return SimpleNamespace(training=False, dit=SimpleNamespace(blocks=blocks), num_layers=layers)


@torch.no_grad()
def test_video_ffn_reuse_contract(cuda_device):
    """test_approximation.py:139-165 re-expressed for the fused phase."""
    from waminfer_b200.blocks import VideoFFN

    torch.manual_seed(0)
    backbone = _backbone(cuda_device)
    phase = VideoFFN(backbone, max_rows=64, max_seq=64)
    n, count, length, dim = 4, 2, 12, 256
    x = torch.randn(1, length, dim, device=cuda_device, dtype=torch.bfloat16)
    normalized = torch.randn_like(x)
    old = torch.randn(1, n, dim, device=cuda_device, dtype=torch.bfloat16)
    indices = torch.tensor([0, 3, *range(n, length)], device=cuda_device)
    time_mod = torch.randn(1, length, 6, dim, device=cuda_device, dtype=x.dtype)
    state = SimpleNamespace(
        time_mod=time_mod,
        extras=dict(token_reuse=dict(n=n, count=count, cache=(None, old)), token_indices=indices,
                    token_outputs=[]),
    )
    phase.ffn_at_layer_for_compile(2, state, normalized, x)
    assert phase.plan.configuration(length - n + count)["up"]["token_pad"] == 16
    clean = state.extras["token_outputs"][0]
    torch.testing.assert_close(clean[:, 1:3], old[:, 1:3], atol=0, rtol=0)
    block = backbone.dit.blocks[2]
    output = block.ffn(normalized)
    output[:, :n] = clean
    gate = (block.modulation + time_mod)[:, :, 5]
    torch.testing.assert_close(state.hidden_states, x + gate * output, atol=0.02, rtol=0.02)
    phase.close()
