"""GPU: attention-side projections on the library's GEMM engine
(``waminfer_b200/projections.py``) against the fp32 oracle, the reference's
packing rule, the unprepared-geometry fallback and weight-change refresh."""

from types import SimpleNamespace

import pytest
import torch
import torch.nn.functional as F

from oracle import ffn as offn

pytestmark = pytest.mark.gpu

D = 3072


def _block(device, g):
    def linear():
        layer = torch.nn.Linear(D, D, device=device, dtype=torch.bfloat16)
        with torch.no_grad():
            layer.weight.copy_(torch.randn(D, D, device=device, generator=g) * 0.02)
            layer.bias.copy_(torch.randn(D, device=device, generator=g) * 0.01)
        return layer.eval()

    self_attn = SimpleNamespace(q=linear(), k=linear(), v=linear(), o=linear(), training=False)
    cross_attn = SimpleNamespace(q=linear(), o=linear(), training=False)
    mod = (torch.randn(1, 6, D, device=device, generator=g) * 0.1).to(torch.bfloat16)
    return SimpleNamespace(self_attn=self_attn, cross_attn=cross_attn, modulation=mod)


@pytest.fixture(scope="module")
def backbone(cuda_device):
    g = torch.Generator(device=cuda_device).manual_seed(61)
    blocks = [_block(cuda_device, g) for _ in range(2)]
    return SimpleNamespace(dit=SimpleNamespace(blocks=blocks), training=False)


def _ref_linear(x, weight, bias):
    return offn.bf16(x.float() @ weight.float().T + bias.float())


@pytest.mark.parametrize("rows", [392, 240])
def test_projections_follow_oracle(cuda_device, backbone, rows):
    from waminfer_b200.projections import PROJECTIONS, PreparedProjections, packed_projection

    proj = PreparedProjections(backbone)
    with torch.no_grad():
        assert proj.prepare(rows=(rows,))
        g = torch.Generator(device=cuda_device).manual_seed(rows)
        x = torch.randn(1, rows, D, device=cuda_device, generator=g).to(torch.bfloat16)
        for layer_id, block in enumerate(backbone.dit.blocks):
            for kind, (attr, names) in PROJECTIONS.items():
                out = getattr(proj, kind)(layer_id, x)
                weight, bias, _ = packed_projection(getattr(block, attr), names)
                assert out.shape == (1, rows, weight.shape[0])
                ok, msg = offn.check_close(out[0], _ref_linear(x[0], weight, bias))
                assert ok, f"layer {layer_id} {kind}: {msg}"
        # q, k, v are the three thirds of the packed projection, as in blocks.py:207
        q, k, v = proj.qkv(0, x).chunk(3, dim=-1)
        ok, msg = offn.check_close(k[0], _ref_linear(x[0], backbone.dit.blocks[0].self_attn.k.weight,
                                                     backbone.dit.blocks[0].self_attn.k.bias))
        assert ok, msg
        assert not proj.prepare(rows=(rows,))  # nothing changed
    proj.close()


def test_unprepared_rows_fall_back_and_weight_changes_refresh(cuda_device, backbone):
    from waminfer_b200.projections import PreparedProjections

    proj = PreparedProjections(backbone)
    block = backbone.dit.blocks[1]
    with torch.no_grad():
        proj.prepare(rows=(128,))
        x = torch.randn(1, 100, D, device=cuda_device).to(torch.bfloat16)
        assert torch.equal(proj.self_out(1, x), F.linear(x, block.self_attn.o.weight, block.self_attn.o.bias))
        x = torch.randn(1, 128, D, device=cuda_device).to(torch.bfloat16)
        before = proj.cross_out(1, x)
        block.cross_attn.o.weight.mul_(2.0)  # bumps the parameter version: the packed copy is stale
        assert proj.prepare(rows=(128,))
        after = proj.cross_out(1, x)
        ref = _ref_linear(x[0], block.cross_attn.o.weight, block.cross_attn.o.bias)
        ok, msg = offn.check_close(after[0], ref)
        assert ok, msg
        assert not torch.equal(before, after)
        block.cross_attn.o.weight.mul_(0.5)
    proj.close()


@pytest.mark.parametrize("mode", [0, 3])
def test_pre_attention_norm_and_qkv(cuda_device, backbone, mode):
    """The pre-attention step of blocks.py:189-208 without Q/K RMSNorm + RoPE:
    modulated_norm (SELF_INPUT, or FFN_RESIDUAL folding the previous FFN) and
    the packed QKV projection, against the oracle."""
    from waminfer_b200.norm import modulated_norm
    from waminfer_b200.projections import PreparedProjections, packed_projection

    rows = 392
    g = torch.Generator(device=cuda_device).manual_seed(70 + mode)
    x = torch.randn(1, rows, D, device=cuda_device, generator=g).to(torch.bfloat16)
    update = torch.randn(1, rows, D, device=cuda_device, generator=g).to(torch.bfloat16) if mode == 3 else None
    time = (torch.randn(1, rows, 6, D, device=cuda_device, generator=g) * 0.1).to(torch.bfloat16)
    block, previous = backbone.dit.blocks[1], backbone.dit.blocks[0].modulation
    proj = PreparedProjections(backbone)
    with torch.no_grad():
        proj.prepare(rows=(rows,))
        y, normalized = modulated_norm(x, update, block.modulation, previous if mode == 3 else None, time, None, None,
                                       mode, 1e-6)
        projected = proj.qkv(1, normalized)
    y_ref, n_ref = offn.modulated_norm(x[0], None if update is None else update[0], block.modulation[0],
                                       previous[0] if mode == 3 else None, time[0], None, None, mode, 1e-6)
    assert torch.equal(y[0].float().cpu(), y_ref.cpu())
    with torch.no_grad():
        weight, bias, _ = packed_projection(block.self_attn, ("q", "k", "v"))
    ok, msg = offn.check_close(projected[0], _ref_linear(normalized[0], weight, bias))
    assert ok, msg
    ok, msg = offn.check_close(projected[0], _ref_linear(n_ref.to(cuda_device), weight, bias))
    assert ok, f"against the oracle's norm: {msg}"
    proj.close()
