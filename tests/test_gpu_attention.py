"""GPU: the tcgen05 masked attention (``wam_ffn::masked_attention``) against
the fp32 oracle (``oracle/attention.py``) and the reference's own Triton
kernel (``wam_infer::masked_attention_mask_tiles_v4`` from baseline/_ref), on
the DiT's shapes: the joint video + action self-attention (392 x 392, no
mask), the video and action cross-attention to a padded 512-token context, the
reference's 513-token context with its prefix mask (``tail``), a strided query
taken from a packed QKV projection, and small ragged shapes with per-(batch,
head, query, key) masks including fully masked rows (zero output).  Tolerance:
the bf16-output rule of the other kernel tests (every element within 2e-2 or
one bf16 ulp of the reference value, mean relative error within 5e-3)."""

import pytest
import torch

from oracle import attention as oattn
from oracle import ffn as offn

pytestmark = pytest.mark.gpu


def _reference_triton():
    import sys
    from pathlib import Path

    sys.path.insert(0, str(Path(__file__).resolve().parents[1] / "baseline"))
    import reference_phase as rp

    if rp.missing(cuda=True):
        return None
    rp.import_reference(cuda=True)
    from WAMInfer import _triton_attention

    return _triton_attention.masked_attention


def _case(dev, seed, b, nq, nk, heads, mask_kind):
    g = torch.Generator(device=dev).manual_seed(seed)
    q = torch.randn(b, nq, heads * 128, device=dev, generator=g).bfloat16()
    k = torch.randn(b, nk, heads * 128, device=dev, generator=g).bfloat16()
    v = torch.randn(b, nk, heads * 128, device=dev, generator=g).bfloat16()
    mask = None
    if mask_kind == "context":  # padded prompt, shared by heads and queries (blocks.py:234-237)
        mask = torch.ones(b, 1, 1, nk, dtype=torch.bool, device=dev)
        mask[..., int(nk * 0.75):] = False
        if nk == 513:
            mask[..., 512] = True  # the extra context position stays
    elif mask_kind == "random":
        mask = torch.rand(b, heads, nq, nk, device=dev, generator=g) < 0.7
        mask[:, :, 0, :] = False  # an all-masked query row
    return q, k, v, mask


@pytest.mark.parametrize("b,nq,nk,heads,mask_kind,tail", [
    (1, 392, 392, 24, None, False),
    (1, 360, 512, 24, "context", False),
    (1, 32, 512, 24, "context", True),
    (1, 240, 513, 24, "context", True),
    (2, 100, 77, 2, "random", False),
    (1, 1, 1, 1, None, False),
    (1, 129, 130, 3, "random", False),
])
def test_masked_attention_vs_oracle_and_reference(cuda_device, b, nq, nk, heads, mask_kind, tail):
    from waminfer_b200.attention import masked_attention

    q, k, v, mask = _case(cuda_device, nq * 7 + nk, b, nq, nk, heads, mask_kind)
    out = masked_attention(q, k, v, mask, heads, tail)
    torch.cuda.synchronize()
    ref = oattn.masked_attention(q, k, v, mask, heads)
    ok, msg = offn.check_close(out, ref)
    print("oracle", (b, nq, nk, heads, mask_kind), msg)
    assert ok, msg
    if mask_kind == "random":
        assert torch.count_nonzero(out.view(b, nq, heads, 128)[:, 0]) == 0  # all-masked rows are zero
    triton = _reference_triton()
    if triton is not None:
        theirs = triton(q, k, v, mask, heads, tail=tail)
        torch.cuda.synchronize()
        ok, msg = offn.check_close(out, theirs.float())
        print("reference Triton", (b, nq, nk, heads, mask_kind), msg)
        assert ok, msg


def test_masked_attention_strided_query_from_packed_projection(cuda_device):
    """q, k, v as the reference takes them: chunks of one packed [392, 3 * 3072]
    QKV projection (blocks.py:204-208), i.e. rows 9216 elements apart."""
    from waminfer_b200.attention import masked_attention

    g = torch.Generator(device=cuda_device).manual_seed(11)
    qkv = torch.randn(1, 392, 3 * 3072, device=cuda_device, generator=g).bfloat16()
    q, k, v = qkv.chunk(3, dim=-1)
    out = masked_attention(q, k, v, None, 24)
    dense = masked_attention(q.contiguous(), k.contiguous(), v.contiguous(), None, 24)
    torch.cuda.synchronize()
    assert torch.equal(out, dense)
    ok, msg = offn.check_close(out, oattn.masked_attention(q, k, v, None, 24))
    assert ok, msg
