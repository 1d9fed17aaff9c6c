"""CPU: the attention oracle (``oracle/attention.py``) against a direct float64
evaluation of softmax(q k^T / sqrt(D)) v per query row, on small seeded
cases of the three layouts (masked with an all-masked row, first-frame
causal, cached prefix).  The oracle rounds the probabilities to bf16 before
the value product, as the reference does, so the comparison allows that
rounding: |difference| within 2^-8 of the row's value scale."""

import math

import torch

from oracle import attention as oattn


def _direct(q, k, v, allowed, heads):
    """float64 softmax attention; allowed(i, j) -> bool; all-masked rows 0."""
    b, nq, hidden = q.shape
    d = hidden // heads
    out = torch.zeros(b, nq, hidden, dtype=torch.float64)
    for bi in range(b):
        for h in range(heads):
            sl = slice(h * d, (h + 1) * d)
            for i in range(nq):
                keys = [j for j in range(k.shape[1]) if allowed(bi, h, i, j)]
                if not keys:
                    continue
                s = torch.tensor([float(q[bi, i, sl].double() @ k[bi, j, sl].double()) / math.sqrt(d) for j in keys],
                                 dtype=torch.float64)
                p = torch.softmax(s, 0)
                out[bi, i, sl] = (p[:, None] * v[bi, keys, sl].double()).sum(0)
    return out


def _close(got, exp):
    scale = exp.abs().amax().item() + 1e-30
    assert (got.double() - exp).abs().max().item() <= scale * 2 ** -8


def _rand(g, *shape):
    return torch.randn(*shape, generator=g).bfloat16()


def test_masked_oracle_against_direct_softmax():
    g = torch.Generator().manual_seed(0)
    heads, d = 2, 16
    q, k, v = _rand(g, 2, 5, heads * d), _rand(g, 2, 9, heads * d), _rand(g, 2, 9, heads * d)
    mask = torch.rand(2, heads, 5, 9, generator=g) < 0.6
    mask[:, :, 0] = False  # an all-masked query row outputs zeros
    got = oattn.masked_attention(q, k, v, mask, heads)
    _close(got, _direct(q, k, v, lambda b, h, i, j: bool(mask[b, h, i, j]), heads))
    assert torch.count_nonzero(got[:, 0]) == 0


def test_joint_first_frame_oracle_against_direct_softmax():
    g = torch.Generator().manual_seed(1)
    heads, d, count, first = 2, 16, 11, 4
    q, k, v = (_rand(g, 1, count, heads * d) for _ in range(3))
    got = oattn.joint_first_frame_attention(q, k, v, first, heads)
    _close(got, _direct(q, k, v, lambda b, h, i, j: j < (first if i < first else count), heads))


def test_current_frame_oracle_against_direct_softmax():
    g = torch.Generator().manual_seed(2)
    heads, d, nc, nv, na = 2, 16, 3, 6, 2
    qv, qa = _rand(g, 1, nv, heads * d), _rand(g, 1, na, heads * d)
    ck, kv, ka = _rand(g, 1, nc, heads * d), _rand(g, 1, nv, heads * d), _rand(g, 1, na, heads * d)
    cv, vv, va = _rand(g, 1, nc, heads * d), _rand(g, 1, nv, heads * d), _rand(g, 1, na, heads * d)
    ov, oa = oattn.current_frame_attention(qv, qa, ck, kv, ka, cv, vv, va, heads)
    full = _direct(torch.cat((qv, qa), 1), torch.cat((ck, kv, ka), 1), torch.cat((cv, vv, va), 1),
                   lambda b, h, i, j: True, heads)
    _close(ov, full[:, :nv])
    _close(oa, full[:, nv:])
