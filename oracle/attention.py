"""torch-fp32 restatement of the reference's attention ops (test infrastructure only).

``masked_attention`` restates the masked op; ``joint_first_frame_attention``
and ``current_frame_attention`` restate the other two layouts as that
function over a built mask / the concatenated segments.

Follows ``_attention_kernel`` (WAMInfer/_triton_attention.py:18-107): scores
``q . k`` scaled by D^-0.5 log2(e); masked keys at -inf; exp2 against the row
maximum (taken as 0 when every key is masked); probabilities rounded to bf16
for the value product while the normaliser sums the fp32 probabilities; the
product divided by the normaliser (1 when it is 0, giving a zero row).  The
reference runs this per key block with a running maximum; one block over all
keys is the same function up to where the bf16 rounding of the probabilities
happens (relative to the running or the final maximum).
"""

from __future__ import annotations

import math

import torch


def masked_attention(q, k, v, mask, heads: int) -> torch.Tensor:
    """q [B, Nq, H*D], k / v [B, Nk, H*D], mask bool broadcastable to [B, H, Nq, Nk]
    or None.  Returns fp32 [B, Nq, H*D]."""
    b, nq, hidden = q.shape
    nk = k.shape[1]
    d = hidden // heads
    qh = q.float().view(b, nq, heads, d).transpose(1, 2)
    kh = k.float().view(b, nk, heads, d).transpose(1, 2)
    vh = v.float().view(b, nk, heads, d).transpose(1, 2)
    scores = (qh @ kh.transpose(-1, -2)) * float(d ** -0.5 * 1.4426950408889634)
    if mask is not None:
        scores = scores.masked_fill(~torch.broadcast_to(mask, scores.shape), -math.inf)
    top = scores.amax(-1, keepdim=True)
    top = torch.where(torch.isinf(top) & (top < 0), torch.zeros_like(top), top)
    p = torch.exp2(scores - top)
    norm = p.sum(-1, keepdim=True)
    out = (p.to(torch.bfloat16).float() @ vh) / torch.where(norm > 0, norm, torch.ones_like(norm))
    return out.transpose(1, 2).reshape(b, nq, hidden)


def joint_first_frame_attention(q, k, v, first: int, heads: int) -> torch.Tensor:
    """``_joint_attention`` (WAMInfer/_triton_attention.py:267-313): rows
    [0, first) attend keys [0, first), rows [first, count) attend every key.
    fp32 [B, count, H*D]."""
    count = q.shape[1]
    rows = torch.arange(count, device=q.device)[:, None]
    keys = torch.arange(count, device=q.device)[None, :]
    mask = keys < torch.where(rows < first, first, count)
    return masked_attention(q, k, v, mask, heads)


def current_frame_attention(qv, qa, ck, kv, ka, cv, vv, va, heads: int):
    """``_split_attention_kernel`` (WAMInfer/_triton_attention.py:337-426): the
    queries qv ++ qa against the keys ck ++ kv ++ ka (values cv ++ vv ++ va),
    unmasked; returns fp32 (ov, oa)."""
    out = masked_attention(torch.cat((qv, qa), 1), torch.cat((ck, kv, ka), 1), torch.cat((cv, vv, va), 1), None,
                           heads)
    return out[:, :qv.shape[1]], out[:, qv.shape[1]:]
