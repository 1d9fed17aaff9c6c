"""The DiT's attention ops on libwamffn (tcgen05, sm_100a).

Mirrors of the reference's three Triton ops (``WAMInfer/_triton_attention.py``),
same signatures and arithmetic (exp2 softmax of scores scaled by D^-0.5 log2 e,
bf16 probabilities in the value product, fp32 normaliser, all-masked rows
output zeros), head dim 128 (the DiT's 24 x 128 heads):

* ``masked_attention(q, k, v, mask, heads, tail=False)`` — op
  ``wam_infer::masked_attention_mask_tiles_v4`` (:238-263).  ``tail`` selects a
  tiling of the 513-token context in the reference and changes no value; it is
  accepted and ignored.
* ``joint_first_frame_attention(q, k, v, video, first, heads)`` — op
  ``wam_infer::joint_first_frame_attention_v2`` (:327-334): the joint video +
  action self-attention whose first ``first`` rows (the clean first frame)
  see only each other.
* ``current_frame_attention(qv, qa, ck, kv, ka, cv, vv, va, heads)`` — op
  ``wam_infer::current_frame_attention_v1`` (:429-484): video and action
  queries against a cached prefix plus the current video and action keys,
  with nothing concatenated.

Each takes an extra ``key_split`` (0 = chosen from the grid size; 1, 2, 4):
the CTAs that share one 128-query tile's keys.
"""

from __future__ import annotations

import ctypes

import torch

from waminfer_b200 import _lib

HEAD_DIM = 128


def _rows(t: torch.Tensor, name: str) -> torch.Tensor:
    """A [batch, rows, width] tensor whose rows sit at one stride across batches."""
    if t.stride(2) != 1 or t.stride(1) % 8 or t.stride(0) != t.shape[1] * t.stride(1) or t.data_ptr() % 16:
        t = t.contiguous()
    return t


@torch.library.custom_op("wam_ffn::masked_attention", mutates_args=())
def masked_attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, mask: torch.Tensor | None, heads: int,
                     tail: bool = False, key_split: int = 0) -> torch.Tensor:
    """out[b, q, h] = softmax_k(q . k / sqrt(128), masked) . v, [batch, nq, heads * 128] bf16.
    mask: bool, broadcastable to [batch, heads, nq, nk] (False = masked), or None.
    key_split: CTAs sharing a query tile's keys (0 = chosen from the grid size; 1, 2, 4)."""
    if q.dim() != 3 or k.dim() != 3 or v.dim() != 3:
        raise ValueError("q, k and v must be [batch, rows, heads * head_dim]")
    batch, nq, hidden = q.shape
    nk = k.shape[1]
    if hidden != heads * HEAD_DIM or k.shape[2] != hidden or v.shape[2] != hidden or k.shape[:2] != v.shape[:2]:
        raise ValueError(f"shapes {tuple(q.shape)}, {tuple(k.shape)}, {tuple(v.shape)} do not hold {heads} heads of "
                         f"{HEAD_DIM}")
    if q.dtype != torch.bfloat16 or k.dtype != torch.bfloat16 or v.dtype != torch.bfloat16:
        raise ValueError("q, k and v must be bf16")
    if not (q.is_cuda and k.is_cuda and v.is_cuda):
        raise ValueError("q, k and v must be CUDA tensors")
    q, k, v = _rows(q, "q"), _rows(k, "k"), _rows(v, "v")
    strides = (0, 0, 0, 0)
    if mask is not None:
        if mask.dtype != torch.bool:
            raise ValueError("mask must be bool (True keeps a key)")
        mask = torch.broadcast_to(mask, (batch, heads, nq, nk))
        strides = mask.stride()
    out = torch.empty(q.shape, dtype=q.dtype, device=q.device)
    args = _lib.AttentionArgs(
        q=q.data_ptr(), q_row_stride=q.stride(1), q_batch_stride=q.stride(0),
        k=k.data_ptr(), k_row_stride=k.stride(1), k_batch_stride=k.stride(0),
        v=v.data_ptr(), v_row_stride=v.stride(1), v_batch_stride=v.stride(0),
        mask=None if mask is None else mask.data_ptr(), mask_strides=(ctypes.c_int64 * 4)(*strides),
        out=out.data_ptr(), status=None,
        batch=batch, nq=nq, nk=nk, heads=heads, head_dim=HEAD_DIM, key_split=key_split)
    with torch.cuda.device(q.device):
        stream = torch.cuda.current_stream(q.device).cuda_stream
        _lib.check(_lib.lib().wamffn_masked_attention(stream, ctypes.byref(args)))
    return out


@masked_attention.register_fake
def _fake_attention(q, k, v, mask, heads, tail=False, key_split=0):
    return torch.empty_like(q)


def _view(t: torch.Tensor, name: str) -> _lib.RowsView:
    if t.dim() != 3:
        raise ValueError(f"{name} must be [batch, rows, heads * head_dim]")
    if t.dtype != torch.bfloat16 or not t.is_cuda:
        raise ValueError(f"{name} must be a bf16 CUDA tensor")
    return _lib.RowsView(data=t.data_ptr(), row_stride=t.stride(1), batch_stride=t.stride(0))


def _check_width(heads: int, **tensors: torch.Tensor) -> None:
    for name, t in tensors.items():
        if t.dim() != 3 or t.shape[2] != heads * HEAD_DIM:
            raise ValueError(f"{name} {tuple(t.shape)} does not hold {heads} heads of {HEAD_DIM}")


@torch.library.custom_op("wam_ffn::joint_first_frame_attention", mutates_args=())
def joint_first_frame_attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, video: int, first: int, heads: int,
                                key_split: int = 0) -> torch.Tensor:
    """Joint video + action self-attention, [batch, count, heads * 128] each:
    query rows [0, first) attend keys [0, first), the others attend all keys.
    ``video`` (the video row count) is part of the reference's signature and
    changes nothing."""
    _check_width(heads, q=q, k=k, v=v)
    if k.shape[:2] != q.shape[:2] or v.shape[:2] != q.shape[:2]:
        raise ValueError(f"q, k, v shapes differ: {tuple(q.shape)}, {tuple(k.shape)}, {tuple(v.shape)}")
    batch, count, _ = q.shape
    q, k, v = _rows(q, "q"), _rows(k, "k"), _rows(v, "v")
    out = torch.empty(q.shape, dtype=q.dtype, device=q.device)
    args = _lib.JointAttentionArgs(q=_view(q, "q"), k=_view(k, "k"), v=_view(v, "v"), out=out.data_ptr(),
                                   status=None, batch=batch, count=count, video=video, first=first, heads=heads,
                                   head_dim=HEAD_DIM, key_split=key_split)
    with torch.cuda.device(q.device):
        stream = torch.cuda.current_stream(q.device).cuda_stream
        _lib.check(_lib.lib().wamffn_joint_first_frame_attention(stream, ctypes.byref(args)))
    return out


@joint_first_frame_attention.register_fake
def _fake_joint(q, k, v, video, first, heads, key_split=0):
    return torch.empty_like(q)


@torch.library.custom_op("wam_ffn::current_frame_attention", mutates_args=())
def current_frame_attention(qv: torch.Tensor, qa: torch.Tensor, ck: torch.Tensor, kv: torch.Tensor,
                            ka: torch.Tensor, cv: torch.Tensor, vv: torch.Tensor, va: torch.Tensor, heads: int,
                            key_split: int = 0) -> tuple[torch.Tensor, torch.Tensor]:
    """Video rows qv [batch, nv, .] and action rows qa [batch, na, .] attend
    ck ++ kv ++ ka (values cv ++ vv ++ va), unmasked; returns (ov, oa)."""
    _check_width(heads, qv=qv, qa=qa, ck=ck, kv=kv, ka=ka, cv=cv, vv=vv, va=va)
    batch, nv, _ = qv.shape
    na, nc = qa.shape[1], ck.shape[1]
    for name, t, rows in (("qa", qa, na), ("kv", kv, nv), ("ka", ka, na), ("cv", cv, nc), ("vv", vv, nv),
                          ("va", va, na)):
        if t.shape[0] != batch or t.shape[1] != rows:
            raise ValueError(f"{name} {tuple(t.shape)}: expected [{batch}, {rows}, {heads * HEAD_DIM}]")
    views = {name: _rows(t, name) for name, t in
             (("qv", qv), ("qa", qa), ("ck", ck), ("kv", kv), ("ka", ka), ("cv", cv), ("vv", vv), ("va", va))}
    ov = torch.empty(qv.shape, dtype=qv.dtype, device=qv.device)
    oa = torch.empty(qa.shape, dtype=qa.dtype, device=qa.device)
    args = _lib.CurrentFrameArgs(**{name: _view(t, name) for name, t in views.items()}, ov=ov.data_ptr(),
                                 oa=oa.data_ptr(), status=None, batch=batch, nc=nc, nv=nv, na=na, heads=heads,
                                 head_dim=HEAD_DIM, key_split=key_split)
    with torch.cuda.device(qv.device):
        stream = torch.cuda.current_stream(qv.device).cuda_stream
        _lib.check(_lib.lib().wamffn_current_frame_attention(stream, ctypes.byref(args)))
    return ov, oa


@current_frame_attention.register_fake
def _fake_current(qv, qa, ck, kv, ka, cv, vv, va, heads, key_split=0):
    return torch.empty_like(qv), torch.empty_like(qa)
