"""Masked multi-head attention op on libwamffn (tcgen05, sm_100a).

Mirror of the reference's ``wam_infer::masked_attention_mask_tiles_v4`` Triton
op (``WAMInfer/_triton_attention.py:238-263``): same signature
``masked_attention(q, k, v, mask, heads, tail=False)``, same arithmetic (exp2
softmax of scores scaled by D^-0.5 log2 e, bf16 probabilities in the value
product, fp32 normaliser, all-masked rows output zeros).  ``tail`` selects a
tiling of the 513-token context in the reference and changes no value; it is
accepted and ignored.  Head dim 128 (the DiT's 24 x 128 heads).
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
                     tail: bool = False) -> torch.Tensor:
    """out[b, q, h] = softmax_k(q . k / sqrt(128), masked) . v, [batch, nq, heads * 128] bf16.
    mask: bool, broadcastable to [batch, heads, nq, nk] (False = masked), or None."""
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
        batch=batch, nq=nq, nk=nk, heads=heads, head_dim=HEAD_DIM)
    with torch.cuda.device(q.device):
        stream = torch.cuda.current_stream(q.device).cuda_stream
        _lib.check(_lib.lib().wamffn_masked_attention(stream, ctypes.byref(args)))
    return out


@masked_attention.register_fake
def _fake_attention(q, k, v, mask, heads, tail=False):
    return torch.empty_like(q)
