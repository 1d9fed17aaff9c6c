"""Modulated norm op (residual update + LayerNorm + adaLN) on libwamffn.

Mirror of the reference's ``wam_infer::modulated_norm`` Triton op
(``WAMInfer/_triton_inference.py:115-221``): same signature, same MODE
constants, same bf16 rounding points, batch 1, one CUDA thread block per row.
"""

from __future__ import annotations

import ctypes

import torch

from waminfer_b200 import _lib

SELF_INPUT = _lib.SELF_INPUT
SELF_RESIDUAL = _lib.SELF_RESIDUAL
CROSS_RESIDUAL = _lib.CROSS_RESIDUAL
FFN_RESIDUAL = _lib.FFN_RESIDUAL


def _ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


def time_row_stride(time: torch.Tensor) -> int:
    """Elements between per-token time rows; 0 when one row is shared
    (the reference's TS, ``_triton_inference.py:214``)."""
    return time.stride(1) if time.ndim == 4 and time.shape[1] != 1 else 0


def _check_modulation(name: str, t: torch.Tensor | None, dim: int) -> None:
    if t is None:
        return
    if t.dtype != torch.bfloat16 or t.shape[-2:] != (6, dim) or t.stride(-1) != 1 or t.stride(-2) != dim:
        raise ValueError(f"{name} must be bf16 with contiguous trailing [6, {dim}] rows")


@torch.library.custom_op("wam_ffn::modulated_norm", mutates_args=())
def modulated_norm(
    x: torch.Tensor,
    update: torch.Tensor | None,
    mod: torch.Tensor,
    previous: torch.Tensor | None,
    time: torch.Tensor,
    weight: torch.Tensor | None,
    bias: torch.Tensor | None,
    mode: int,
    eps: float,
) -> tuple[torch.Tensor, torch.Tensor]:
    """Returns the updated residual and the normalised input to the next GEMM.

    SELF_INPUT normalises the state; SELF_RESIDUAL adds the gated self-attention
    output and applies the affine LayerNorm; CROSS_RESIDUAL adds the
    cross-attention output and modulates with the FFN shift/scale slots;
    FFN_RESIDUAL folds the previous block's gated FFN output.
    """
    if x.dim() != 3 or x.shape[0] != 1:
        raise ValueError("modulated_norm expects x of shape [1, rows, dim] (batch 1)")
    rows, dim = x.shape[1], x.shape[2]
    if x.dtype != torch.bfloat16 or x.stride(2) != 1:
        raise ValueError("x must be bf16 with a contiguous last dimension")
    if update is not None and (update.dtype != torch.bfloat16 or update.stride(-1) != 1):
        raise ValueError("update must be bf16 with a contiguous last dimension")
    _check_modulation("mod", mod, dim)
    _check_modulation("previous", previous, dim)
    _check_modulation("time", time, dim)
    y = torch.empty(x.shape, dtype=x.dtype, device=x.device)
    norm = torch.empty(x.shape, dtype=x.dtype, device=x.device)
    args = _lib.NormArgs(
        x=x.data_ptr(),
        x_stride=x.stride(1),
        update=_ptr(update),
        update_stride=0 if update is None else update.stride(1),
        mod=mod.data_ptr(),
        previous=_ptr(previous),
        time=time.data_ptr(),
        time_stride=time_row_stride(time),
        weight=_ptr(weight),
        bias=_ptr(bias),
        y=y.data_ptr(),
        norm=norm.data_ptr(),
        rows=rows,
        dim=dim,
        mode=int(mode),
        eps=float(eps),
    )
    with torch.cuda.device(x.device):
        stream = torch.cuda.current_stream(x.device).cuda_stream
        _lib.check(_lib.lib().wamffn_modulated_norm(stream, ctypes.byref(args)))
    return y, norm


@modulated_norm.register_fake
def _fake_norm(x, update, mod, previous, time, weight, bias, mode, eps):
    return torch.empty_like(x), torch.empty_like(x)
