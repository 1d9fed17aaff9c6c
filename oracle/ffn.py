"""torch-fp32 CPU restatement of the reference FFN path (test infrastructure only).

Tensors are fp32 holding bf16-representable values; ``bf16()`` marks each point
where the reference rounds to bf16.  Row layout: x [S, d]; mod [6, d];
time [S, 6, d] (per token) or [6, d] (shared).
"""

from __future__ import annotations

import torch
import torch.nn.functional as F

SELF_INPUT, SELF_RESIDUAL, CROSS_RESIDUAL, FFN_RESIDUAL = 0, 1, 2, 3


def bf16(t: torch.Tensor) -> torch.Tensor:
    """Round to bfloat16 (nearest even) and widen back to fp32."""
    return t.to(torch.bfloat16).to(torch.float32)


def modulation(mod: torch.Tensor, time: torch.Tensor, slot: int) -> torch.Tensor:
    """bf16(mod[slot] + time[row, slot]) -- WAMInfer/_triton_inference.py:123-127."""
    t = time[..., slot, :]
    return bf16(mod[slot].float() + t.float())


def modulated_norm(x, update, mod, previous, time, weight, bias, mode: int, eps: float):
    """WAMInfer/_triton_inference.py:149-176 (one row per Triton program).

    Returns (y, norm), both bf16-valued fp32 [S, d].
    """
    x = x.float()
    if mode > 0 and update is not None:  # the fused block allows no update (FFN slots on x itself)
        u = update.float()
        if mode == SELF_RESIDUAL:
            u = bf16(modulation(mod, time, 2) * u)          # :155-157
        elif mode == FFN_RESIDUAL:
            u = bf16(modulation(previous, time, 5) * u)     # :158-160
        x = bf16(x + u)                                     # :161
    d = x.shape[-1]
    centered = x - x.sum(-1, keepdim=True) / d              # :162
    variance = (centered * centered).sum(-1, keepdim=True) / d  # :163
    n = centered * torch.rsqrt(variance + eps)              # :164
    if mode == SELF_RESIDUAL:
        n = n * weight.float() + bias.float()               # :165-168
    else:
        n = bf16(n)                                         # :170
        shift = modulation(mod, time, 3 if mode == CROSS_RESIDUAL else 0)
        scale = modulation(mod, time, 4 if mode == CROSS_RESIDUAL else 1)
        scale = bf16(1.0 + scale)                           # :173
        n = bf16(n * scale) + shift                         # :174
    return bf16(x), bf16(n)                                 # bf16 stores, :175-176


def gelu_tanh(x: torch.Tensor) -> torch.Tensor:
    return F.gelu(x, approximate="tanh")


def prepared_ffn(x, w_up, b_up, w_down, b_down):
    """Prepared (cuBLASLt) contract: fp32 accumulation, bias + GELU in one fp32
    epilogue, bf16 hidden, bias epilogue on the down GEMM
    (WAMInfer/ffn.py:1-4, WAMInfer/_cublaslt_inference.cpp:70-83)."""
    h = bf16(gelu_tanh(x.float() @ w_up.float().T + b_up.float()))
    return bf16(h @ w_down.float().T + b_down.float())


def native_ffn(x, w_up, b_up, w_down, b_down):
    """The reference's native bf16 path (WAMInfer/blocks.py:254-258): Linear,
    bf16, GELU(tanh), bf16, Linear, bf16."""
    h = bf16(x.float() @ w_up.float().T + b_up.float())
    h = bf16(gelu_tanh(h))
    return bf16(h @ w_down.float().T + b_down.float())


def gate_residual(y, output, mod, time):
    """bf16(y + bf16(bf16(mod[5] + time[5]) * output)) -- the FFN_RESIDUAL fold
    (WAMInfer/_triton_inference.py:158-161) and the last-layer update
    (WAMInfer/blocks.py:265-268)."""
    return bf16(y.float() + bf16(modulation(mod, time, 5) * output.float()))


def ffn_block(x, update, normalized, mod, time, w_up, b_up, w_down, b_down, indices, cache, cache_rows: int,
              eps: float, ffn=prepared_ffn):
    """One layer's FFN phase in sequence order.

    x, update, normalized: [S, d]; indices: [M] ints (-1 = pad) or None;
    cache: [cache_rows, d] previous FFN outputs or None.
    Returns (x_next [S, d], output [S, d], clean [cache_rows, d] or None, o [M, d]).

    Follows WAMInfer/blocks.py:241-244 (CROSS_RESIDUAL norm), :249-251 (gather),
    :252-258 (FFN), :259-264 (index_copy into the cache copy + cat with the
    fresh rows), :265-271 (gate, applied immediately).
    """
    if normalized is None:
        y, n = modulated_norm(x, update, mod, None, time, None, None, CROSS_RESIDUAL, eps)
    else:
        y, n = x.float(), normalized.float()
    S, d = y.shape
    dev = y.device
    if indices is None:
        idx = torch.arange(S, device=dev)
    else:
        idx = torch.as_tensor(indices).long().to(dev)
    pad = idx < 0
    a = n[idx.clamp_min(0)]
    a[pad] = 0.0
    o = ffn(a, w_up, b_up, w_down, b_down).to(dev)
    output = torch.zeros(S, d, device=dev)
    if cache_rows > 0 and cache is not None:
        output[:cache_rows] = cache.float().to(dev)
    # index_copy semantics with later entries winning on duplicates: each row
    # takes the last gather slot j that names it.
    slots = torch.arange(idx.numel(), device=dev)
    last = torch.full((S,), -1, dtype=torch.long, device=dev)
    last.scatter_reduce_(0, idx[~pad], slots[~pad], reduce="amax")
    rows = torch.nonzero(last >= 0).flatten()
    output[rows] = o[last[rows]]
    clean = output[:cache_rows].clone() if cache_rows > 0 else None
    x_next = gate_residual(y, output, mod, time)
    return x_next, output, clean, o


MAX_ABS = 2e-2    # elementwise bound (or one bf16 ulp of the reference value, whichever is larger)
MEAN_REL = 5e-3   # mean |error| / mean |reference|


def bf16_ulp(t: torch.Tensor) -> torch.Tensor:
    """Spacing of bfloat16 values at |t| (8 significant bits)."""
    _, exponent = torch.frexp(t.float().abs().clamp_min(2.0**-126))
    return torch.ldexp(torch.ones_like(t, dtype=torch.float32), exponent - 8)


def check_close(actual: torch.Tensor, expected: torch.Tensor, max_abs: float = MAX_ABS,
                mean_rel: float = MEAN_REL) -> tuple[bool, str]:
    """Parity rule for bf16 outputs against the fp32 oracle: every element within
    max(max_abs, 1 bf16 ulp of the reference) -- two correct implementations
    that accumulate in different orders can round one ulp apart, and one ulp
    exceeds 2e-2 above |x| = 4 -- and the mean relative error within mean_rel."""
    a, e = actual.float().cpu(), expected.float().cpu()
    if not bool(torch.isfinite(a).all()):
        return False, "non-finite output"
    err = (a - e).abs()
    bound = torch.maximum(torch.full_like(e, max_abs), bf16_ulp(e))
    over = err - bound
    excess = float(over.max())
    rel = float(err.mean() / e.abs().mean().clamp_min(1e-12))
    ok = excess <= 0 and rel <= mean_rel
    worst = tuple(int(i) for i in torch.nonzero(over == over.max())[0])
    return ok, (f"max abs {float(err.max()):.4g} (worst excess over bound {excess:.3g} at {worst}: "
                f"got {float(a[worst]):.6g}, expected {float(e[worst]):.6g}; "
                f"{int((over > 0).sum())} elements over), mean rel {rel:.3g}")
