"""The reference's CPU FFN path, timed as the CPU baseline (test/bench infrastructure only).

Restates what ``VideoAdapter.ffn_at_layer_for_compile`` does when the native
FFN runs (``WAMInfer/blocks.py:246-272`` with ``vb.ffn = None``): row gather,
``Linear -> GELU(tanh) -> Linear`` in bf16 torch, cache ``index_copy`` + ``cat``,
and the gated residual -- plus the CROSS_RESIDUAL LayerNorm/adaLN prologue of
``WAMInfer/_triton_inference.py:149-176`` in torch.  Used only by ``bench.py``
(CPU-baseline leg and ``--impl reference``).
"""

from __future__ import annotations

import time

import torch
import torch.nn.functional as F


def _norm_bf16(x, mod, time_mod, eps=1e-6):
    xf = x.float()
    mean = xf.mean(-1, keepdim=True)
    c = xf - mean
    n = (c * torch.rsqrt((c * c).mean(-1, keepdim=True) + eps)).bfloat16()
    shift = (mod[3] + time_mod[:, 3]).bfloat16()
    scale = (1.0 + (mod[4] + time_mod[:, 4]).bfloat16().float()).bfloat16()
    return ((n * scale).bfloat16() + shift).bfloat16()


def layer(x, time_mod, w, indices=None, cache=None, n=0):
    """One FFN phase on CPU tensors (bf16). Returns (x_next, clean)."""
    normalized = _norm_bf16(x, w["mod"], time_mod)
    a = normalized.index_select(0, indices) if indices is not None else normalized
    h = F.gelu(F.linear(a, w["w_up"], w["b_up"]), approximate="tanh")
    out = F.linear(h, w["w_down"], w["b_down"])
    clean = None
    if indices is not None:
        count = indices.numel() - (x.shape[0] - n)
        clean = cache.index_copy(0, indices[:count], out[:count])
        out = torch.cat((clean, out[count:]), dim=0)
    gate = (w["mod"][5] + time_mod[:, 5]).bfloat16()
    return (x + gate * out).bfloat16(), clean


def make_layer(d, h, seed=0):
    g = torch.Generator().manual_seed(seed)

    def rnd(*shape, std):
        return (torch.randn(*shape, generator=g) * std).bfloat16()

    return dict(w_up=rnd(h, d, std=0.02), b_up=rnd(h, std=0.01), w_down=rnd(d, h, std=0.02),
                b_down=rnd(d, std=0.01), mod=rnd(6, d, std=0.1).float())


def time_layers(geo, sample_layers: int, min_seconds: float = 10.0, max_reps: int = 50):
    """Times `sample_layers` reuse layers and `sample_layers` full layers,
    repeated until `min_seconds` of work; returns (flops, seconds)."""
    w = make_layer(geo.d, geo.h)
    g = torch.Generator().manual_seed(1)
    x = torch.randn(geo.seq, geo.d, generator=g).bfloat16()
    time_mod = (torch.randn(geo.seq, 6, geo.d, generator=g) * 0.1).bfloat16().float()
    chosen = torch.randperm(geo.current, generator=g)[: geo.count].sort().values
    indices = torch.cat((chosen, torch.arange(geo.current, geo.seq)))
    cache = torch.randn(geo.current, geo.d, generator=g).bfloat16()
    per_rep = 4 * geo.d * geo.h * sample_layers * (geo.reuse_rows + geo.seq)
    layer(x, time_mod, w)  # warm-up (thread pool, weight packing)
    flops, seconds, reps = 0, 0.0, 0
    while reps < max_reps and (seconds < min_seconds or reps == 0):
        t0 = time.perf_counter()
        y = x
        for _ in range(sample_layers):
            y, _ = layer(y, time_mod, w, indices, cache, geo.current)
        for _ in range(sample_layers):
            y, _ = layer(y, time_mod, w)
        seconds += time.perf_counter() - t0
        flops += per_rep
        reps += 1
    return flops, seconds
