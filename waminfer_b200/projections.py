"""Attention-side projections on the same tcgen05 GEMM engine: the packed QKV
projection of ``pre_attn_at_layer_for_compile``
(``WAMInfer/blocks.py:204-208``), the self-attention output projection
(``blocks.py:218``) and the cross-attention query / output projections
(``blocks.py:234, 240``).

The reference packs Q, K and V into one [3d, d] weight per block with
``prepare_packed_weights`` (``blocks.py:27-46``, called from
``runtime.py:284-287``) and runs ``torch.nn.functional.linear`` on it (cuBLAS).
Here ``PreparedProjections`` keeps, per block, tile-packed copies of the packed
QKV weight and of the three d x d projections (refreshed when a parameter's
signature changes, the reference's contract), builds one library ``Plan`` per
(projection, row count) -- bias epilogue, split-K chosen by timing -- and runs
them through the ``wam_ffn::prepared_ffn_linear_v1`` op.  A row count that was
not prepared falls back to the module's own linear, as ``PreparedFFN`` does.

The modulated norms around these projections are the library's
``wam_ffn::modulated_norm`` (``waminfer_b200/norm.py``); the Q/K RMSNorm +
RoPE and the attention kernels stay with the caller.
"""

from __future__ import annotations

import torch
import torch.nn.functional as F

from waminfer_b200.blocks import _parameter_signature
from waminfer_b200.ffn import _IDS, _PLANS, Plan, pack_weight, prepared_linear

# projection -> (attention module on the block, Linear names packed along the output features)
PROJECTIONS = {
    "qkv": ("self_attn", ("q", "k", "v")),
    "self_out": ("self_attn", ("o",)),
    "cross_q": ("cross_attn", ("q",)),
    "cross_out": ("cross_attn", ("o",)),
}


def packed_projection(attention, names) -> tuple[torch.Tensor, torch.Tensor | None, tuple]:
    """The reference's packing rule (``blocks.py:27-46``): same-shaped
    projections concatenated along the output features; biases all present or
    all absent.  Returns (weight [n*out, in], bias or None, signature)."""
    if attention.training or torch.is_grad_enabled():
        raise RuntimeError("Projection packing requires eval mode and disabled gradients.")
    layers = [getattr(attention, name) for name in names]
    if len({(layer.in_features, layer.out_features) for layer in layers}) != 1:
        raise ValueError("Packed projections must have matching dimensions.")
    biases = [layer.bias for layer in layers]
    if any(b is None for b in biases) and not all(b is None for b in biases):
        raise ValueError("Packed projections must all use bias or all omit it.")
    signature = tuple(_parameter_signature(p) for layer in layers for p in (layer.weight, layer.bias))
    weight = torch.cat([layer.weight.detach() for layer in layers]) if len(layers) > 1 else layers[0].weight.detach()
    bias = None
    if biases[0] is not None:
        bias = torch.cat([b.detach() for b in biases]) if len(layers) > 1 else biases[0].detach()
    return weight, bias, signature


class PreparedProjections:
    """Per-model plans for the attention projections of every block of
    ``backbone.dit.blocks``; same prepare / call / close life cycle as
    ``PreparedFFN``."""

    max_plans = 64

    def __init__(self, backbone):
        self.backbone = backbone
        self.weights = {}      # (layer, kind) -> tile-packed weight
        self.biases = {}       # (layer, kind) -> bias (zeros when the reference has none)
        self.signatures = {}
        self.plans = {}        # (layer, kind, rows) -> plan id
        self.keys = {}

    def _plan(self, kind, weight, bias, rows):
        key = (weight.device, rows, tuple(weight.shape), kind)
        if key not in self.keys:
            if len(self.keys) >= self.max_plans:
                raise RuntimeError("Projection preparation supports at most 64 device/shape plans per model.")
            k = weight.shape[1] * 64
            x = torch.empty(rows, k, device=weight.device, dtype=weight.dtype)
            plan = Plan(x, weight, bias, True, False)
            plan_id = next(_IDS)
            _PLANS[plan_id] = plan
            self.keys[key] = plan_id
        return self.keys[key]

    def prepare(self, rows) -> bool:
        """Refreshes packed weights whose signature changed and builds plans for
        every (block, projection, row count); returns whether anything changed."""
        if torch.is_grad_enabled() or getattr(self.backbone, "training", False):
            raise RuntimeError("Projection preparation requires eval mode and disabled gradients.")
        changed = False
        for layer_id, block in enumerate(self.backbone.dit.blocks):
            for kind, (attr, names) in PROJECTIONS.items():
                attention = getattr(block, attr)
                weight, bias, signature = packed_projection(attention, names)
                if weight.dtype != torch.bfloat16 or weight.device.type != "cuda":
                    raise ValueError("Prepared projections require CUDA BF16 linear layers.")
                key = (layer_id, kind)
                if self.signatures.get(key) != signature:
                    self.weights[key] = pack_weight(weight)
                    self.biases[key] = bias.contiguous() if bias is not None else torch.zeros(
                        weight.shape[0], device=weight.device, dtype=weight.dtype)
                    self.signatures[key] = signature
                    changed = True
                for m in rows:
                    pid = self._plan(kind, self.weights[key], self.biases[key], m)
                    changed |= self.plans.get((layer_id, kind, m)) != pid
                    self.plans[layer_id, kind, m] = pid
        return changed

    def run(self, layer_id: int, kind: str, inputs: torch.Tensor) -> torch.Tensor:
        rows = inputs.numel() // inputs.shape[-1]
        key = (layer_id, kind)
        flat = inputs.reshape(rows, inputs.shape[-1])
        pid = self.plans.get((layer_id, kind, rows))
        if pid is None:
            # Unprepared geometry: the module's own linear (no planning during capture).
            attr, names = PROJECTIONS[kind]
            weight, bias, _ = packed_projection(getattr(self.backbone.dit.blocks[layer_id], attr), names)
            out = F.linear(flat, weight, bias)
        else:
            out = prepared_linear(flat.contiguous(), self.weights[key], self.biases[key], pid)
        return out.reshape(*inputs.shape[:-1], out.shape[-1])

    def qkv(self, layer_id, normalized):
        """``F.linear(flat, qkv_weight, qkv_bias)`` of ``blocks.py:205-206``; the
        caller chunks it into q, k, v."""
        return self.run(layer_id, "qkv", normalized)

    def self_out(self, layer_id, attended):
        return self.run(layer_id, "self_out", attended)

    def cross_q(self, layer_id, normalized):
        return self.run(layer_id, "cross_q", normalized)

    def cross_out(self, layer_id, context):
        return self.run(layer_id, "cross_out", context)

    def close(self):
        for plan_id in self.keys.values():
            plan = _PLANS.pop(plan_id, None)
            if plan is not None:
                plan.close()
        self.keys.clear()
        self.plans.clear()
        self.weights.clear()
        self.biases.clear()
        self.signatures.clear()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
