"""The reference's own FFN phase, run from the unmodified WAMInfer package
installed in baseline/_ref (a baseline and a checker; the product never
imports this module).

    python -m pip install --no-index --no-build-isolation --no-deps \
        --find-links /opt/wheelhouse --target baseline/_ref <WAMInfer checkout>

WAMInfer's package ``__init__`` imports the absent ``openwam``; registering a
stub parent package whose ``__path__`` is the installed package directory
lets ``WAMInfer.blocks``, ``WAMInfer.ffn``, ``WAMInfer.approximation`` and
``WAMInfer._triton_inference`` import unchanged.

A pass is what the reference's layer loop does between two FFNs when no
attention runs (every layer's FFN input is the previous layer's residual), per
layer:

* the FFN_RESIDUAL modulated norm that folds the previous layer's deferred,
  gated FFN output (``pre_attn_at_layer_for_compile``,
  WAMInfer/blocks.py:189-203; SELF_INPUT at layer 0);
* the CROSS_RESIDUAL norm of the FFN input with a zero cross-attention output
  (WAMInfer/blocks.py:241-243);
* ``VideoAdapter.ffn_at_layer_for_compile`` (WAMInfer/blocks.py:246-272): row
  gather, the FFN (``PreparedFFN``'s cuBLASLt plans, WAMInfer/ffn.py:96-107,
  or the native ``Linear -> GELU(tanh) -> Linear`` when ``ffn`` is None),
  history ``index_copy`` + ``cat``, and the last layer's gate;

and after a token-reuse pass the history stack of WAMInfer/runtime.py:263.

The modulated norm is the reference's Triton kernel on a GPU.  On the CPU the
caller supplies a restatement with the same signature (the Triton kernel has
no CPU path).
"""

from __future__ import annotations

import sys
import types
from pathlib import Path
from types import SimpleNamespace

import torch

REF_ROOT = Path(__file__).resolve().parent / "_ref"
CUBLASLT_EXTENSION = "wam_infer_ffn_v1"


def missing(cuda: bool) -> str | None:
    """Why the reference cannot run here, or None."""
    if not (REF_ROOT / "WAMInfer" / "blocks.py").exists():
        return "baseline/_ref/WAMInfer is not installed"
    if cuda and not (REF_ROOT / f"{CUBLASLT_EXTENSION}.so").exists():
        return f"baseline/_ref/{CUBLASLT_EXTENSION}.so (the reference's cuBLASLt extension) is not built"
    return None


def import_reference(cuda: bool) -> SimpleNamespace:
    """The reference's modules, imported through a stub parent package.  With
    cuda, also its cuBLASLt extension (prebuilt from its own source into
    baseline/_ref) and its Triton modulated norm."""
    reason = missing(cuda)
    if reason is not None:
        raise FileNotFoundError(reason)
    if "WAMInfer" not in sys.modules:
        pkg = types.ModuleType("WAMInfer")
        pkg.__path__ = [str(REF_ROOT / "WAMInfer")]
        sys.modules["WAMInfer"] = pkg
    if str(REF_ROOT) not in sys.path:
        sys.path.insert(0, str(REF_ROOT))
    from WAMInfer import approximation, blocks, ffn

    ns = SimpleNamespace(blocks=blocks, ffn=ffn, approximation=approximation, modulated_norm=None, modes=None)
    if cuda:
        import importlib

        ext = importlib.import_module(CUBLASLT_EXTENSION)
        ffn._extension = lambda: ext  # the reference's own extension, built from its source
        from WAMInfer import _triton_inference as ti

        ns.modulated_norm = ti.modulated_norm
        ns.modes = (ti.SELF_INPUT, ti.SELF_RESIDUAL, ti.CROSS_RESIDUAL, ti.FFN_RESIDUAL)
    return ns


def make_blocks(layer_weights, device, eps: float = 1e-6) -> list[SimpleNamespace]:
    """DiT blocks holding what the FFN phase reads: ``ffn`` (nn.Sequential of
    Linear(d, h), GELU(tanh), Linear(h, d), bf16, eval), ``modulation``
    [1, 6, d] and ``norm2.eps``.  `layer_weights` yields objects with w_up,
    b_up, w_down, b_down, mod."""
    blocks = []
    for w in layer_weights:
        h, d = w.w_up.shape
        kw = dict(device=device, dtype=torch.bfloat16)
        with torch.device("meta"):
            ffn = torch.nn.Sequential(torch.nn.Linear(d, h), torch.nn.GELU(approximate="tanh"), torch.nn.Linear(h, d))
        ffn = ffn.to_empty(device=device).to(torch.bfloat16).eval()
        with torch.no_grad():
            ffn[0].weight.copy_(w.w_up)
            ffn[0].bias.copy_(w.b_up)
            ffn[2].weight.copy_(w.w_down)
            ffn[2].bias.copy_(w.b_down)
        for p in ffn.parameters():
            p.requires_grad_(False)
        mod = w.mod.to(**kw).reshape(1, 6, d)
        blocks.append(SimpleNamespace(ffn=ffn, modulation=mod, norm2=SimpleNamespace(eps=eps),
                                      norm1=SimpleNamespace(eps=eps)))
    return blocks


class ReferencePhase:
    """The reference's FFN phase over `blocks` (one VideoAdapter: plans and
    workspaces are per model in the reference, WAMInfer/ffn.py:5-6).

    prepared_rows: row counts to prepare ``PreparedFFN`` for (its cuBLASLt
    plans, GPU only); None runs the native FFN (``vb.ffn = None``).
    norm: a callable with the signature of the reference's modulated norm;
    None uses the reference's Triton kernel (GPU)."""

    SELF_INPUT, SELF_RESIDUAL, CROSS_RESIDUAL, FFN_RESIDUAL = 0, 1, 2, 3

    def __init__(self, ref: SimpleNamespace, blocks, device, prepared_rows=None, norm=None):
        self.ref, self.blocks, self.device = ref, blocks, torch.device(device)
        native = SimpleNamespace(dit=SimpleNamespace(blocks=blocks), num_layers=len(blocks), training=False)
        self.vb = ref.blocks.VideoAdapter(native)
        self.vb.ffn = None
        if prepared_rows is not None:
            with torch.no_grad():
                self.vb.ffn = ref.ffn.PreparedFFN(self.vb)
                self.vb.ffn.prepare(rows=tuple(sorted(set(int(r) for r in prepared_rows))))
        self.norm = norm if norm is not None else ref.modulated_norm
        if self.norm is None:
            raise ValueError("no modulated norm: pass a restatement on the CPU")

    def run_pass(self, x, time, indices=None, history=None, n: int = 0, count: int = 0):
        """One pass over every layer.  x [seq, d] bf16, time [seq, 6, d] bf16;
        with `indices` (the select_tokens list: `count` current rows, then the
        future rows) layers 1.. gather them and read history [layers-1, n, d].
        Returns (x_out [seq, d], history_out [layers-1, n, d] or None)."""
        d = x.shape[-1]
        zero = torch.zeros(1, x.shape[0], d, device=x.device, dtype=x.dtype)
        extras = {}
        if indices is not None:
            extras = dict(token_reuse=dict(n=n, count=count, cache=history[:, None]),
                          token_indices=indices, token_outputs=[])
        state = SimpleNamespace(time_mod=time[None], extras=extras, hidden_states=x[None])
        with torch.no_grad():
            for layer, block in enumerate(self.blocks):
                pending = state.extras.pop("_inference_ffn_residual", None)
                update, previous = (None, None) if pending is None else pending
                mode = self.SELF_INPUT if pending is None else self.FFN_RESIDUAL
                xs, _ = self.norm(state.hidden_states, update, block.modulation, previous, state.time_mod, None, None,
                                  mode, block.norm1.eps)
                xs, normalized = self.norm(xs, zero, block.modulation, None, state.time_mod, None, None,
                                           self.CROSS_RESIDUAL, block.norm2.eps)
                self.vb.ffn_at_layer_for_compile(layer, state, normalized, xs)
            hist = None
            if indices is not None:
                hist = torch.stack(state.extras["token_outputs"])[:, 0]
        return state.hidden_states[0], hist

    def close(self):
        if self.vb.ffn is not None:
            self.vb.ffn.close()
            self.vb.ffn = None


def random_blocks(layers: int, d: int, h: int, device, seed: int = 0, eps: float = 1e-6) -> list[SimpleNamespace]:
    """Blocks with seeded synthetic weights (W ~ N(0, 0.02), biases ~ N(0, 0.01),
    modulation ~ N(0, 0.1), bf16) built without a second copy of the 5.3 GB
    of 30-layer FFN weights (the CPU baseline's host memory).  One base pair
    of weight matrices is drawn; layer l's matrices are the base ones with
    their elements rotated by l x 104729 positions (distinct weights of the
    same distribution; seeded RNG over 5.3 G values would take minutes on the
    host)."""
    g = torch.Generator(device=device).manual_seed(seed)
    base_up = (torch.randn(h * d, device=device, generator=g) * 0.02).to(torch.bfloat16)
    base_dn = (torch.randn(d * h, device=device, generator=g) * 0.02).to(torch.bfloat16)
    blocks = []
    for layer in range(layers):
        with torch.device("meta"):
            ffn = torch.nn.Sequential(torch.nn.Linear(d, h), torch.nn.GELU(approximate="tanh"), torch.nn.Linear(h, d))
        ffn = ffn.to_empty(device=device).to(torch.bfloat16).eval()
        shift = layer * 104729
        with torch.no_grad():
            ffn[0].weight.copy_(torch.roll(base_up, shift).view(h, d))
            ffn[2].weight.copy_(torch.roll(base_dn, shift).view(d, h))
            ffn[0].bias.copy_((torch.randn(h, device=device, generator=g) * 0.01).to(torch.bfloat16))
            ffn[2].bias.copy_((torch.randn(d, device=device, generator=g) * 0.01).to(torch.bfloat16))
        for p in ffn.parameters():
            p.requires_grad_(False)
        mod = (torch.randn(1, 6, d, device=device, generator=g) * 0.1).to(torch.bfloat16)
        blocks.append(SimpleNamespace(ffn=ffn, modulation=mod, norm2=SimpleNamespace(eps=eps),
                                      norm1=SimpleNamespace(eps=eps)))
    return blocks
