"""Video FFN phase on the fused libwamffn block kernels.

Host-side mirror of the reference's FFN call site,
``VideoAdapter.ffn_at_layer_for_compile`` (``WAMInfer/blocks.py:246-272``):
row gather by ``token_indices`` (``:249-251``), the FFN, the scatter of the
recomputed current-frame rows into a copy of the previous request's cache and
the concatenation with the fresh rows (``:259-264``), and the gated residual
that the reference defers to the next layer's FFN_RESIDUAL norm
(``:269-271`` + ``WAMInfer/_triton_inference.py:158-161``) or applies in torch
on the last layer (``:265-268``).  Here all of it is one op, ``wam_ffn::ffn_block``,
that launches four kernels (norm/gather, up GEMM, down GEMM, reduce/scatter/gate).

Applying the gate inside the FFN op instead of the next layer's norm gives the
same bf16 values: the reference rounds ``x + bf16(gate*out)`` to bf16 before
its LayerNorm, which is exactly the residual this op returns.
"""

from __future__ import annotations

import ctypes
from itertools import count

import torch

from waminfer_b200 import _lib
from waminfer_b200.norm import time_row_stride


def _parameter_signature(parameter):
    """Identity + storage + version key of a parameter: a change means packed
    state (plans, captured graphs) must be refreshed.  Same fields as the
    reference's key (``WAMInfer/blocks.py:12-24``); inference tensors have no
    version counter, so they never compare equal."""
    if parameter is None:
        return None
    version = object() if parameter.is_inference() else parameter._version
    return (
        id(parameter),
        parameter.data_ptr(),
        parameter.shape,
        parameter.stride(),
        parameter.dtype,
        parameter.device,
        version,
    )


class BlockPlan:
    """Scratch and launch configuration of the fused FFN block on one device."""

    def __init__(self, device: torch.device, max_rows: int, max_seq: int, d_model: int, d_hidden: int,
                 tune: bool = False):
        if torch.cuda.is_current_stream_capturing():
            raise RuntimeError("FFN block planning must finish before CUDA Graph capture")
        self.device = torch.device(device)
        self.max_rows, self.max_seq, self.d, self.h = max_rows, max_seq, d_model, d_hidden
        handle = ctypes.c_void_p()
        _lib.check(_lib.lib().wamffn_block_plan_create(
            self.device.index, max_rows, max_seq, d_model, d_hidden, int(tune), ctypes.byref(handle)))
        self._handle = handle

    @property
    def handle(self):
        if self._handle is None:
            raise RuntimeError("block plan is closed")
        return self._handle

    def run(self, args: _lib.BlockArgs, stream: int) -> None:
        _lib.check(_lib.lib().wamffn_block_run(self.handle, stream, ctypes.byref(args)))

    def configuration(self, rows: int) -> dict:
        values = (ctypes.c_uint32 * 16)()
        _lib.check(_lib.lib().wamffn_block_configuration(self.handle, rows, values, 16))
        names = ("feature_tile", "token_pad", "mma_count", "stages", "split_k", "tmem_columns", "tuned")
        up, down = dict(zip(names, values[:7])), dict(zip(names, values[7:14]))
        up["streamk_groups"], down["streamk_groups"] = values[14], values[15]
        return {"up": up, "down": down}

    def set_streamk(self, enabled: bool) -> None:
        """Stream-K up projection (every SM pair takes an equal range of the
        tiles' K blocks) on or off for launches enqueued from now on."""
        _lib.check(_lib.lib().wamffn_block_plan_set_streamk(self.handle, 1 if enabled else 0))

    def set_splits(self, rows: int, splits: int) -> None:
        """Down-projection split-K factor for `rows` gathered rows (0: all row
        counts); 0 restores the SM-filling heuristic.  Lanes of concurrent
        requests run with fewer splits (``FFNStack(lanes=...)``)."""
        _lib.check(_lib.lib().wamffn_block_plan_set_splits(self.handle, rows, splits))

    def status(self, clear: bool = True) -> int:
        """Device status word (timeout / bad-index bits); synchronises the device."""
        value = ctypes.c_uint32()
        _lib.check(_lib.lib().wamffn_block_status(self.handle, ctypes.byref(value), int(clear)))
        return int(value.value)

    def close(self) -> None:
        if getattr(self, "_handle", None) is not None:
            _lib.lib().wamffn_block_plan_destroy(self._handle)
            self._handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


_BLOCK_PLANS: dict[int, BlockPlan] = {}
_BLOCK_IDS = count()


def register_block_plan(plan: BlockPlan) -> int:
    plan_id = next(_BLOCK_IDS)
    _BLOCK_PLANS[plan_id] = plan
    return plan_id


def release_block_plan(plan_id: int) -> None:
    plan = _BLOCK_PLANS.pop(plan_id, None)
    if plan is not None:
        plan.close()


def _rows2d(t: torch.Tensor, dim: int, name: str) -> torch.Tensor:
    if t.dtype != torch.bfloat16:
        raise ValueError(f"{name} must be bfloat16")
    if t.dim() == 3:
        if t.shape[0] != 1:
            raise ValueError(f"{name} must have batch 1")
        t = t[0]
    if t.dim() != 2 or t.shape[1] != dim or not t.is_contiguous():
        raise ValueError(f"{name} must be a contiguous [rows, {dim}] (or [1, rows, {dim}]) tensor")
    return t


def block_args(x, update, normalized, mod, time, w_up, b_up, w_down, b_down, indices, cache, cache_rows,
               eps, x_out, output, clean, y=None) -> _lib.BlockArgs:
    """Builds the C argument struct from torch tensors (shape/dtype checked)."""
    packed = w_up.dim() == 4
    h, d = (w_up.shape[0] * 128, w_up.shape[1] * 64) if packed else (w_up.shape[0], w_up.shape[1])
    x2 = _rows2d(x, d, "x")
    seq = x2.shape[0]
    if update is not None:
        _rows2d(update, d, "update")
    if normalized is not None:
        _rows2d(normalized, d, "normalized")
    if mod.dtype != torch.bfloat16 or mod.shape[-2:] != (6, d) or not mod.is_contiguous():
        raise ValueError(f"mod must be a contiguous bf16 [1, 6, {d}] tensor")
    if time.dtype != torch.bfloat16 or time.shape[-2:] != (6, d) or time.stride(-1) != 1 or time.stride(-2) != d:
        raise ValueError(f"time must be bf16 with contiguous trailing [6, {d}] rows")
    if time.ndim == 4 and time.shape[1] not in (1, seq):
        raise ValueError("per-token time must have one row per sequence row")
    for name, w, shape in (("w_up", w_up, (h, d)), ("w_down", w_down, (d, h))):
        want = (shape[0] // 128, shape[1] // 64, 128, 64) if packed else shape
        if w.dtype != torch.bfloat16 or tuple(w.shape) != want or not w.is_contiguous():
            raise ValueError(f"{name} must be a contiguous bf16 {list(shape)} (out, in) matrix"
                             f"{' in the packed layout' if packed else ''}")
    for name, b, n in (("b_up", b_up, h), ("b_down", b_down, d)):
        if b.dtype != torch.bfloat16 or b.numel() != n or not b.is_contiguous():
            raise ValueError(f"{name} must be a contiguous bf16 vector of {n}")
    if indices is not None:
        if indices.dtype not in (torch.int32, torch.int64) or indices.dim() != 1 or not indices.is_contiguous():
            raise ValueError("indices must be a contiguous int32/int64 vector")
        rows = indices.numel()
    else:
        rows = seq
    if cache is not None:
        _rows2d(cache, d, "cache")
    return _lib.BlockArgs(
        x=x2.data_ptr(),
        update=None if update is None else update.data_ptr(),
        normalized=None if normalized is None else normalized.data_ptr(),
        mod=mod.data_ptr(),
        time=time.data_ptr(),
        time_stride=time_row_stride(time),
        w_up=w_up.data_ptr(),
        b_up=b_up.data_ptr(),
        w_down=w_down.data_ptr(),
        b_down=b_down.data_ptr(),
        weights_packed=int(packed),
        indices=None if indices is None else indices.data_ptr(),
        index_bytes=0 if indices is None else indices.element_size(),
        rows=rows,
        seq=seq,
        cache_rows=cache_rows,
        cache_in=None if cache is None else cache.data_ptr(),
        cache_out=None if clean is None else clean.data_ptr(),
        y=None if y is None else y.data_ptr(),
        output=None if output is None else output.data_ptr(),
        x_out=None if x_out is None else x_out.data_ptr(),
        eps=float(eps),
    )


@torch.library.custom_op("wam_ffn::ffn_block", mutates_args=())
def ffn_block(
    x: torch.Tensor,
    update: torch.Tensor | None,
    normalized: torch.Tensor | None,
    mod: torch.Tensor,
    time: torch.Tensor,
    w_up: torch.Tensor,
    b_up: torch.Tensor,
    w_down: torch.Tensor,
    b_down: torch.Tensor,
    indices: torch.Tensor | None,
    cache: torch.Tensor | None,
    cache_rows: int,
    plan_id: int,
    eps: float,
    want_output: bool,
) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    """One layer's FFN phase.  Returns ``(x_next, output, clean)``:

    * ``x_next``  residual after the gated FFN update, shaped like ``x``;
    * ``output``  FFN output in sequence order (empty unless ``want_output``);
    * ``clean``   ``[1, cache_rows, d]`` rows to keep as this layer's FFN history
      (empty when ``cache_rows == 0``).
    """
    plan = _BLOCK_PLANS[plan_id]
    d = w_up.shape[1] * 64 if w_up.dim() == 4 else w_up.shape[1]
    x_next = torch.empty_like(x)
    seq = x.numel() // d
    output = torch.empty_like(x) if want_output else x.new_empty((0,))
    clean = x.new_empty((1, cache_rows, d)) if cache_rows > 0 else x.new_empty((0,))
    args = block_args(x, update, normalized, mod, time, w_up, b_up, w_down, b_down, indices, cache, cache_rows,
                      eps, x_next, output if want_output else None, clean if cache_rows > 0 else None)
    if args.seq != seq:
        raise ValueError("x must hold whole rows")
    with torch.cuda.device(x.device):
        plan.run(args, torch.cuda.current_stream(x.device).cuda_stream)
    return x_next, output, clean


@ffn_block.register_fake
def _fake_block(x, update, normalized, mod, time, w_up, b_up, w_down, b_down, indices, cache, cache_rows, plan_id,
                eps, want_output):
    d = w_up.shape[1] * 64 if w_up.dim() == 4 else w_up.shape[1]
    output = torch.empty_like(x) if want_output else x.new_empty((0,))
    clean = x.new_empty((1, cache_rows, d)) if cache_rows > 0 else x.new_empty((0,))
    return torch.empty_like(x), output, clean


class VideoFFN:
    """Drop-in FFN phase for the reference's ``VideoAdapter``.

    ``ffn_at_layer_for_compile(layer_id, state, normalized, x)`` keeps the
    reference's signature and state contract (``WAMInfer/blocks.py:246-272``):
    ``state.extras['token_reuse']`` / ``['token_indices']`` select rows,
    ``['token_outputs']`` receives each layer's ``[1, n, d]`` FFN history and
    ``state.hidden_states`` the residual.  The gate is applied here instead of
    being deferred, so the next layer's pre-attention norm sees no pending
    FFN residual (SELF_INPUT gives the same values as FFN_RESIDUAL would).

    ``post_attn_ffn(layer_id, state, x, cross_output)`` additionally fuses the
    CROSS_RESIDUAL norm that ends ``post_attn_at_layer_for_compile``
    (``WAMInfer/blocks.py:241-244``).
    """

    def __init__(self, backbone, *, max_rows: int, max_seq: int, tune: bool = False):
        self.backbone = backbone
        blocks = backbone.dit.blocks
        first = blocks[0].ffn
        self.d, self.h = first[0].in_features, first[0].out_features
        device = first[0].weight.device
        self.plan_id = register_block_plan(BlockPlan(device, max_rows, max_seq, self.d, self.h, tune))
        self.eps = [getattr(getattr(b, "norm2", None), "eps", 1e-6) for b in blocks]
        self.packed = {}
        self.signatures = {}

    @property
    def plan(self) -> BlockPlan:
        return _BLOCK_PLANS[self.plan_id]

    def prepare(self) -> bool:
        """Refreshes the tile-packed weight copies whose parameter signature
        changed (the repack of ``PreparedFFN.prepare``); returns whether any did."""
        from waminfer_b200.ffn import pack_weight

        if torch.is_grad_enabled() or getattr(self.backbone, "training", False):
            raise RuntimeError("FFN preparation requires eval mode and disabled gradients.")
        changed = False
        for layer_id, block in enumerate(self.backbone.dit.blocks):
            ffn = block.ffn
            if not isinstance(ffn[1], torch.nn.GELU) or ffn[1].approximate != "tanh":
                raise ValueError("Fused FFN requires tanh GELU.")
            for index in (0, 2):
                layer = ffn[index]
                if layer.weight.dtype != torch.bfloat16 or layer.weight.device.type != "cuda" or layer.bias is None:
                    raise ValueError("Fused FFN requires CUDA BF16 linear layers with bias.")
                signature = _parameter_signature(layer.weight)
                if self.signatures.get((layer_id, index)) != signature:
                    self.packed[layer_id, index] = pack_weight(layer.weight.detach())
                    self.signatures[layer_id, index] = signature
                    changed = True
        return changed

    def _weights(self, layer_id):
        ffn = self.backbone.dit.blocks[layer_id].ffn
        if (layer_id, 0) not in self.packed:
            self.prepare()
        return self.packed[layer_id, 0], ffn[0].bias, self.packed[layer_id, 2], ffn[2].bias

    def _run(self, layer_id, state, x, update, normalized):
        block = self.backbone.dit.blocks[layer_id]
        reuse = state.extras.get("token_reuse") if layer_id > 0 else None
        indices = state.extras.get("token_indices") if reuse is not None else None
        n = reuse["n"] if reuse is not None else 0
        cache = reuse["cache"][layer_id - 1] if indices is not None else None
        w_up, b_up, w_down, b_down = self._weights(layer_id)
        x_next, _, clean = ffn_block(
            x, update, normalized, block.modulation, state.time_mod, w_up, b_up, w_down, b_down,
            indices, cache, n, self.plan_id, self.eps[layer_id], False,
        )
        if reuse is not None:
            state.extras["token_outputs"].append(clean)
        state.hidden_states = x_next
        return state

    def ffn_at_layer_for_compile(self, layer_id, state, normalized, x):
        return self._run(layer_id, state, x, None, normalized)

    def post_attn_ffn(self, layer_id, state, x, cross_output):
        return self._run(layer_id, state, x, cross_output, None)

    def close(self):
        release_block_plan(self.plan_id)

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
