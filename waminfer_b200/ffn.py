"""Per-model BF16 FFN plans backed by hand-written sm_100a kernels.

Host-side mirror of the reference's ``WAMInfer/ffn.py`` (PreparedFFN,
the module-global plan registry and the ``prepared_ffn_linear_v1`` custom op),
with cuBLASLt replaced by libwamffn's tcgen05 GEMMs:

* the up projection fuses bias and tanh-GELU in its epilogue with no bf16
  rounding before the GELU (the reference's GELU_BIAS epilogue contract,
  ``WAMInfer/ffn.py:1-6``, ``WAMInfer/_cublaslt_inference.cpp:73``);
* the down projection is split-K with a deterministic reduction + bias.

Plans and their workspaces are owned per model, never process-wide
(``WAMInfer/ffn.py:5-6``).  Like the reference, ``prepare`` keeps a repacked
copy of every weight, refreshed when the parameter's signature changes; the
copy is tile-packed ([out/128, in/64, 128, 64]) so that the GEMMs stream each
128 x 64 weight tile as one contiguous 16 KB block from HBM.
"""

from __future__ import annotations

import ctypes
from itertools import count

import torch

from waminfer_b200 import _lib
from waminfer_b200.blocks import _parameter_signature

_PLANS: dict[int, "Plan"] = {}
_IDS = count()


def _stream_handle(device: torch.device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def packed_shape(n_out: int, k_in: int) -> tuple[int, int, int, int]:
    return (n_out // 128, k_in // 64, 128, 64)


def pack_weight(weight: torch.Tensor) -> torch.Tensor:
    """Tile-packed copy of an [out, in] bf16 weight: [out/128, in/64, 128, 64],
    so every 128 x 64 tile a GEMM CTA streams is one contiguous 16 KB block
    (``wamffn_pack_weight``; the reference makes its repacked copy at the same
    point, ``WAMInfer/ffn.py:82-88``)."""
    if weight.dim() != 2 or weight.dtype != torch.bfloat16 or not weight.is_cuda:
        raise ValueError("pack_weight expects a CUDA bf16 [out, in] matrix")
    n_out, k_in = weight.shape
    src = weight.contiguous()
    dst = torch.empty(packed_shape(n_out, k_in), dtype=weight.dtype, device=weight.device)
    with torch.cuda.device(weight.device):
        _lib.check(_lib.lib().wamffn_pack_weight(_stream_handle(weight.device), src.data_ptr(), dst.data_ptr(),
                                                 n_out, k_in))
    return dst


class Plan:
    """One linear GEMM plan on one device (replaces ``Plan`` of
    ``WAMInfer/_cublaslt_inference.cpp:41-190``).

    Same constructor and ``run`` contract as the reference: ``x`` fixes the row
    count, ``weight``/``bias`` the output shape; ``exhaustive`` times the
    candidate split-K factors on the device; planning is refused during CUDA
    graph capture (``cpp:167-168``).
    """

    def __init__(self, x: torch.Tensor, weight: torch.Tensor, bias: torch.Tensor, exhaustive: bool, gelu: bool = False,
                 packed: bool | None = None):
        if not (x.is_cuda and weight.device == x.device and bias.device == x.device):
            raise RuntimeError("Plan tensors must share one CUDA device")
        if not (x.dtype == torch.bfloat16 and weight.dtype == x.dtype and bias.dtype == x.dtype):
            raise RuntimeError("Plan tensors must be bfloat16")
        if packed is None:
            packed = weight.dim() == 4
        n = weight.shape[0] * 128 if packed else weight.shape[0]
        k = weight.shape[1] * 64 if packed else weight.shape[1]
        if not (x.dim() == 2 and bias.dim() == 1 and bias.numel() == n and k == x.shape[1]):
            raise RuntimeError("Plan shapes do not form x[m,k] . weight[n,k]^T + bias[n]")
        if torch.cuda.is_current_stream_capturing():
            raise RuntimeError("GEMM tuning must finish before CUDA Graph capture")
        self.m, self.n, self.k = x.shape[0], n, k
        self.gelu = bool(gelu)
        self.packed = bool(packed)
        self.device = x.device
        flags = (_lib.LINEAR_GELU if self.gelu else 0) | (_lib.WEIGHTS_PACKED if self.packed else 0)
        handle = ctypes.c_void_p()
        _lib.check(_lib.lib().wamffn_linear_plan_create(
            x.device.index, self.m, self.n, self.k, flags, int(bool(exhaustive)), ctypes.byref(handle)))
        self._handle = handle

    def run(self, x: torch.Tensor, weight: torch.Tensor, bias: torch.Tensor) -> torch.Tensor:
        """Replaces ``Plan::run`` (``cpp:177-188``): checks the bound tensors and
        launches into a freshly allocated output on the current stream."""
        if self._handle is None:
            raise RuntimeError("plan is closed")
        if not (x.device == self.device and weight.device == x.device and bias.device == x.device):
            raise RuntimeError("tensors are not on the plan's device")
        if not (x.dtype == torch.bfloat16 and weight.dtype == x.dtype and bias.dtype == x.dtype):
            raise RuntimeError("tensors must be bfloat16")
        if not (x.is_contiguous() and x.dim() == 2 and x.shape[0] == self.m and x.shape[1] == self.k):
            raise RuntimeError(f"x must be contiguous [{self.m}, {self.k}]")
        if self.packed:
            if not (weight.is_contiguous() and tuple(weight.shape) == packed_shape(self.n, self.k)):
                raise RuntimeError(f"weight must be the packed copy of a [{self.n}, {self.k}] matrix")
        elif not (weight.dim() == 2 and weight.shape == (self.n, self.k) and weight.stride() == (self.k, 1)):
            raise RuntimeError(f"weight must be a contiguous [{self.n}, {self.k}] (out, in) matrix")
        if not (bias.is_contiguous() and bias.numel() == self.n):
            raise RuntimeError("bias must be contiguous with one entry per output feature")
        out = torch.empty((self.m, self.n), dtype=x.dtype, device=x.device)
        _lib.check(_lib.lib().wamffn_linear_run(
            self._handle, _stream_handle(x.device), x.data_ptr(), weight.data_ptr(), bias.data_ptr(), out.data_ptr()))
        return out

    def selected_configuration(self) -> list[int]:
        """{feature_tile, token_pad, mma_count, stages, split_k, tmem_columns, tuned}
        (the reference reports its cuBLASLt config ids, ``cpp:189``)."""
        values = (ctypes.c_uint32 * 7)()
        _lib.check(_lib.lib().wamffn_linear_configuration(self._handle, values, 7))
        return list(values)

    def layout(self) -> dict:
        """The GEMM layout the plan runs: split-K factor, token groups and
        stream-K CTA groups (0: data-parallel grid)."""
        values = (ctypes.c_uint32 * 9)()
        _lib.check(_lib.lib().wamffn_linear_configuration(self._handle, values, 9))
        return {"split_k": int(values[4]), "token_groups": int(values[8]), "streamk_groups": int(values[7])}

    def set_layout(self, split_k: int, token_groups: int = 1) -> None:
        """Overrides the tuner's choice (K split into ``split_k`` slices, rows
        cut into ``token_groups`` groups); synchronises the device."""
        if self._handle is None:
            raise RuntimeError("plan is closed")
        if torch.cuda.is_current_stream_capturing():
            raise RuntimeError("a plan's layout must be set before CUDA Graph capture")
        _lib.check(_lib.lib().wamffn_linear_plan_set_layout(self._handle, int(split_k), int(token_groups)))

    def status(self, clear: bool = True) -> int:
        """Device status word (timeout / bad-index bits); synchronises the device."""
        value = ctypes.c_uint32()
        _lib.check(_lib.lib().wamffn_linear_status(self._handle, ctypes.byref(value), int(clear)))
        return int(value.value)

    def close(self) -> None:
        if getattr(self, "_handle", None) is not None:
            _lib.lib().wamffn_linear_plan_destroy(self._handle)
            self._handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


@torch.library.custom_op("wam_ffn::prepared_ffn_linear_v1", mutates_args=())
def prepared_linear(x: torch.Tensor, weight: torch.Tensor, bias: torch.Tensor, plan_id: int) -> torch.Tensor:
    return _PLANS[plan_id].run(x, weight, bias)


@prepared_linear.register_fake
def _fake_linear(x, weight, bias, plan_id):
    n = weight.shape[0] * 128 if weight.dim() == 4 else weight.shape[0]
    return torch.empty((x.shape[0], n), dtype=x.dtype, device=x.device)


class PreparedFFN:
    """Drop-in for the reference's ``PreparedFFN`` (``WAMInfer/ffn.py:48-118``):
    same ``prepare(rows)`` / ``forward(layer_id, inputs)`` / ``close()`` API,
    same plan keys, same native fallback for an unprepared row count."""

    max_plans = 32

    def __init__(self, backbone):
        self.backbone = backbone
        self.weights = {}
        self.signatures = {}
        self.plans = {}
        self.keys = {}

    def _plan(self, weight, bias, rows, gelu):
        key = (weight.device, rows, tuple(weight.shape), weight.stride(), gelu)
        if key not in self.keys:
            if len(self.keys) >= self.max_plans:
                raise RuntimeError("FFN preparation supports at most 32 device/shape plans per model.")
            k = weight.shape[1] * 64 if weight.dim() == 4 else weight.shape[1]
            x = torch.empty(rows, k, device=weight.device, dtype=weight.dtype)
            plan = Plan(x, weight, bias, True, gelu)
            plan_id = next(_IDS)
            _PLANS[plan_id] = plan
            self.keys[key] = plan_id
        return self.keys[key]

    def prepare(self, rows):
        """Validates the FFN layers, refreshes weights whose signature changed and
        builds plans for every (layer, row count); returns whether anything changed."""
        if torch.is_grad_enabled() or self.backbone.training:
            raise RuntimeError("FFN preparation requires eval mode and disabled gradients.")
        changed = False
        for layer_id, block in enumerate(self.backbone.dit.blocks):
            ffn = block.ffn
            if not isinstance(ffn[1], torch.nn.GELU) or ffn[1].approximate != "tanh":
                raise ValueError("Fused FFN requires tanh GELU.")
            packed = []
            for index in (0, 2):
                layer = ffn[index]
                if layer.weight.dtype != torch.bfloat16 or layer.weight.device.type != "cuda" or layer.bias is None:
                    raise ValueError("Fused FFN requires CUDA BF16 linear layers with bias.")
                key = (layer_id, index)
                signature = _parameter_signature(layer.weight)
                if self.signatures.get(key) != signature:
                    self.weights[key] = pack_weight(layer.weight.detach())
                    self.signatures[key] = signature
                    changed = True
                packed.append(self.weights[key])
            for m in rows:
                key = (layer_id, m)
                ids = (self._plan(packed[0], ffn[0].bias, m, True), self._plan(packed[1], ffn[2].bias, m, False))
                changed |= self.plans.get(key) != ids
                self.plans[key] = ids
        return changed

    def forward(self, layer_id, inputs):
        ffn = self.backbone.dit.blocks[layer_id].ffn
        rows = inputs.numel() // inputs.shape[-1]
        if (layer_id, rows) not in self.plans:
            # Unprepared geometry: keep the native FFN instead of planning during capture.
            return ffn(inputs)
        up, down = self.plans[layer_id, rows]
        x = inputs.reshape(rows, inputs.shape[-1])
        x = prepared_linear(x, self.weights[layer_id, 0], ffn[0].bias, up)
        x = prepared_linear(x, self.weights[layer_id, 2], ffn[2].bias, down)
        return x.reshape(*inputs.shape[:-1], x.shape[-1])

    def __del__(self):
        self.close()

    def close(self):
        for plan_id in self.keys.values():
            plan = _PLANS.pop(plan_id, None)
            if plan is not None:
                plan.close()
        self.keys.clear()
        self.plans.clear()
        self.weights.clear()
        self.signatures.clear()
