"""ctypes binding of libwamffn.so, the sm_100a CUDA library behind every op.

The library is built in-tree (``waminfer_b200/libwamffn.so``) by
``waminfer_b200.build``.  There is no fallback: if the library is missing or
was built without sm_100a code, every op raises instead of silently running
some other implementation.
"""

from __future__ import annotations

import ctypes
import os
import threading
from pathlib import Path

LIB_PATH = Path(__file__).with_name("libwamffn.so")

WAMFFN_OK = 0
WAMFFN_ERR_INVALID = 1
WAMFFN_ERR_CUDA = 2
WAMFFN_ERR_UNSUPPORTED = 3
WAMFFN_ERR_CAPTURE = 4
WAMFFN_ERR_DEVICE = 5

DEV_TIMEOUT = 1
DEV_BAD_INDEX = 2

SELF_INPUT = 0
SELF_RESIDUAL = 1
CROSS_RESIDUAL = 2
FFN_RESIDUAL = 3

# Every symbol include/wamffn.h declares; tests check the library exports them all.
EXPORTED_SYMBOLS = (
    "wamffn_abi_version",
    "wamffn_last_error",
    "wamffn_launch_count",
    "wamffn_linear_plan_create",
    "wamffn_linear_plan_destroy",
    "wamffn_linear_run",
    "wamffn_linear_configuration",
    "wamffn_linear_plan_set_layout",
    "wamffn_linear_status",
    "wamffn_linear_run_static",
    "wamffn_selftest_wait_timeout",
    "wamffn_ffn_run",
    "wamffn_modulated_norm",
    "wamffn_block_plan_create",
    "wamffn_block_plan_destroy",
    "wamffn_block_run",
    "wamffn_block_status",
    "wamffn_block_configuration",
    "wamffn_block_plan_set_splits",
    "wamffn_block_plan_set_streamk",
    "wamffn_masked_attention",
    "wamffn_joint_first_frame_attention",
    "wamffn_current_frame_attention",
    "wamffn_rgb_mandatory",
    "wamffn_select_tokens",
    "wamffn_pack_weight",
    "wamffn_trace_enable",
    "wamffn_stack_run",
    "wamffn_stack_run_tp",
)

# int allreduce(void* user, float* buffer, int64_t count, void* stream)
ALLREDUCE_FN = ctypes.CFUNCTYPE(ctypes.c_int, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int64, ctypes.c_void_p)

LINEAR_GELU = 1
WEIGHTS_PACKED = 2


class NormArgs(ctypes.Structure):
    """Mirror of ``wamffn_norm_args``."""

    _fields_ = [
        ("x", ctypes.c_void_p),
        ("x_stride", ctypes.c_int64),
        ("update", ctypes.c_void_p),
        ("update_stride", ctypes.c_int64),
        ("mod", ctypes.c_void_p),
        ("previous", ctypes.c_void_p),
        ("time", ctypes.c_void_p),
        ("time_stride", ctypes.c_int64),
        ("weight", ctypes.c_void_p),
        ("bias", ctypes.c_void_p),
        ("y", ctypes.c_void_p),
        ("norm", ctypes.c_void_p),
        ("rows", ctypes.c_int),
        ("dim", ctypes.c_int),
        ("mode", ctypes.c_int),
        ("eps", ctypes.c_float),
    ]


class AttentionArgs(ctypes.Structure):
    """Mirror of ``wamffn_attention_args``."""

    _fields_ = [
        ("q", ctypes.c_void_p),
        ("q_row_stride", ctypes.c_int64),
        ("q_batch_stride", ctypes.c_int64),
        ("k", ctypes.c_void_p),
        ("k_row_stride", ctypes.c_int64),
        ("k_batch_stride", ctypes.c_int64),
        ("v", ctypes.c_void_p),
        ("v_row_stride", ctypes.c_int64),
        ("v_batch_stride", ctypes.c_int64),
        ("mask", ctypes.c_void_p),
        ("mask_strides", ctypes.c_int64 * 4),
        ("out", ctypes.c_void_p),
        ("status", ctypes.c_void_p),
        ("batch", ctypes.c_int),
        ("nq", ctypes.c_int),
        ("nk", ctypes.c_int),
        ("heads", ctypes.c_int),
        ("head_dim", ctypes.c_int),
        ("key_split", ctypes.c_int),
    ]


class RowsView(ctypes.Structure):
    """Mirror of ``wamffn_rows_view``."""

    _fields_ = [("data", ctypes.c_void_p), ("row_stride", ctypes.c_int64), ("batch_stride", ctypes.c_int64)]


class JointAttentionArgs(ctypes.Structure):
    """Mirror of ``wamffn_joint_attention_args``."""

    _fields_ = [
        ("q", RowsView),
        ("k", RowsView),
        ("v", RowsView),
        ("out", ctypes.c_void_p),
        ("status", ctypes.c_void_p),
        ("batch", ctypes.c_int),
        ("count", ctypes.c_int),
        ("video", ctypes.c_int),
        ("first", ctypes.c_int),
        ("heads", ctypes.c_int),
        ("head_dim", ctypes.c_int),
        ("key_split", ctypes.c_int),
    ]


class CurrentFrameArgs(ctypes.Structure):
    """Mirror of ``wamffn_current_frame_args``."""

    _fields_ = [
        *[(name, RowsView) for name in ("qv", "qa", "ck", "kv", "ka", "cv", "vv", "va")],
        ("ov", ctypes.c_void_p),
        ("oa", ctypes.c_void_p),
        ("status", ctypes.c_void_p),
        ("batch", ctypes.c_int),
        ("nc", ctypes.c_int),
        ("nv", ctypes.c_int),
        ("na", ctypes.c_int),
        ("heads", ctypes.c_int),
        ("head_dim", ctypes.c_int),
        ("key_split", ctypes.c_int),
    ]


class BlockArgs(ctypes.Structure):
    """Mirror of ``wamffn_block_args``."""

    _fields_ = [
        ("x", ctypes.c_void_p),
        ("update", ctypes.c_void_p),
        ("normalized", ctypes.c_void_p),
        ("mod", ctypes.c_void_p),
        ("time", ctypes.c_void_p),
        ("time_stride", ctypes.c_int64),
        ("w_up", ctypes.c_void_p),
        ("b_up", ctypes.c_void_p),
        ("w_down", ctypes.c_void_p),
        ("b_down", ctypes.c_void_p),
        ("weights_packed", ctypes.c_int),
        ("indices", ctypes.c_void_p),
        ("index_bytes", ctypes.c_int),
        ("rows", ctypes.c_int),
        ("seq", ctypes.c_int),
        ("cache_rows", ctypes.c_int),
        ("cache_in", ctypes.c_void_p),
        ("cache_out", ctypes.c_void_p),
        ("y", ctypes.c_void_p),
        ("output", ctypes.c_void_p),
        ("x_out", ctypes.c_void_p),
        ("eps", ctypes.c_float),
    ]


class SelectArgs(ctypes.Structure):
    """Mirror of ``wamffn_select_args``."""

    _fields_ = [
        ("now", ctypes.c_void_p),
        ("now_stride", ctypes.c_int64),
        ("before", ctypes.c_void_p),
        ("mandatory", ctypes.c_void_p),
        ("n", ctypes.c_int),
        ("dim", ctypes.c_int),
        ("count", ctypes.c_int),
        ("seq", ctypes.c_int),
        ("indices", ctypes.c_void_p),
        ("features_out", ctypes.c_void_p),
    ]


class LayerWeights(ctypes.Structure):
    """Mirror of ``wamffn_layer_weights``."""

    _fields_ = [
        ("w_up", ctypes.c_void_p),
        ("b_up", ctypes.c_void_p),
        ("w_down", ctypes.c_void_p),
        ("b_down", ctypes.c_void_p),
        ("mod", ctypes.c_void_p),
    ]


class StackArgs(ctypes.Structure):
    """Mirror of ``wamffn_stack_args``."""

    _fields_ = [
        ("layers", ctypes.c_int),
        ("weights", ctypes.POINTER(LayerWeights)),
        ("weights_packed", ctypes.c_int),
        ("x", ctypes.c_void_p),
        ("time", ctypes.c_void_p),
        ("time_stride", ctypes.c_int64),
        ("seq", ctypes.c_int),
        ("indices", ctypes.c_void_p),
        ("index_bytes", ctypes.c_int),
        ("rows", ctypes.c_int),
        ("first_gathered_layer", ctypes.c_int),
        ("cache_rows", ctypes.c_int),
        ("cache_in", ctypes.c_void_p),
        ("cache_out", ctypes.c_void_p),
        ("x_out", ctypes.c_void_p),
        ("eps", ctypes.c_float),
    ]


class WamffnError(RuntimeError):
    """A libwamffn entry point returned a non-zero status."""

    def __init__(self, code: int, message: str):
        super().__init__(f"libwamffn error {code}: {message}")
        self.code = code


_lock = threading.Lock()
_lib = None


def _declare(lib):
    vp, i, u32p = ctypes.c_void_p, ctypes.c_int, ctypes.POINTER(ctypes.c_uint32)
    lib.wamffn_abi_version.restype = i
    lib.wamffn_last_error.restype = ctypes.c_char_p
    lib.wamffn_launch_count.restype = ctypes.c_ulonglong
    lib.wamffn_linear_plan_create.argtypes = [i, i, i, i, i, i, ctypes.POINTER(vp)]
    lib.wamffn_linear_plan_destroy.argtypes = [vp]
    lib.wamffn_linear_run.argtypes = [vp, vp, vp, vp, vp, vp]
    lib.wamffn_linear_configuration.argtypes = [vp, u32p, i]
    lib.wamffn_linear_plan_set_layout.argtypes = [vp, i, i]
    lib.wamffn_linear_status.argtypes = [vp, u32p, i]
    lib.wamffn_linear_run_static.argtypes = [i, vp, i, i, i, i, i, vp, vp, vp, vp, vp]
    lib.wamffn_selftest_wait_timeout.argtypes = [vp, vp, ctypes.c_int64]
    lib.wamffn_ffn_run.argtypes = [vp, vp, vp, vp, vp, vp, vp, vp, vp]
    lib.wamffn_modulated_norm.argtypes = [vp, ctypes.POINTER(NormArgs)]
    lib.wamffn_block_plan_create.argtypes = [i, i, i, i, i, i, ctypes.POINTER(vp)]
    lib.wamffn_block_plan_destroy.argtypes = [vp]
    lib.wamffn_block_run.argtypes = [vp, vp, ctypes.POINTER(BlockArgs)]
    lib.wamffn_block_status.argtypes = [vp, u32p, i]
    lib.wamffn_block_configuration.argtypes = [vp, i, u32p, i]
    lib.wamffn_block_plan_set_splits.argtypes = [vp, i, i]
    lib.wamffn_block_plan_set_streamk.argtypes = [vp, i]
    lib.wamffn_masked_attention.argtypes = [vp, ctypes.POINTER(AttentionArgs)]
    lib.wamffn_joint_first_frame_attention.argtypes = [vp, ctypes.POINTER(JointAttentionArgs)]
    lib.wamffn_current_frame_attention.argtypes = [vp, ctypes.POINTER(CurrentFrameArgs)]
    lib.wamffn_rgb_mandatory.argtypes = [vp, vp, vp, i, i, i, i, vp]
    lib.wamffn_select_tokens.argtypes = [vp, ctypes.POINTER(SelectArgs)]
    lib.wamffn_pack_weight.argtypes = [vp, vp, vp, i, i]
    lib.wamffn_trace_enable.argtypes = [i, vp, i]
    lib.wamffn_stack_run.argtypes = [vp, vp, ctypes.POINTER(StackArgs)]
    lib.wamffn_stack_run_tp.argtypes = [vp, vp, ctypes.POINTER(StackArgs), vp, ALLREDUCE_FN, vp]
    for name in EXPORTED_SYMBOLS:
        if name not in ("wamffn_last_error", "wamffn_launch_count"):
            getattr(lib, name).restype = i


def lib():
    """Returns the loaded library, loading it on first use (raises if absent)."""
    global _lib
    if _lib is None:
        with _lock:
            if _lib is None:
                path = os.environ.get("WAMFFN_LIBRARY", str(LIB_PATH))
                if not Path(path).exists():
                    raise ImportError(
                        f"{path} is missing: build it with `python -c 'import __graft_entry__ as g; g.build()'` "
                        "or `python -m waminfer_b200.build` (there is no CPU or library fallback)"
                    )
                handle = ctypes.CDLL(path)
                _declare(handle)
                if handle.wamffn_abi_version() != 2:
                    raise ImportError(f"{path} has ABI {handle.wamffn_abi_version()}, expected 2")
                _lib = handle
    return _lib


def check(status: int) -> None:
    """Raises WamffnError for a non-zero status with the library's message."""
    if status != WAMFFN_OK:
        message = lib().wamffn_last_error().decode(errors="replace")
        raise WamffnError(status, message)


def launch_count() -> int:
    return int(lib().wamffn_launch_count())
