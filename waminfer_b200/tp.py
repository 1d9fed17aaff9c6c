"""Tensor-parallel FFN stack: the hidden dimension split across ranks.

The reference runs every FFN on one GPU (``WAMInfer/blocks.py:252-258`` over
``WAMInfer/ffn.py:96-107``).  This secondary mode splits h = 14336 the
Megatron way: rank r holds rows [r*h/g, (r+1)*h/g) of W_up and b_up (column
parallel: its share of the hidden features) and the matching columns of W_down
(row parallel over K).  Each rank computes

    Y_r = GELU(X W_up,r^T + b_up,r) W_down,r^T          (fp32, [M, d])

and one sum over the ranks per layer gives the down projection before its
bias; the bias, gated residual, history scatter and the next layer's norm then
run once on the reduced sum, identically on every rank
(``wamffn_stack_run_tp``).  The sum is a ``torch.distributed.all_reduce``
(NCCL over NVLink on B200, gloo on CPU) issued from the library's host
callback on the current stream.

Every rank receives the same inputs (x, time, indices, history) and produces
the same outputs, so the history and residual stay replicated.
"""

from __future__ import annotations

import ctypes

import torch
import torch.distributed as dist

from waminfer_b200 import _lib
from waminfer_b200.stack import FFNStack, Geometry, LayerWeights, Request

# Hidden columns per rank are a multiple of one 2-SM UMMA pair tile.
SHARD_GRANULE = 256


def shard_bounds(h: int, rank: int, world: int) -> tuple[int, int]:
    """Hidden columns [lo, hi) held by `rank` of `world`."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"rank {rank} outside a world of {world}")
    if h % (SHARD_GRANULE * world):
        raise ValueError(f"h={h} does not split into {world} shards of whole {SHARD_GRANULE}-column tiles")
    per = h // world
    return rank * per, (rank + 1) * per


def slice_layer(w: LayerWeights, rank: int, world: int) -> LayerWeights:
    """This rank's shard of one layer: W_up / b_up rows and W_down columns of
    its hidden range; the down bias and the modulation stay whole (they apply
    after the reduction)."""
    lo, hi = shard_bounds(w.w_up.shape[0], rank, world)
    return LayerWeights(w.w_up[lo:hi].contiguous(), w.b_up[lo:hi].contiguous(), w.w_down[:, lo:hi].contiguous(),
                        w.b_down, w.mod)


def slice_weights(weights: list[LayerWeights], rank: int, world: int) -> list[LayerWeights]:
    return [slice_layer(w, rank, world) for w in weights]


class TPStack(FFNStack):
    """The FFN stack of one tensor-parallel rank (weights: this rank's shards)."""

    def __init__(self, shards: list[LayerWeights], geo: Geometry, device, group=None, eps: float = 1e-6):
        super().__init__(shards, geo, device, eps)
        self.group = group
        self.world = dist.get_world_size(group)
        self.reduce = torch.empty(geo.seq, geo.d, dtype=torch.float32, device=self.device)
        self._callback = _lib.ALLREDUCE_FN(self._allreduce)
        self.error: BaseException | None = None

    def _allreduce(self, user, buffer, count, stream) -> int:
        # Host callback of wamffn_stack_run_tp: sum this layer's [rows, d]
        # down projection over the ranks, in place, on the current stream.
        try:
            if buffer != self.reduce.data_ptr():
                raise RuntimeError("allreduce called on an unexpected buffer")
            dist.all_reduce(self.reduce.view(-1)[:count], group=self.group)
            return 0
        except BaseException as exc:  # reported through the library's status
            self.error = exc
            return _lib.WAMFFN_ERR_CUDA

    def enqueue_pass(self, x_in, x_final, time, stream: int | None = None, reuse: Request | None = None) -> None:
        """One pass of the L layers with one all-reduce per layer.  Runs on the
        current stream (the collective is issued there by torch)."""
        current = torch.cuda.current_stream(self.device).cuda_stream
        if stream is not None and stream != current:
            raise ValueError("the tensor-parallel stack runs on the current stream")
        a = self._stack_args(x_in, x_final, time, reuse)
        self.error = None
        status = _lib.lib().wamffn_stack_run_tp(self.plan.handle, current, ctypes.byref(a), self.reduce.data_ptr(),
                                                self._callback, None)
        if self.error is not None:
            raise RuntimeError(f"tensor-parallel all-reduce failed: {self.error}") from self.error
        _lib.check(status)

    def launches_per_request(self) -> int:
        return 2 * (1 + 4 * self.geo.layers)
