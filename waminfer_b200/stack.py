"""30-layer video-DiT FFN stack on the fused block kernels.

A *request* here is the FFN work of one WAMInfer observation under the 2F
motion-adaptive schedule with cross-observation token reuse
(``WAMInfer/runtime.py:157-201``, ``WAMInfer/approximation.py:70-84``): the
Transformer runs at Euler updates 0 and 3 only, so the FFN stack runs twice.

* update 0 (token reuse): layer 0 recomputes every row
  (``WAMInfer/blocks.py:248``); layers 1..L-1 gather the ``count`` selected
  current-frame rows plus every future-frame and action row, and scatter the
  recomputed current rows into the per-layer history ``[L-1, n, d]``
  (``WAMInfer/blocks.py:249-264``, ``WAMInfer/runtime.py:263``).
* update 3 (full refresh): every row of every layer.

A pass is one ``wamffn_stack_run``: up GEMM, down GEMM and one fused
layer-boundary kernel per layer (split-K reduction, history scatter, gated
residual, next layer's norm + gather).  Everything a request touches is
preallocated, so a request (or a batch of them) can be captured into one
CUDA graph.

Lanes: requests share nothing but the weights, so ``FFNStack(lanes=k)`` runs a
batch of requests on k streams forked from the caller's stream (one block plan,
i.e. one set of scratch buffers, per lane; the packed weights are shared) and
joins them back.  The hardware then schedules CTAs of different requests'
kernels side by side: SMs the up projection leaves idle (56 UMMA pairs on 148
SMs), the layer-boundary kernels and the launch ramps are filled by the other
lanes.  Each request's own launches keep their order and their results are
bit-identical to a single lane with the same split-K factor.
"""

from __future__ import annotations

import ctypes
import os
from dataclasses import dataclass

import torch

from waminfer_b200 import _lib
from waminfer_b200.blocks import BlockPlan


@dataclass
class LayerWeights:
    w_up: torch.Tensor    # [h, d]
    b_up: torch.Tensor    # [h]
    w_down: torch.Tensor  # [d, h]
    b_down: torch.Tensor  # [d]
    mod: torch.Tensor     # [1, 6, d] block.modulation


def make_weights(layers: int, d: int, h: int, device, seed: int = 0) -> list[LayerWeights]:
    """Seeded synthetic weights: W ~ N(0, 0.02), biases ~ N(0, 0.01), modulation ~ N(0, 0.1)."""
    out = []
    for layer in range(layers):
        g = torch.Generator(device=device).manual_seed(seed * 1000 + layer)

        def rnd(*shape, std):
            return (torch.randn(*shape, device=device, generator=g) * std).to(torch.bfloat16)

        out.append(LayerWeights(rnd(h, d, std=0.02), rnd(h, std=0.01), rnd(d, h, std=0.02), rnd(d, std=0.01),
                                rnd(1, 6, d, std=0.1)))
    return out


def ffn_flops(rows: int, d: int, h: int) -> int:
    """Algorithmic FLOPs of one FFN layer over `rows` real rows: 2 GEMMs of 2*M*d*h."""
    return 4 * rows * d * h


@dataclass
class Geometry:
    """Row counts of one request (default: 384x320 RGB, 9 frames -> 3 latent
    frames of 12x10 tokens, 32 action rows carried with the video rows)."""

    layers: int = 30
    d: int = 3072
    h: int = 14336
    current: int = 120     # n: current-observation rows (cacheable)
    future: int = 240      # future-frame rows (always recomputed)
    action: int = 32       # action rows (always recomputed)
    count: int = 32        # refreshed current rows (capacity bucket)

    @property
    def seq(self) -> int:
        return self.current + self.future + self.action

    @property
    def reuse_rows(self) -> int:
        return self.count + self.future + self.action

    def request_rows(self) -> list[int]:
        """Rows of each of the 2*L layer passes of one 2F request."""
        return [self.seq] + [self.reuse_rows] * (self.layers - 1) + [self.seq] * self.layers

    def request_flops(self) -> int:
        return sum(ffn_flops(m, self.d, self.h) for m in self.request_rows())


class Request:
    """Device buffers of one request: inputs of both passes, the history it
    reads and the history it writes."""

    def __init__(self, geo: Geometry, device, seed: int, history_in: torch.Tensor | None = None):
        g = torch.Generator(device=device).manual_seed(10_000 + seed)
        s, d = geo.seq, geo.d

        def rnd(*shape, std=1.0):
            return (torch.randn(*shape, device=device, generator=g) * std).to(torch.bfloat16)

        self.x = [rnd(s, d), rnd(s, d)]                    # residual stream entering update 0 / update 3
        self.time = [rnd(s, 6, d, std=0.1), rnd(s, 6, d, std=0.1)]  # per-token time modulation per update
        cg = torch.Generator().manual_seed(20_000 + seed)
        chosen = torch.randperm(geo.current, generator=cg)[: geo.count].sort().values
        self.indices = torch.cat((chosen, torch.arange(geo.current, s))).to(torch.int64).to(device)
        self.history_in = history_in if history_in is not None else rnd(geo.layers - 1, geo.current, d)
        self.history_out = torch.empty_like(self.history_in)
        self.out = [torch.empty(s, d, device=device, dtype=torch.bfloat16) for _ in range(2)]


class FFNStack:
    """L fused FFN blocks over resident weights on one device."""

    def __init__(self, weights: list[LayerWeights], geo: Geometry, device, eps: float = 1e-6, lanes: int = 1,
                 down_splits: int | None = None, streamk: bool | None = None):
        from waminfer_b200.ffn import pack_weight

        if lanes < 1:
            raise ValueError("lanes must be at least 1")
        pass_flag = os.environ.get("WAMFFN_PASS", "")
        if lanes > 1 and pass_flag and pass_flag[0] not in "0nNfF":  # the library's reading of the flag
            # The persistent pass kernel's grid barriers need every SM: lanes would starve each other.
            raise ValueError("WAMFFN_PASS=1 (one persistent launch per pass) cannot run in concurrent lanes")
        self.weights, self.geo, self.device, self.eps = weights, geo, torch.device(device), eps
        # Tile-packed copies streamed by the GEMMs (one contiguous 16 KB block per tile).
        self.packed = [(pack_weight(w.w_up), pack_weight(w.w_down)) for w in weights]
        # d_hidden from the weights: a tensor-parallel rank holds h / world columns.
        self.plans = [BlockPlan(self.device, max_rows=geo.seq, max_seq=geo.seq, d_model=geo.d,
                                d_hidden=weights[0].w_up.shape[0]) for _ in range(lanes)]
        self.plan = self.plans[0]
        if down_splits is not None:
            for plan in self.plans:
                plan.set_splits(0, down_splits)
        if streamk is not None:
            self.set_streamk(streamk)
        self._streams = [torch.cuda.Stream(self.device) for _ in range(lanes)] if lanes > 1 else []
        self._pingpong = [torch.empty(geo.seq, geo.d, device=device, dtype=torch.bfloat16) for _ in range(2)]
        self._keep = []  # argument structs referenced by enqueued launches
        self._layer_array = (_lib.LayerWeights * len(weights))()
        for i, (w, (w_up, w_down)) in enumerate(zip(weights, self.packed)):
            self._layer_array[i] = _lib.LayerWeights(w_up.data_ptr(), w.b_up.data_ptr(), w_down.data_ptr(),
                                                     w.b_down.data_ptr(), w.mod.data_ptr())

    def _args(self, layer: int, x, x_out, time, indices=None, cache_in=None, cache_out=None, n=0):
        w = self.weights[layer]
        w_up, w_down = self.packed[layer]
        a = _lib.BlockArgs()
        a.x = x.data_ptr()
        a.mod = w.mod.data_ptr()
        a.time = time.data_ptr()
        a.time_stride = 6 * self.geo.d
        a.w_up, a.b_up = w_up.data_ptr(), w.b_up.data_ptr()
        a.w_down, a.b_down = w_down.data_ptr(), w.b_down.data_ptr()
        a.weights_packed = 1
        if indices is not None:
            a.indices = indices.data_ptr()
            a.index_bytes = indices.element_size()
            a.rows = indices.numel()
        else:
            a.rows = self.geo.seq
        a.seq = self.geo.seq
        a.cache_rows = n
        a.cache_in = None if cache_in is None else cache_in.data_ptr()
        a.cache_out = None if cache_out is None else cache_out.data_ptr()
        a.x_out = x_out.data_ptr()
        a.eps = self.eps
        return a

    def _stack_args(self, x_in, x_final, time, reuse: "Request | None") -> "_lib.StackArgs":
        geo = self.geo
        a = _lib.StackArgs()
        a.layers = len(self.weights)
        a.weights = ctypes.cast(self._layer_array, ctypes.POINTER(_lib.LayerWeights))
        a.weights_packed = 1
        a.x = x_in.data_ptr()
        a.time = time.data_ptr()
        a.time_stride = 6 * geo.d
        a.seq = geo.seq
        if reuse is not None:
            a.indices = reuse.indices.data_ptr()
            a.index_bytes = reuse.indices.element_size()
            a.rows = reuse.indices.numel()
            a.first_gathered_layer = 1
            a.cache_rows = geo.current
            a.cache_in = reuse.history_in.data_ptr()
            a.cache_out = reuse.history_out.data_ptr()
        a.x_out = x_final.data_ptr()
        a.eps = self.eps
        self._keep.append(a)
        return a

    def enqueue_pass(self, x_in, x_final, time, stream: int, reuse: "Request | None" = None,
                     plan: BlockPlan | None = None) -> None:
        """Runs the L layers with one ``wamffn_stack_run`` (fused layer
        boundaries); with `reuse`, layers 1.. gather its indices and read /
        write its history.  `plan` picks a lane's scratch (default: lane 0)."""
        a = self._stack_args(x_in, x_final, time, reuse)
        plan = self.plan if plan is None else plan
        _lib.check(_lib.lib().wamffn_stack_run(plan.handle, stream, ctypes.byref(a)))

    def enqueue_pass_blocks(self, x_in, x_final, time, stream: int, reuse: "Request | None" = None) -> None:
        """Same pass as ``enqueue_pass`` with one ``wamffn_block_run`` per layer
        (four kernels per layer, no fused boundary)."""
        geo = self.geo
        src = x_in
        for layer in range(len(self.weights)):
            dst = x_final if layer == geo.layers - 1 else self._pingpong[layer % 2]
            if reuse is not None and layer > 0:
                a = self._args(layer, src, dst, time, reuse.indices, reuse.history_in[layer - 1],
                               reuse.history_out[layer - 1], geo.current)
            else:
                a = self._args(layer, src, dst, time)
            self._keep.append(a)
            _lib.check(_lib.lib().wamffn_block_run(self.plan.handle, stream, ctypes.byref(a)))
            src = dst

    def _enqueue_request(self, req: Request, stream: int, plan: BlockPlan) -> None:
        self.enqueue_pass(req.x[0], req.out[0], req.time[0], stream, reuse=req, plan=plan)  # update 0, token reuse
        self.enqueue_pass(req.x[1], req.out[1], req.time[1], stream, plan=plan)             # update 3, full refresh

    def enqueue_request(self, req: Request, stream: int) -> None:
        self._keep.clear()
        self._enqueue_request(req, stream, self.plan)

    def set_down_splits(self, splits: int) -> None:
        """Split-K factor of every lane's down projection for launches enqueued
        from now on (0: the SM-filling heuristic, best for one lane)."""
        for plan in self.plans:
            plan.set_splits(0, splits)

    def set_streamk(self, enabled: bool) -> None:
        """Stream-K up projection (every SM pair takes an equal share of the
        feature tiles' K blocks) on every lane, for launches enqueued from now on."""
        for plan in self.plans:
            plan.set_streamk(enabled)

    def enqueue_requests(self, requests: list[Request], stream: int, lanes: int | None = None) -> None:
        """A batch of independent requests.  With one lane they run in order on
        `stream`; with k lanes (default: all of the stack's) request i runs on
        lane i mod k, the lanes' streams wait for `stream` first and `stream`
        waits for every lane at the end, so the batch is one fork / join
        (capturable into one CUDA graph)."""
        self._keep.clear()
        k = len(self.plans) if lanes is None else lanes
        if k < 1 or k > len(self.plans):
            raise ValueError(f"lanes={k} outside [1, {len(self.plans)}]")
        k = min(k, max(1, len(requests)))
        if k == 1:
            for req in requests:
                self._enqueue_request(req, stream, self.plan)
            return
        origin = torch.cuda.ExternalStream(stream, device=self.device)
        fork = torch.cuda.Event()
        fork.record(origin)
        lane_streams = self._streams[:k]
        for lane_stream in lane_streams:
            lane_stream.wait_event(fork)
        for i, req in enumerate(requests):
            j = i % k
            self._enqueue_request(req, lane_streams[j].cuda_stream, self.plans[j])
        for lane_stream in lane_streams:
            join = torch.cuda.Event()
            join.record(lane_stream)
            origin.wait_event(join)

    def status(self, clear: bool = True) -> int:
        """OR of every lane's device status word (synchronises the device)."""
        value = 0
        for plan in self.plans:
            value |= plan.status(clear)
        return value

    def launches_per_request(self) -> int:
        return 2 * (1 + 3 * self.geo.layers)

    def close(self):
        for plan in self.plans:
            plan.close()
