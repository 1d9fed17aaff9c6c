"""Tensor-parallel FFN stack (hidden dimension split across ranks).

* CPU: the shard layout, and the reduction math of the split on two gloo
  ranks against the oracle's single-device FFN;
* GPU (two or more devices): ``TPStack`` on two NCCL ranks against the
  single-GPU stack -- outputs within the multi-layer tolerance, every rank
  bit-identical, history rows that no layer recomputes untouched.
"""

from __future__ import annotations

import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

from oracle import ffn as offn
from waminfer_b200.stack import LayerWeights
from waminfer_b200.tp import shard_bounds, slice_layer


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _layer(d: int, h: int, seed: int, device="cpu") -> LayerWeights:
    g = torch.Generator(device=device).manual_seed(seed)

    def rnd(*shape, std):
        return (torch.randn(*shape, generator=g, device=device) * std).to(torch.bfloat16)

    return LayerWeights(rnd(h, d, std=0.02), rnd(h, std=0.01), rnd(d, h, std=0.02), rnd(d, std=0.01),
                        rnd(1, 6, d, std=0.1))


def test_shards_tile_the_hidden_dimension():
    w = _layer(256, 2048, seed=1)
    for world in (1, 2, 4, 8):
        bounds = [shard_bounds(2048, r, world) for r in range(world)]
        assert bounds[0][0] == 0 and bounds[-1][1] == 2048
        assert all(a[1] == b[0] for a, b in zip(bounds, bounds[1:]))
        shards = [slice_layer(w, r, world) for r in range(world)]
        assert torch.equal(torch.cat([s.w_up for s in shards]), w.w_up)
        assert torch.equal(torch.cat([s.b_up for s in shards]), w.b_up)
        assert torch.equal(torch.cat([s.w_down for s in shards], dim=1), w.w_down)
        assert all(s.b_down is w.b_down and s.mod is w.mod for s in shards)
    with pytest.raises(ValueError):
        shard_bounds(2048, 0, 3)


def _gloo_rank(rank: int, world: int, port: int, out_dir: str) -> None:
    import torch.distributed as dist

    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world)
    try:
        d, h, m = 256, 1024, 48
        w = _layer(d, h, seed=11)
        x = torch.randn(m, d, generator=torch.Generator().manual_seed(12)).to(torch.bfloat16)
        s = slice_layer(w, rank, world)
        # This rank's share: bf16 hidden shard, fp32 partial of the down GEMM (no bias).
        hid = offn.bf16(offn.gelu_tanh(x.float() @ s.w_up.float().T + s.b_up.float()))
        y = hid @ s.w_down.float().T
        dist.all_reduce(y)
        out = offn.bf16(y + w.b_down.float())
        torch.save(out, os.path.join(out_dir, f"rank{rank}.pt"))
    finally:
        dist.destroy_process_group()


def test_tp_reduction_math_on_gloo_ranks(tmp_path):
    world = 2
    mp.start_processes(_gloo_rank, args=(world, _free_port(), str(tmp_path)), nprocs=world, start_method="spawn")
    outs = [torch.load(tmp_path / f"rank{r}.pt") for r in range(world)]
    assert torch.equal(outs[0], outs[1])  # the reduced sum is replicated
    d, h, m = 256, 1024, 48
    w = _layer(d, h, seed=11)
    x = torch.randn(m, d, generator=torch.Generator().manual_seed(12)).to(torch.bfloat16)
    ref = offn.prepared_ffn(x, w.w_up, w.b_up, w.w_down, w.b_down)
    ok, msg = offn.check_close(outs[0], ref)
    assert ok, msg


def _nccl_rank(rank: int, world: int, port: int, out_dir: str) -> None:
    import torch.distributed as dist

    from waminfer_b200.stack import Geometry, Request, make_weights
    from waminfer_b200.tp import TPStack, slice_weights

    dev = torch.device("cuda", rank)
    torch.cuda.set_device(dev)
    dist.init_process_group("nccl", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            device_id=dev)
    try:
        geo = Geometry(layers=3)
        weights = make_weights(geo.layers, geo.d, geo.h, dev, seed=21)
        stack = TPStack(slice_weights(weights, rank, world), geo, dev)
        req = Request(geo, dev, seed=22)
        stack.enqueue_pass(req.x[0], req.out[0], req.time[0], reuse=req)
        stack.enqueue_pass(req.x[1], req.out[1], req.time[1])
        torch.cuda.synchronize()
        assert stack.plan.status() == 0
        torch.save({"out0": req.out[0].cpu(), "out1": req.out[1].cpu(), "hist": req.history_out.cpu()},
                   os.path.join(out_dir, f"rank{rank}.pt"))
        stack.close()
    finally:
        dist.destroy_process_group()


@pytest.mark.gpu
def test_tp_stack_on_two_gpus_matches_one_gpu(cuda_device, tmp_path):
    if torch.cuda.device_count() < 2:
        pytest.skip("two or more GPUs required")
    from waminfer_b200.stack import FFNStack, Geometry, Request, make_weights

    world = 2
    mp.start_processes(_nccl_rank, args=(world, _free_port(), str(tmp_path)), nprocs=world, start_method="spawn")
    outs = [torch.load(tmp_path / f"rank{r}.pt") for r in range(world)]
    for key in ("out0", "out1", "hist"):
        assert torch.equal(outs[0][key], outs[1][key]), key  # replicated after every reduction

    geo = Geometry(layers=3)
    weights = make_weights(geo.layers, geo.d, geo.h, cuda_device, seed=21)
    stack = FFNStack(weights, geo, cuda_device)
    req = Request(geo, cuda_device, seed=22)
    s = torch.cuda.current_stream(cuda_device).cuda_stream
    stack.enqueue_pass(req.x[0], req.out[0], req.time[0], s, reuse=req)
    stack.enqueue_pass(req.x[1], req.out[1], req.time[1], s)
    torch.cuda.synchronize()
    # Different summation order (split-K within each rank, then across ranks):
    # the multi-layer tolerance of the stack tests.
    for key, ref in (("out0", req.out[0]), ("out1", req.out[1]), ("hist", req.history_out)):
        ok, msg = offn.check_close(outs[0][key], ref, max_abs=6e-2)
        assert ok, f"{key}: {msg}"
    kept = sorted(set(range(geo.current)) - set(req.indices[: geo.count].tolist()))
    assert torch.equal(outs[0]["hist"][:, kept], req.history_in[:, kept].cpu())
    stack.close()


@pytest.mark.gpu
def test_tp_entry_point_identity_and_failing_reduction(cuda_device):
    """wamffn_stack_run_tp on one GPU: with an identity reduction hook the
    pass equals wamffn_stack_run bit for bit (the rank's split sum is the
    boundary's own split-order sum); a hook that fails at layer 1 stops the
    enqueue with the hook's status and a message, and the plan keeps working."""
    import ctypes

    from waminfer_b200 import _lib
    from waminfer_b200.stack import FFNStack, Geometry, Request, make_weights

    geo = Geometry(layers=3)
    stack = FFNStack(make_weights(geo.layers, geo.d, geo.h, cuda_device, seed=23), geo, cuda_device)
    req = Request(geo, cuda_device, seed=24)
    s = torch.cuda.current_stream(cuda_device).cuda_stream
    reduce = torch.empty(geo.seq, geo.d, dtype=torch.float32, device=cuda_device)
    calls = []

    def hook(fail_at):
        def fn(user, buffer, count, stream):
            calls.append(count)
            return 5 if len(calls) - 1 == fail_at else 0
        return _lib.ALLREDUCE_FN(fn)

    expected = torch.empty_like(req.out[0])
    stack.enqueue_pass(req.x[0], expected, req.time[0], s, reuse=req)
    identity = hook(-1)
    args = stack._stack_args(req.x[0], req.out[0], req.time[0], req)
    assert _lib.lib().wamffn_stack_run_tp(stack.plan.handle, s, ctypes.byref(args), reduce.data_ptr(), identity,
                                          None) == 0
    torch.cuda.synchronize()
    assert len(calls) == geo.layers and calls[0] == geo.seq * geo.d and calls[1] == req.indices.numel() * geo.d
    assert torch.equal(req.out[0], expected)

    calls.clear()
    failing = hook(1)
    args = stack._stack_args(req.x[0], req.out[0], req.time[0], req)
    status = _lib.lib().wamffn_stack_run_tp(stack.plan.handle, s, ctypes.byref(args), reduce.data_ptr(), failing,
                                            None)
    assert status == 5 and len(calls) == 2
    assert "allreduce callback failed at layer 1" in _lib.lib().wamffn_last_error().decode()
    torch.cuda.synchronize()
    stack.enqueue_pass(req.x[1], req.out[1], req.time[1], s)
    torch.cuda.synchronize()
    assert stack.status() == 0
    stack.close()
