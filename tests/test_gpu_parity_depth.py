"""GPU: parity of the configuration the benchmark times, at full depth.

The benchmark's request is 30 FFN layers twice: the token-reuse pass of Euler
update 0 (layer 0 over 392 rows, layers 1..29 over 32 selected + 240 future +
32 action = 304 rows, history [29, 120, 3072]) and the full-refresh pass of
update 3 (30 x 392 rows).  These tests run exactly that request through
``FFNStack`` and compare it with

* the fp32 oracle (``oracle/ffn.py``: the reference's bf16 rounding points,
  fp32 GEMMs without TF32, evaluated on the GPU so that 60 layers take
  milliseconds), and
* the reference's own FFN phase on the same GPU and the same inputs
  (``baseline/reference_phase.py``: the unmodified WAMInfer package's
  ``VideoAdapter.ffn_at_layer_for_compile`` over its cuBLASLt ``PreparedFFN``
  plans and its Triton modulated norms), itself measured against the oracle.

Tolerances (measured on B200; the numbers are printed by every test).

* Single layer (the history of the first gathered layer): every element
  within 2e-2, except elements whose bf16 ulp exceeds 2e-2 (|x| >= 4), which
  are within one ulp; mean relative error <= 5e-3.  Measured: 117 of 368,640
  elements one ulp (0.031) away, all at |x| >= 4; mean-rel 4.6e-4.
* 30 layers: the residual stream is rounded to bf16 after every layer, so two
  correct implementations whose fp32 sums differ in the last bits drift apart
  by whole ulps of the residual, a random walk over the layers (the history's
  mean-rel grows from 4.6e-4 at layer 1 to 4.2e-3 at layer 29).  North star's
  2e-2 / 5e-3 is not reachable there by any implementation with the
  reference's bf16 rounding points: the reference's own FFN phase (cuBLASLt +
  Triton, same inputs) is 0.19 max-abs / 7.4e-3 mean-rel away from the fp32
  oracle.  The bound at depth is therefore stated two ways: against the
  reference's own deviation on identical inputs (mean-rel within 10 % of it,
  max-abs within two bf16 ulps of the worst value above it) when the
  reference is installed, and as the absolute bound its measurement supports
  (mean-rel <= 1e-2, max-abs <= 0.25) always.
* 10 Euler updates: the latents are rounded to bf16 after every update on top
  of the stack's deviation: mean-rel <= 2e-2, max-abs <= 0.25, and the same
  comparison with the reference's own FFN phase driving the same schedule.
* Indices, gather positions and history rows that were not refreshed are
  bit-exact.
"""

from __future__ import annotations

import gc
import json
import os

import pytest
import torch

from oracle import euler as oeuler
from oracle import ffn as offn

pytestmark = pytest.mark.gpu

MAX_ABS = 2e-2          # north star, per element, single layer
MEAN_REL = 5e-3         # north star
DEPTH_MAX_ABS = 0.25    # 30 layers (the reference's own phase: 0.19)
DEPTH_MEAN_REL = 1e-2   # 30 layers (the reference's own phase: 7.4e-3)
EULER_MAX_ABS = 0.25
EULER_MEAN_REL = 2e-2
REF_MEAN_REL_RATIO = 1.10  # at most 10 % above the reference's own mean-rel
REF_SLACK_ULPS = 2.0       # max-abs at most two ulps (of the worst value) above the reference's
LAYERS = 30
ROW_COUNTS = (392, 304, 360, 272, 336, 240)  # the benchmark's and the reference's own row counts


def _stats(got: torch.Tensor, ref: torch.Tensor) -> dict:
    g, r = got.float(), ref.float().to(got.device)
    err = (g - r).abs()
    worst = int(err.argmax())
    return {
        "max_abs": float(err.max()),
        "mean_rel": float(err.mean() / r.abs().mean().clamp_min(1e-12)),
        "over_2e-2": int((err > MAX_ABS).sum()),
        "elements": err.numel(),
        "worst_ref_value": float(r.flatten()[worst]),
        "worst_ulp": float(offn.bf16_ulp(r.flatten()[worst:worst + 1])[0]),
    }


def _report(name: str, stats: dict) -> None:
    line = json.dumps({"parity": name, **{k: (round(v, 6) if isinstance(v, float) else v) for k, v in stats.items()}})
    print(line)
    path = os.environ.get("WAMFFN_PARITY_LOG")
    if path:
        with open(path, "a") as f:
            f.write(line + "\n")


def _oracle_pass(weights, x, time, indices=None, history=None, n=0):
    """fp32 oracle of one pass on the device; returns (x_out, [per-layer clean history])."""
    dev = x.device
    y = x.float()
    t = time.float()
    clean_layers = []
    for layer, w in enumerate(weights):
        reuse = indices is not None and layer > 0
        cache = history[layer - 1].float() if reuse else None
        y, _, clean, _ = offn.ffn_block(
            y, None, None, w.mod[0].float(), t, w.w_up, w.b_up, w.w_down, w.b_down,
            indices if reuse else None, cache, n if reuse else 0, 1e-6,
            ffn=lambda a, wu, bu, wd, bd: offn.prepared_ffn(a.to(dev), wu, bu, wd, bd))
        if reuse:
            clean_layers.append(clean)
    return y, clean_layers


@pytest.fixture(scope="module")
def weights(cuda_device):
    from waminfer_b200.stack import make_weights

    torch.backends.cuda.matmul.allow_tf32 = False
    w = make_weights(LAYERS, 3072, 14336, cuda_device, seed=41)
    yield w
    del w
    gc.collect()
    torch.cuda.empty_cache()


def _run_request(stack, req, stream):
    stack.enqueue_pass(req.x[0], req.out[0], req.time[0], stream, reuse=req)
    stack.enqueue_pass(req.x[1], req.out[1], req.time[1], stream)
    torch.cuda.synchronize()
    assert stack.plan.status() == 0


@pytest.fixture(scope="module")
def bench_request(cuda_device, weights):
    """The benchmark's request on the default 30-layer geometry, our stack and the oracle."""
    from waminfer_b200.stack import FFNStack, Geometry, Request

    geo = Geometry()
    assert (geo.layers, geo.seq, geo.reuse_rows) == (LAYERS, 392, 304)
    stack = FFNStack(weights, geo, cuda_device)
    req = Request(geo, cuda_device, seed=43)
    _run_request(stack, req, torch.cuda.current_stream(cuda_device).cuda_stream)
    stack.close()
    del stack
    ref0, clean = _oracle_pass(weights, req.x[0], req.time[0], req.indices, req.history_in, geo.current)
    ref1, _ = _oracle_pass(weights, req.x[1], req.time[1])
    yield geo, req, (ref0, torch.stack(clean)), ref1
    gc.collect()
    torch.cuda.empty_cache()


def _single_layer_ok(got, ref) -> dict:
    """North star's single-layer rule with the bf16 ulp made explicit: every
    element within 2e-2 or, where one ulp of the value exceeds 2e-2, within
    one ulp; mean-rel <= 5e-3."""
    s = _stats(got, ref)
    g, r = got.float(), ref.float().to(got.device)
    err = (g - r).abs()
    ulp = offn.bf16_ulp(r)
    over = err > MAX_ABS
    s["over_2e-2_below_ulp_4"] = int((over & (ulp <= MAX_ABS)).sum())  # must be 0
    s["over_one_ulp"] = int((over & (err > ulp)).sum())                 # must be 0
    return s


@pytest.fixture(scope="module")
def reference(cuda_device, weights):
    """The reference's own FFN phase over the same weights (None when
    baseline/_ref is not installed), prepared for every row count used here."""
    import sys
    from pathlib import Path

    sys.path.insert(0, str(Path(__file__).resolve().parents[1] / "baseline"))
    import reference_phase as rp

    if rp.missing(cuda=True):
        yield None
        return
    ref = rp.import_reference(cuda=True)
    phase = rp.ReferencePhase(ref, rp.make_blocks(weights, cuda_device), cuda_device, prepared_rows=ROW_COUNTS)
    yield phase
    phase.close()
    del phase
    gc.collect()
    torch.cuda.empty_cache()


def _check_depth(name, ours, oracle, theirs=None, mean_rel=DEPTH_MEAN_REL, max_abs=DEPTH_MAX_ABS):
    s = _stats(ours, oracle)
    _report(name, s)
    assert s["mean_rel"] <= mean_rel and s["max_abs"] <= max_abs, (name, s)
    if theirs is not None:
        r = _stats(theirs, oracle)
        _report(name + ".reference_phase_vs_oracle", r)
        _report(name + ".vs_reference_phase", _stats(ours, theirs))
        assert s["mean_rel"] <= REF_MEAN_REL_RATIO * r["mean_rel"], (name, s, r)
        assert s["max_abs"] <= r["max_abs"] + REF_SLACK_ULPS * max(s["worst_ulp"], r["worst_ulp"]), (name, s, r)


def test_bench_request_first_layer_and_indices(bench_request):
    """Layer 1's history (the first gathered layer) is within the single-layer
    rule; rows that were not refreshed are bit-exact in every layer."""
    geo, req, (ref0, ref_hist), _ = bench_request
    s = _single_layer_ok(req.history_out[0], ref_hist[0])
    _report("bench_request.history_layer1", s)
    assert s["over_2e-2_below_ulp_4"] == 0 and s["over_one_ulp"] == 0 and s["mean_rel"] <= MEAN_REL, s
    chosen = req.indices[: geo.count].cpu().tolist()
    kept = sorted(set(range(geo.current)) - set(chosen))
    assert torch.equal(req.history_out[:, kept], req.history_in[:, kept])
    # the refreshed rows are the FFN outputs (not the old history)
    assert not torch.equal(req.history_out[:, chosen], req.history_in[:, chosen])


def test_bench_request_at_depth(bench_request, reference):
    """Both passes of the benchmark's request against the fp32 oracle and
    against the reference's own FFN phase on the same inputs, with the
    per-layer growth of the history deviation printed."""
    geo, req, (ref0, ref_hist), ref1 = bench_request
    for layer in (1, 2, 4, 8, 16, 29):
        _report(f"bench_request.history_layer{layer}", _stats(req.history_out[layer - 1], ref_hist[layer - 1]))
    theirs0 = theirs1 = theirs_hist = None
    if reference is not None:
        theirs0, theirs_hist = reference.run_pass(req.x[0], req.time[0], req.indices, req.history_in, geo.current,
                                                  geo.count)
        theirs1, _ = reference.run_pass(req.x[1], req.time[1])
        torch.cuda.synchronize()
        # untouched history rows are the same bits in both implementations
        kept = sorted(set(range(geo.current)) - set(req.indices[: geo.count].cpu().tolist()))
        assert torch.equal(req.history_out[:, kept], theirs_hist[:, kept])
    _check_depth("bench_request.reuse_pass_out", req.out[0], ref0, theirs0)
    _check_depth("bench_request.full_pass_out", req.out[1], ref1, theirs1)
    _check_depth("bench_request.history_all", req.history_out, ref_hist, theirs_hist)


@pytest.mark.parametrize("count", [32, 64, 96])
def test_reference_row_buckets_at_depth(cuda_device, weights, reference, count):
    """The reference's own row counts (no action rows; seq = 360): layer 0 at
    360 rows, layers 1..29 at count + 240 = 272 / 304 / 336 rows, 30 layers."""
    from waminfer_b200.stack import FFNStack, Geometry, Request

    geo = Geometry(action=0, count=count)
    assert geo.seq == 360 and geo.reuse_rows == count + 240
    stack = FFNStack(weights, geo, cuda_device)
    req = Request(geo, cuda_device, seed=50 + count)
    stream = torch.cuda.current_stream(cuda_device).cuda_stream
    stack.enqueue_pass(req.x[0], req.out[0], req.time[0], stream, reuse=req)
    torch.cuda.synchronize()
    assert stack.plan.status() == 0
    stack.close()
    ref, clean = _oracle_pass(weights, req.x[0], req.time[0], req.indices, req.history_in, geo.current)
    theirs = theirs_hist = None
    if reference is not None:
        theirs, theirs_hist = reference.run_pass(req.x[0], req.time[0], req.indices, req.history_in, geo.current,
                                                 count)
    _check_depth(f"buckets_{count + 240}.out", req.out[0], ref, theirs)
    _check_depth(f"buckets_{count + 240}.history", req.history_out, torch.stack(clean), theirs_hist)
    kept = sorted(set(range(geo.current)) - set(req.indices[:count].cpu().tolist()))
    assert torch.equal(req.history_out[:, kept], req.history_in[:, kept])


def test_future_rows_pass_at_depth(cuda_device, weights, reference):
    """Euler updates 1..9 of the reference: only the 240 future rows, full refresh, 30 layers."""
    from waminfer_b200.stack import FFNStack, Geometry, Request

    geo = Geometry(current=0, future=240, action=0, count=0)
    stack = FFNStack(weights, geo, cuda_device)
    req = Request(geo, cuda_device, seed=60)
    stream = torch.cuda.current_stream(cuda_device).cuda_stream
    stack.enqueue_pass(req.x[1], req.out[1], req.time[1], stream)
    torch.cuda.synchronize()
    assert stack.plan.status() == 0
    stack.close()
    ref, _ = _oracle_pass(weights, req.x[1], req.time[1])
    theirs = reference.run_pass(req.x[1], req.time[1])[0] if reference is not None else None
    _check_depth("future_240.out", req.out[1], ref, theirs)


@pytest.mark.parametrize("amplitude_m,nfe", [(0.10, 2), (0.02, 4)])
def test_euler_actions_at_depth(cuda_device, weights, reference, amplitude_m, nfe):
    """The motion-adaptive schedule over the 30-layer stack: the 32 action rows
    after 10 Euler updates against the oracle's schedule on the fp32 oracle,
    and against the same schedule driven by the reference's own FFN phase."""
    from waminfer_b200.euler import run_euler, time_modulation
    from waminfer_b200.stack import FFNStack, Geometry, Request

    geo = Geometry()
    stack = FFNStack(weights, geo, cuda_device)
    req = Request(geo, cuda_device, seed=32)
    g = torch.Generator(device=cuda_device).manual_seed(33)
    actions = torch.randn(geo.action, geo.d, device=cuda_device, generator=g).to(torch.bfloat16)
    result = run_euler(stack, req, actions, amplitude_m, seed=5)
    torch.cuda.synchronize()
    assert stack.plan.status() == 0
    stack.close()
    assert result.nfe == nfe and result.fresh == oeuler.fresh_updates(nfe)
    n_video = geo.seq - geo.action
    times = {k: time_modulation(geo, k, cuda_device, 5) for k in result.fresh}
    args = (weights, req.x[0][:n_video], actions, times, req.indices, req.history_in, geo.current, amplitude_m)
    ref, fresh, ref_nfe = oeuler.run_euler(*args, device=cuda_device)
    assert (fresh, ref_nfe) == (result.fresh, result.nfe)
    theirs = None
    if reference is not None:
        def reference_pass(x, time, idx, hist, n):
            bf = torch.bfloat16
            out, _ = reference.run_pass(x.to(bf), time.to(bf), idx, hist, n, geo.count if idx is not None else 0)
            return out

        theirs, fresh_r, nfe_r = oeuler.run_euler(*args, device=cuda_device, pass_fn=reference_pass)
        assert (fresh_r, nfe_r) == (fresh, ref_nfe)
    _check_depth(f"euler_{nfe}f.actions", result.actions, ref, theirs, EULER_MEAN_REL, EULER_MAX_ABS)
