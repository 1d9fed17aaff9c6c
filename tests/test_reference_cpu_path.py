"""CPU: the benchmark's reference arm runs the reference's own FFN path
(baseline/_ref, ``VideoAdapter.ffn_at_layer_for_compile`` with the native
FFN) and computes what the oracle computes: a small geometry, both passes of a
request (token reuse with history, then full refresh), against the oracle's
native-FFN restatement (``oracle/ffn.py::native_ffn``: bf16 after the first
Linear and after GELU, as torch's bf16 modules round)."""

import sys
from pathlib import Path

import pytest
import torch

from oracle import ffn as offn

ROOT = Path(__file__).resolve().parents[1]


def _oracle_pass(blocks, x, time, indices=None, history=None, n=0):
    y = x.float()
    clean_layers = []
    for layer, b in enumerate(blocks):
        reuse = indices is not None and layer > 0
        y, _, clean, _ = offn.ffn_block(
            y, None, None, b.modulation[0].float(), time.float(), b.ffn[0].weight, b.ffn[0].bias, b.ffn[2].weight,
            b.ffn[2].bias, indices if reuse else None, history[layer - 1].float() if reuse else None,
            n if reuse else 0, 1e-6, ffn=offn.native_ffn)
        if reuse:
            clean_layers.append(clean)
    return y, clean_layers


def test_cpu_reference_arm_follows_oracle():
    sys.path.insert(0, str(ROOT / "baseline"))
    import reference_phase as rp

    if rp.missing(cuda=False):
        pytest.skip(rp.missing(cuda=False))
    import bench
    from waminfer_b200.stack import Geometry

    geo = Geometry(layers=3, d=256, h=512, current=24, future=48, action=8, count=8)
    ref = bench.CpuReference(geo, seed=3)
    x0, hist = ref.phase.run_pass(ref.x[0], ref.time[0], ref.indices, ref.history, geo.current, geo.count)
    x1, _ = ref.phase.run_pass(ref.x[1], ref.time[1])
    o0, clean = _oracle_pass(ref.phase.blocks, ref.x[0], ref.time[0], ref.indices, ref.history, geo.current)
    o1, _ = _oracle_pass(ref.phase.blocks, ref.x[1], ref.time[1])
    for name, got, exp in (("reuse pass", x0, o0), ("full pass", x1, o1), ("history", hist, torch.stack(clean))):
        ok, msg = offn.check_close(got, exp)
        assert ok, f"{name}: {msg}"
    kept = sorted(set(range(geo.current)) - set(ref.indices[: geo.count].tolist()))
    assert torch.equal(hist[:, kept], ref.history[:, kept])
    sample = bench._cpu_sample(geo, 2, 1.0, 4)
    assert sample["kind"] == "reference" and sample["cores"] == 4 and sample["cpu_model"]
