"""The phase-trace decoder (``waminfer_b200/trace.py``): synthetic records on
CPU; on the GPU, the launches of a one-layer stack pass."""

import pytest
import torch

from waminfer_b200.trace import BOUNDARY, WORDS, Trace, decode, group_launches


def _buffer(records):
    buf = torch.zeros((len(records) + 1) * WORDS, dtype=torch.int64)
    buf[0] = len(records)
    for i, (kind, x, y, times) in enumerate(records, start=1):
        row = [x | (y << 16) | (kind << 32)] + list(times) + [i % 148, 8]
        buf[i * WORDS:(i + 1) * WORDS] = torch.tensor(row[:WORDS])
    return buf


def test_decode_and_group_synthetic_records():
    t = [1000, 3000, 20000, 21000, 25000]  # start, ready, issued, epilogue, end (ns)
    recs = [(0, x, 0, [v + 10 * x for v in t]) for x in range(4)]          # launch 1: GELU GEMM, 4 CTAs
    recs += [(2, x, y, [v + 30000 for v in t]) for y in range(2) for x in range(2)]  # launch 2: partials
    recs += [(2, 0, 0, [v + 60000 for v in t])]                            # launch 3: repeats (0, 0)
    recs += [(BOUNDARY, b, 0, [90000, 91000, 93000, 93000, 95000]) for b in range(3)]
    records = decode(_buffer(recs))
    assert len(records) == 12 and records[0]["kind"] == 0 and records[-1]["kind"] == BOUNDARY
    launches = group_launches(records)
    assert [(l["kind"], l["ctas"]) for l in launches] == [
        ("gemm: bias + GELU", 4), ("gemm: split-K partials", 4), ("gemm: split-K partials", 1), ("layer boundary", 3)]
    assert launches[0]["mainloop_us"] == (17.0, 17.0, 17.0)
    assert launches[3]["reduce_us"] == (2.0, 2.0, 2.0)


@pytest.mark.gpu
def test_trace_of_one_stack_layer(cuda_device):
    from waminfer_b200.stack import FFNStack, Geometry, Request, make_weights

    geo = Geometry(layers=1)
    stack = FFNStack(make_weights(1, geo.d, geo.h, cuda_device, seed=9), geo, cuda_device)
    req = Request(geo, cuda_device, seed=10)
    s = torch.cuda.current_stream(cuda_device).cuda_stream
    stack.enqueue_pass(req.x[1], req.out[1], req.time[1], s)  # compiles nothing, warms the plan
    with Trace(cuda_device) as trace:
        stack.enqueue_pass(req.x[1], req.out[1], req.time[1], s)
    launches = trace.launches()
    assert [l["kind"] for l in launches] == ["gemm: bias + GELU", "gemm: split-K partials", "layer boundary"]
    assert launches[0]["ctas"] == geo.h // 128 and launches[2]["ctas"] == geo.seq
    assert all(l["end_us"] > l["start_us"] for l in launches)
    stack.close()
