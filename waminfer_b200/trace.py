"""Per-CTA phase timeline of the library's kernels (``wamffn_trace_enable``).

    with Trace(device) as trace:
        stack.enqueue_pass(...)          # eager launches (not inside a graph capture)
    for launch in trace.launches():
        print(launch["kind"], launch["ctas"], launch["mainloop_us"], launch["epilogue_us"])

Every GEMM CTA records {start, operands ready, MMAs issued, accumulator ready,
epilogue done} and every layer-boundary CTA {start, wait done, reduction done,
end} in globaltimer nanoseconds.  Records are appended in CTA start order;
a launch is the run of records of one kind in which no (x, y) CTA index
repeats.  This is the library's own tracing facility (the reference relies on
external Nsight traces); it perturbs timings by one global atomic per CTA.
"""

from __future__ import annotations

import statistics

import torch

from waminfer_b200 import _lib

WORDS = 8
KINDS = {0: "gemm: bias + GELU", 1: "gemm: bias", 2: "gemm: split-K partials", 7: "layer boundary",
         8: "masked attention"}
BOUNDARY = 7
ATTENTION = 8


def decode(buffer: torch.Tensor) -> list[dict]:
    """Records of a trace buffer ([records * 8] int64, record 0 = counter)."""
    words = buffer.detach().cpu().view(-1, WORDS).tolist()
    count = min(int(words[0][0]), len(words) - 1)
    out = []
    for w in words[1:1 + count]:
        tag = w[0]
        kind = (tag >> 32) & 0xFFFF
        rec = {"kind": kind, "x": tag & 0xFFFF, "y": (tag >> 16) & 0xFFFF, "sm": w[6], "start": w[1], "end": w[5]}
        if kind == BOUNDARY:
            rec.update(waited=w[2], reduced=w[3])
        elif kind == ATTENTION:
            # {first S ready, last S ready or first cluster barrier, last P.V done,
            #  sm | key blocks << 32, second cluster barrier}; rank in tag bits 48-51
            rec.update(sm=w[6] & 0xFFFFFFFF, key_blocks=w[6] >> 32, rank=(tag >> 48) & 0xF, first_s=w[2],
                       last_s_or_combine=w[3], last_pv=w[4], exchanged=w[7])
        else:
            rec.update(ready=w[2], issued=w[3], epilogue=w[4], k_blocks=w[7])
        out.append(rec)
    return out


def group_launches(records: list[dict]) -> list[dict]:
    """Splits records into launches and summarises each (times in us,
    relative to the first record's start; min / median / max over CTAs)."""
    launches, current, seen = [], [], set()
    for r in records:
        key = (r["x"], r["y"])
        if current and (r["kind"] != current[0]["kind"] or key in seen):
            launches.append(current)
            current, seen = [], set()
        current.append(r)
        seen.add(key)
    if current:
        launches.append(current)
    if not launches:
        return []
    t0 = min(r["start"] for r in records)
    out = []
    for recs in launches:
        kind = recs[0]["kind"]

        def span(a, b):
            v = [(r[b] - r[a]) / 1e3 for r in recs if r.get(a) and r.get(b)]
            return (min(v), statistics.median(v), max(v)) if v else None

        summary = {"kind": KINDS.get(kind, str(kind)), "ctas": len(recs),
                   "start_us": (min(r["start"] for r in recs) - t0) / 1e3,
                   "end_us": (max(r["end"] for r in recs) - t0) / 1e3}
        if kind == BOUNDARY:
            summary.update(wait_us=span("start", "waited"), reduce_us=span("waited", "reduced"),
                           finish_us=span("reduced", "end"))
        elif kind == ATTENTION:
            summary.update(setup_us=span("start", "first_s"), mainloop_us=span("first_s", "last_pv"),
                           epilogue_us=span("last_pv", "end"))
        else:
            summary.update(setup_us=span("start", "ready"), mainloop_us=span("ready", "issued"),
                           epilogue_us=span("epilogue", "end"))
        out.append(summary)
    return out


class Trace:
    """Context manager: enables tracing on `device` into a fresh buffer of
    `records` records and switches it off on exit (synchronising the device)."""

    def __init__(self, device, records: int = 16384):
        self.device = torch.device(device)
        self.buffer = torch.zeros(records * WORDS, dtype=torch.int64, device=self.device)
        self.records_capacity = records

    def __enter__(self) -> "Trace":
        torch.cuda.synchronize(self.device)
        _lib.check(_lib.lib().wamffn_trace_enable(self.device.index or 0, self.buffer.data_ptr(),
                                                  self.records_capacity))
        return self

    def __exit__(self, *exc) -> None:
        torch.cuda.synchronize(self.device)
        _lib.check(_lib.lib().wamffn_trace_enable(self.device.index or 0, None, 0))

    def records(self) -> list[dict]:
        return decode(self.buffer)

    def launches(self) -> list[dict]:
        return group_launches(self.records())
