"""Benchmark of the B200 video-DiT FFN stack (WAMInfer's hot path).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Workload (metric "FFN-stack ms/request and TFLOP/s (2F, 32/120 reuse)"):
one step = R requests per GPU; one request = the FFN stack of one observation
under the 2F schedule with 32/120 token reuse -- 30 layers at update 0 (layer 0
over all 392 rows, layers 1..29 over 32 selected + 240 future + 32 action rows
with cache scatter) and 30 layers at update 3 over all 392 rows.  d = 3072,
hidden = 14336, tanh-GELU, seeded synthetic weights and activations.
Requests are independent: with N GPUs each rank runs its own R requests (weak
scaling, no data-path collective; one all-reduce of the elapsed time only).
On each GPU the R requests run over --lanes concurrent lanes (streams with
their own scratch over the shared weights; the headline throughput); the same
requests on one lane give the per-request latency (`latency_ms_per_request`).
"""

from __future__ import annotations

import argparse
import json
import os
import signal
import statistics
import subprocess
import sys
import tempfile
import time
from pathlib import Path

import torch

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

METRIC = "FFN-stack ms/request and TFLOP/s (2F, 32/120 reuse) at 1/2/4/8 B200; % bf16 roofline"
FALLBACK_PEAKS = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}
# dram__bytes_read.sum + dram__bytes_write.sum of one up-projection launch at
# M = 392 from the committed ncu capture (profiles/umma_gemm_ffn_m392.md):
# 90.57 MB read + 3.86 MB written.
UP_GEMM_DRAM_BYTES = 94_424_832


def parse():
    p = argparse.ArgumentParser()
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=10)
    p.add_argument("--warmup", type=int, default=3)
    p.add_argument("--impl", choices=("ours", "reference"), default="ours")
    p.add_argument("--requests", type=int, default=24, help="requests per GPU per step")
    p.add_argument("--lanes", type=int, default=6,
                   help="concurrent request lanes per GPU (streams with their own scratch, shared weights)")
    p.add_argument("--down-splits", type=int, default=1,
                   help="split-K of the down projection when lanes > 1 (one lane uses the SM-filling heuristic)")
    p.add_argument("--layers", type=int, default=30)
    p.add_argument("--cpu-seconds", type=float, default=10.0,
                   help="minimum host-core time of the CPU baseline sample (whole requests)")
    p.add_argument("--no-cpu-baseline", action="store_true")
    p.add_argument("--no-e2e", action="store_true")
    p.add_argument("--no-gpu-baselines", action="store_true")
    p.add_argument("--no-tp", action="store_true",
                   help="with --gpus N > 1, skip the tensor-parallel line reported beside the headline")
    p.add_argument("--tp-requests", type=int, default=4, help="requests per step of that tensor-parallel line")
    p.add_argument("--only", choices=("norm", "projections", "dominant", "attention"),
                   help="profiling aid: time one component on cuda:0 and print its JSON (no bench line): the "
                        "modulated norm against the reference's Triton kernel, the attention projections against "
                        "torch, or the up-projection GEMM alone")
    p.add_argument("--proj-layout", default=None, metavar="SxG",
                   help="with --only projections: run every projection plan at split-K S x G token groups instead "
                        "of the tuner's choice (a profiler's slowed timings would mislead the tuner)")
    p.add_argument("--tp", action="store_true",
                   help="tensor-parallel mode: every request's FFN hidden dimension split across the --gpus ranks "
                        "(one all-reduce per layer, strong scaling); not the default bench line")
    return p.parse_args()


def peaks():
    path = ROOT / "MEASURED_PEAKS.json"
    if path.exists():
        data = json.loads(path.read_text())
        return {k: float(data[k]) for k in FALLBACK_PEAKS}, "measured"
    return dict(FALLBACK_PEAKS), "fallback"


class Clocks:
    """Samples SM clocks and throttle reasons with nvidia-smi during the timed region."""

    FIELDS = ("index,uuid,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, uuid: str | None, enabled: bool = True):
        self.uuid = uuid
        self.enabled = enabled  # only the rank that prints the line samples (one nvidia-smi per box)
        self.proc = None
        self.file = None

    def __enter__(self):
        if not self.enabled:
            return self
        try:
            self.file = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)
            # Only this GPU: querying all eight at 100 ms stretched the sampling
            # period past a short timed region on 8-GPU boxes.
            targets = [[]]
            if self.uuid:
                targets.insert(0, ["-i", self.uuid if self.uuid.startswith("GPU-") else f"GPU-{self.uuid}"])
            for target in targets:  # this GPU by UUID; all GPUs if nvidia-smi rejects the id
                self.proc = subprocess.Popen(
                    ["nvidia-smi", *target, f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                     "-lms", "100"],
                    stdout=self.file, stderr=subprocess.DEVNULL, start_new_session=True)
                # nvidia-smi takes a moment to start on a multi-GPU box: begin
                # the timed region only once it samples (bounded wait), so that
                # short regions still get samples; earlier lines are dropped.
                deadline = time.time() + 10.0
                while time.time() < deadline and self.proc.poll() is None:
                    if Path(self.file.name).stat().st_size > 0:
                        break
                    time.sleep(0.02)
                if Path(self.file.name).stat().st_size > 0:
                    break
                if self.proc.poll() is None:  # no sample in time: stop it before the next attempt
                    os.killpg(self.proc.pid, signal.SIGTERM)
                    self.proc.wait(timeout=10)
            self.skip = len(Path(self.file.name).read_text().splitlines())
        except Exception:
            self.proc = None
        return self

    def __exit__(self, *exc):
        if self.proc is not None:
            try:
                os.killpg(self.proc.pid, signal.SIGTERM)
            except Exception:
                pass
            self.proc.wait(timeout=10)

    def summary(self):
        if not self.enabled:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["sampled on rank 0 only"]}
        if self.proc is None or self.file is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.file.flush()
        rows = []
        for line in Path(self.file.name).read_text().splitlines()[getattr(self, "skip", 0):]:
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 10:
                continue
            if self.uuid and self.uuid not in parts[1]:
                continue
            rows.append(parts)
        os.unlink(self.file.name)
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no samples"]}
        sm = [float(r[2]) for r in rows if r[2].replace(".", "").isdigit()]
        mx = [float(r[3]) for r in rows if r[3].replace(".", "").isdigit()]
        names = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")
        reasons = sorted({n for r in rows for n, v in zip(names, r[6:10]) if v.lower() == "active"})
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": reasons, "samples": len(rows)}


def dist_setup(n_gpus):
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import datetime

        import torch.distributed as dist

        backend = "nccl" if torch.cuda.is_available() else "gloo"
        if backend == "nccl":
            torch.cuda.set_device(local)
        dist.init_process_group(backend, timeout=datetime.timedelta(seconds=300))
    return world, rank, local


def barrier(world):
    if world > 1:
        import torch.distributed as dist

        dist.barrier()


def max_over_ranks(value: float, world: int, device) -> float:
    if world == 1:
        return value
    import torch.distributed as dist

    t = torch.tensor([value], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


# ------------------------------------------------------------------ CPU side
def cpu_model() -> str:
    try:
        for line in Path("/proc/cpuinfo").read_text().splitlines():
            if line.startswith("model name"):
                return line.split(":", 1)[1].strip()
    except OSError:
        pass
    import platform

    return platform.processor() or "unknown"


class CpuReference:
    """The reference's own FFN path on the host cores, whole requests: the
    unmodified WAMInfer package from baseline/_ref (``VideoAdapter.
    ffn_at_layer_for_compile`` with ``vb.ffn = None``, i.e. its gather,
    native bf16 ``Linear -> GELU(tanh) -> Linear``, history index_copy / cat
    and last-layer gate, WAMInfer/blocks.py:246-272, and the history stack of
    runtime.py:263), driven layer by layer as in baseline/reference_phase.py.
    The reference's modulated norm is a Triton kernel with no CPU path, so the
    oracle's torch restatement of it (oracle/ffn.py, rounding points of
    WAMInfer/_triton_inference.py:149-176) stands in for it on the CPU.
    A request is the benchmark's: the update-0 pass with 32/120 token reuse
    and the update-3 full pass, 30 layers each, seeded synthetic bf16 weights."""

    def __init__(self, geo, seed: int = 0):
        sys.path.insert(0, str(ROOT / "baseline"))
        import reference_phase as rp
        from oracle import ffn as offn

        reason = rp.missing(cuda=False)
        if reason is not None:
            raise FileNotFoundError(reason)
        self.geo = geo
        ref = rp.import_reference(cuda=False)
        blocks = rp.random_blocks(geo.layers, geo.d, geo.h, "cpu", seed=seed)

        def norm(x, update, mod, previous, time_mod, weight, bias, mode, eps):
            y, n = offn.modulated_norm(x[0], None if update is None else update[0], mod[0],
                                       None if previous is None else previous[0], time_mod[0], weight, bias, mode, eps)
            return y.to(torch.bfloat16)[None], n.to(torch.bfloat16)[None]

        self.phase = rp.ReferencePhase(ref, blocks, "cpu", prepared_rows=None, norm=norm)
        g = torch.Generator().manual_seed(10_000 + seed)
        s, d = geo.seq, geo.d
        self.x = [torch.randn(s, d, generator=g).to(torch.bfloat16) for _ in range(2)]
        self.time = [(torch.randn(s, 6, d, generator=g) * 0.1).to(torch.bfloat16) for _ in range(2)]
        chosen = torch.randperm(geo.current, generator=g)[: geo.count].sort().values
        self.indices = torch.cat((chosen, torch.arange(geo.current, s)))
        self.history = torch.randn(geo.layers - 1, geo.current, d, generator=g).to(torch.bfloat16)

    def request(self) -> None:
        geo = self.geo
        self.phase.run_pass(self.x[0], self.time[0], self.indices, self.history, geo.current, geo.count)
        self.phase.run_pass(self.x[1], self.time[1])

    def time_requests(self, min_seconds: float, min_requests: int = 1) -> tuple[int, float]:
        done, t0 = 0, time.perf_counter()
        while done < min_requests or time.perf_counter() - t0 < min_seconds:
            self.request()
            done += 1
        return done, time.perf_counter() - t0


def _cpu_sample(geo, requests: int, seconds: float, threads: int) -> dict:
    per_request = seconds / requests
    return {
        "value": geo.request_flops() / per_request / 1e12,
        "unit": "TFLOP/s",
        "cores": threads,
        "cpu_model": cpu_model(),
        "kind": "reference",
        "ms_per_request": per_request * 1e3,
        "sample": f"{requests} whole request(s) ({2 * geo.layers} FFN layer passes each: update 0 with "
                  f"{geo.count}/{geo.current} reuse, update 3 full) in {seconds:.1f} s through the reference's own "
                  f"CPU code path (baseline/_ref VideoAdapter.ffn_at_layer_for_compile, native bf16 FFN; the "
                  f"Triton norm restated in torch), torch bf16 on {threads} host threads",
    }


def cpu_baseline(geo, min_seconds: float = 10.0):
    """The reference's CPU FFN path timed on all host cores over whole requests
    (at least `min_seconds` of work after one untimed warm-up request)."""
    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    ref = CpuReference(geo)
    ref.request()
    requests, seconds = ref.time_requests(min_seconds)
    return _cpu_sample(geo, requests, seconds, threads)


def run_reference(args, world, rank):
    """The reference arm: the reference's own CPU implementation of the path
    (CpuReference) on all host threads; each step is one whole request."""
    from waminfer_b200.stack import Geometry

    if rank != 0:
        return
    geo = Geometry(layers=args.layers)
    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    try:
        ref = CpuReference(geo)
    except FileNotFoundError as exc:
        print(json.dumps({"impl": "reference", "unavailable": f"reference CPU path: {exc}"}), flush=True)
        return
    for _ in range(max(0, args.warmup)):
        ref.request()
    times = []
    for _ in range(args.steps):
        _, seconds = ref.time_requests(0.0, 1)
        times.append(seconds)
    total = sum(times)
    sample = _cpu_sample(geo, len(times), total, threads)
    value = sample["value"]
    ms = total / len(times) * 1e3
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": "TFLOP/s", "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms, "ms_per_request": ms,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic", "config": config_dict(geo, args, world),
        "cpu_baseline": sample,
        "e2e": {"value": value, "unit": "TFLOP/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def config_dict(geo, args, world):
    return {
        "workload": "c4-request: 2F schedule, 32/120 token reuse, 30-layer FFN stack",
        "layers": geo.layers, "d_model": geo.d, "d_hidden": geo.h,
        "rows_update0": [geo.seq] + [geo.reuse_rows] * (geo.layers - 1), "rows_update3": geo.seq,
        "requests_per_gpu_per_step": args.requests, "requests_per_step": args.requests * world,
        "parallelism": f"request-parallel x{world}",
        "lanes_per_gpu": args.lanes, "down_splits": args.down_splits if args.lanes > 1 else "heuristic",
        "l2": "no flush needed: each pass streams 30 x 176 MB of weights through the 126 MB L2",
    }


# ------------------------------------------------------------------ GPU side
def time_dominant_kernel(device, geo, pk):
    """CUDA-event timing of the up-projection GEMM (M = 392) launched alone:
    achieved TFLOP/s against the burst bf16 peak."""
    from waminfer_b200.ffn import Plan, pack_weight

    g = torch.Generator(device=device).manual_seed(77)
    m = geo.seq
    x = (torch.randn(m, geo.d, device=device, generator=g)).to(torch.bfloat16)
    w = pack_weight((torch.randn(geo.h, geo.d, device=device, generator=g) * 0.02).to(torch.bfloat16))
    b = torch.zeros(geo.h, device=device, dtype=torch.bfloat16)
    plan = Plan(x, w, b, exhaustive=False, gelu=True)
    # Rotate over weight copies (4 x 88 MB > L2) so every launch streams its
    # weights from HBM; launches are replayed from a CUDA graph so no host gap
    # sits between them.
    ws = [w] + [w.clone() for _ in range(3)]
    iters = 40
    stream = torch.cuda.Stream(device)
    with torch.cuda.stream(stream):
        for i in range(3):
            plan.run(x, ws[i % 4], b)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=stream):
            for i in range(iters):
                plan.run(x, ws[i % 4], b)
        graph.replay()
        torch.cuda.synchronize(device)
        samples = []
        for _ in range(3):
            start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            start.record(stream)
            graph.replay()
            end.record(stream)
            end.synchronize()
            samples.append(start.elapsed_time(end) / iters)
    ms = statistics.median(samples)
    graph.reset()
    flops = 2 * m * geo.d * geo.h
    achieved = flops / (ms * 1e-3) / 1e12
    plan.close()
    del ws
    return {
        "kernel": "umma_gemm_kernel (up projection + bias + GELU, M=392)",
        "bound": "tensor", "achieved": achieved, "peak": pk["bf16_tflops"], "unit": "TFLOP/s",
        "frac": achieved / pk["bf16_tflops"], "us_per_launch": ms * 1e3,
        "traffic": UP_GEMM_DRAM_BYTES,
        "algorithmic_bytes": 2 * (geo.h * geo.d + m * geo.d + m * geo.h),
    }


def _graph_ms_per_replay(fn, device, replays):
    stream = torch.cuda.Stream(device)
    with torch.cuda.stream(stream):
        for _ in range(2):
            fn()
        torch.cuda.synchronize(device)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=stream):
            fn()
        graph.replay()
        torch.cuda.synchronize(device)
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        start.record(stream)
        for _ in range(replays):
            graph.replay()
        end.record(stream)
        end.synchronize()
    ms = start.elapsed_time(end) / replays
    graph.reset()
    return ms


def _capture(fn, device):
    """fn captured into a CUDA graph (after two eager warm-up calls) on a side stream."""
    stream = torch.cuda.Stream(device)
    with torch.cuda.stream(stream):
        for _ in range(2):
            fn()
        torch.cuda.synchronize(device)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=stream):
            fn()
    torch.cuda.synchronize(device)
    return graph, stream


def _time_replays(graph, stream, replays):
    with torch.cuda.stream(stream):
        graph.replay()
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        start.record(stream)
        for _ in range(replays):
            graph.replay()
        end.record(stream)
        end.synchronize()
    return start.elapsed_time(end) / replays


def reference_ffn_phase_ms(device, geo, weights, replays, lanes=1, ours_latency=None, ours_lanes=None):
    """The reference's own FFN phase on this GPU, per layer as its blocks run
    it without attention: the FFN_RESIDUAL norm that folds the previous
    layer's gated FFN output (``pre_attn_at_layer_for_compile``,
    WAMInfer/blocks.py:189-203), the CROSS_RESIDUAL norm of the FFN input
    (blocks.py:241-243, zero cross output), then
    ``VideoAdapter.ffn_at_layer_for_compile`` (gather, PreparedFFN's cuBLASLt
    plans, history scatter / concat, last-layer gate; blocks.py:246-272), and
    the history stack of the reuse pass (runtime.py:263).  The WAMInfer
    package is the unmodified reference installed in baseline/_ref (imported
    through a stub parent package: its __init__ needs the absent openwam);
    the cuBLASLt extension is the one built from its source there.

    Returns the latency and, with lanes > 1, the throughput of `lanes`
    requests run concurrently on as many streams, each lane a VideoAdapter
    with its own PreparedFFN (plans and workspaces are per model in the
    reference, ffn.py:5-6) over the shared weights.  Latency is timed over a
    graph of requests run back to back; with `ours_latency` = (graph, stream,
    requests) this library's one-lane graph is timed in alternation with it,
    so both see the same clocks (sustained GEMM load runs into the 1 kW power
    cap, and a short burst would run faster than a long one); `ours_lanes`
    does the same for the lane throughput (the reference then runs as many
    requests per lane as this library's lanes graph)."""
    sys.path.insert(0, str(ROOT / "baseline"))
    import reference_phase as rp
    from waminfer_b200.stack import Request

    ref = rp.import_reference(cuda=True)
    blocks = rp.make_blocks(weights, device)

    def make_lane(seed):
        phase = rp.ReferencePhase(ref, blocks, device, prepared_rows=geo.request_rows())
        req = Request(geo, device, seed=seed)

        def request():
            phase.run_pass(req.x[0], req.time[0], req.indices, req.history_in, geo.current, geo.count)
            phase.run_pass(req.x[1], req.time[1])

        return phase, request

    lanes_ = [make_lane(4242 + i) for i in range(lanes)]
    back_to_back = ours_latency[2] if ours_latency is not None else 1

    def sequential():
        for _ in range(back_to_back):
            lanes_[0][1]()

    ref_graph, ref_stream = _capture(sequential, device)
    ref_ms, ours_ms = [], []
    for _ in range(3):
        if ours_latency is not None:
            ours_ms.append(_time_replays(ours_latency[0], ours_latency[1], 1) / back_to_back)
        ref_ms.append(_time_replays(ref_graph, ref_stream, max(1, replays // back_to_back)) / back_to_back)
    ref_graph.reset()
    out = {"latency_ms": statistics.median(ref_ms), "latency_requests_back_to_back": back_to_back}
    if ours_ms:
        out["ours_latency_ms"] = statistics.median(ours_ms)
    if lanes > 1:
        streams = [torch.cuda.Stream(device) for _ in range(lanes)]
        total = ours_lanes[2] if ours_lanes is not None else lanes
        per_lane = max(1, total // lanes)

        def concurrent():
            origin = torch.cuda.current_stream(device)
            for st in streams:
                st.wait_stream(origin)
            for st, (_, fn) in zip(streams, lanes_):
                with torch.cuda.stream(st):
                    for _ in range(per_lane):
                        fn()
            for st in streams:
                origin.wait_stream(st)

        lanes_graph, lanes_stream = _capture(concurrent, device)
        ref_ms, ours_ms = [], []
        for _ in range(3):
            if ours_lanes is not None:
                ours_ms.append(_time_replays(ours_lanes[0], ours_lanes[1], 1) / total)
            ref_ms.append(_time_replays(lanes_graph, lanes_stream, 1) / (per_lane * lanes))
        lanes_graph.reset()
        out["lanes_ms_per_request"] = statistics.median(ref_ms)
        if ours_ms:
            out["ours_lanes_ms"] = statistics.median(ours_ms)
    for phase, _ in lanes_:
        phase.close()
    return out


def reference_geometry_timings(device, weights, stream, requests=8):
    """One-lane request latency at the reference's own row semantics (the
    runtime's token-reuse buckets, runtime.py:157-201): 360 video rows (3
    latent frames of 120; the action rows run in the action branch, not in
    the video FFN), update 0 with 32 / 64 / 96 refreshed current rows (272 /
    304 / 336 FFN rows from layer 1), update 3 full.  Each bucket is timed in
    alternation with the reference's FFN phase on the same geometry
    (``reference_ffn_phase_ms``)."""
    from waminfer_b200.stack import FFNStack, Geometry, Request

    out = {}
    for count in (32, 64, 96):
        geo = Geometry(layers=len(weights), action=0, count=count)
        stack = FFNStack(weights, geo, device, lanes=1)
        reqs = [Request(geo, device, seed=77_000 + i) for i in range(requests)]
        handle = stream.cuda_stream
        with torch.cuda.stream(stream):
            stack.enqueue_requests(reqs, handle, lanes=1)
        torch.cuda.synchronize(device)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=stream):
            stack.enqueue_requests(reqs, handle, lanes=1)
        ref = reference_ffn_phase_ms(device, geo, weights, replays=requests, lanes=1,
                                     ours_latency=(graph, stream, requests))
        graph.reset()
        stack.close()
        del stack, reqs
        out[f"count_{count}"] = {
            "rows_update0": geo.reuse_rows, "rows_update3": geo.seq,
            "ours_latency_ms_per_request": ref.get("ours_latency_ms"),
            "reference_ffn_phase_ms_per_request": ref["latency_ms"],
            "speedup_vs_reference_ffn_phase": ref["latency_ms"] / ref["ours_latency_ms"]}
    return out


def norm_timings(device, geo, replays):
    """The modulated norm at S = 392 with per-token time rows,
    CROSS_RESIDUAL and FFN_RESIDUAL modes: this library's op against the
    reference's Triton kernel (baseline/_ref, imported through the stub parent
    package), 30 distinct inputs per replay so that each call reads its rows
    from HBM."""
    import types

    from waminfer_b200.norm import modulated_norm

    ref_root = ROOT / "baseline" / "_ref"
    if "WAMInfer" not in sys.modules:
        pkg = types.ModuleType("WAMInfer")
        pkg.__path__ = [str(ref_root / "WAMInfer")]
        sys.modules["WAMInfer"] = pkg
    from WAMInfer import _triton_inference as rt

    g = torch.Generator(device=device).manual_seed(5)
    s, d, n = geo.seq, geo.d, 30

    def rnd(*shape, std=1.0):
        return (torch.randn(*shape, device=device, generator=g) * std).to(torch.bfloat16)

    xs = [rnd(1, s, d) for _ in range(n)]
    ups = [rnd(1, s, d) for _ in range(n)]
    times = [rnd(1, s, 6, d, std=0.1) for _ in range(n)]
    mod, prev = rnd(1, 6, d, std=0.1), rnd(1, 6, d, std=0.1)
    out = {}
    for name, mode, previous in (("cross_residual", rt.CROSS_RESIDUAL, None), ("ffn_residual", rt.FFN_RESIDUAL, prev)):
        def ours():
            for x, u, t in zip(xs, ups, times):
                modulated_norm(x, u, mod, previous, t, None, None, mode, 1e-6)

        def reference():
            for x, u, t in zip(xs, ups, times):
                rt.modulated_norm(x, u, mod, previous, t, None, None, mode, 1e-6)

        with torch.no_grad():
            t_ours = _graph_ms_per_replay(ours, device, replays) / n * 1e3
            t_ref = _graph_ms_per_replay(reference, device, replays) / n * 1e3
        out[name] = {"ours_us": t_ours, "reference_triton_us": t_ref, "speedup": t_ref / t_ours}
    return out


ATTENTION_SHAPES = {  # (nq, nk, masked, tail): the DiT's attention calls at the default request geometry
    "joint_392x392": (392, 392, False, False),          # video + action self-attention (joint.py:55-87)
    "video_context_360x512": (360, 512, True, False),   # video cross-attention (blocks.py:233-239)
    "action_context_32x512": (32, 512, True, True),     # action cross-attention (blocks.py:135)
    "future_context_240x513": (240, 513, True, True),   # updates 1-9: future rows, 513-token context
}


def attention_timings(device, replays, heads=24):
    """This library's masked attention against the reference's Triton kernel
    (baseline/_ref) on the DiT's attention shapes, 20 calls per graph replay on
    seeded inputs (the text mask pads the last quarter of the context)."""
    sys.path.insert(0, str(ROOT / "baseline"))
    import reference_phase as rp
    from waminfer_b200.attention import masked_attention

    reference = None
    if not rp.missing(cuda=True):
        rp.import_reference(cuda=True)
        from WAMInfer import _triton_attention

        reference = _triton_attention.masked_attention
    g = torch.Generator(device=device).manual_seed(3)
    out = {}
    for name, (nq, nk, masked, tail) in ATTENTION_SHAPES.items():
        q, k, v = (torch.randn(1, n, heads * 128, device=device, generator=g).bfloat16() for n in (nq, nk, nk))
        mask = None
        if masked:
            mask = torch.ones(1, 1, 1, nk, dtype=torch.bool, device=device)
            mask[..., int(nk * 0.75):] = False
        calls = 20
        with torch.no_grad():
            ours = _graph_ms_per_replay(lambda: [masked_attention(q, k, v, mask, heads, tail) for _ in range(calls)],
                                        device, replays) / calls * 1e3
            entry = {"ours_us": ours}
            # The same call at each forced key split (CTAs per query tile).
            entry["key_split_us"] = {
                str(split): _graph_ms_per_replay(
                    lambda: [masked_attention(q, k, v, mask, heads, tail, split) for _ in range(calls)], device,
                    replays) / calls * 1e3 for split in (1, 2, 4)}
            if reference is not None:
                theirs = _graph_ms_per_replay(
                    lambda: [reference(q, k, v, mask, heads, tail=tail) for _ in range(calls)], device, replays) / calls
                entry.update(reference_triton_us=theirs * 1e3, speedup=theirs * 1e3 / ours)
        out[name] = entry
    # The joint loop's structured layouts (joint.py:55-87): first-frame-causal
    # self-attention over 360 video + 32 action rows (first frame 120 rows),
    # and the current-frame step against a cached 120-row first frame.
    from waminfer_b200.attention import current_frame_attention, joint_first_frame_attention

    def rnd(rows):
        return torch.randn(1, rows, heads * 128, device=device, generator=g).bfloat16()

    q, k, v = rnd(392), rnd(392), rnd(392)
    calls = 20
    with torch.no_grad():
        ours = _graph_ms_per_replay(lambda: [joint_first_frame_attention(q, k, v, 360, 120, heads)
                                             for _ in range(calls)], device, replays) / calls * 1e3
        entry = {"ours_us": ours}
        if reference is not None:
            ref_joint = _triton_attention.joint_first_frame_attention
            theirs = _graph_ms_per_replay(lambda: [ref_joint(q, k, v, 360, 120, heads) for _ in range(calls)],
                                          device, replays) / calls * 1e3
            entry.update(reference_triton_us=theirs, speedup=theirs / ours)
        out["joint_first_frame_392"] = entry
        seg = dict(qv=rnd(240), qa=rnd(32), ck=rnd(120), kv=rnd(240), ka=rnd(32), cv=rnd(120), vv=rnd(240),
                   va=rnd(32))
        ours = _graph_ms_per_replay(lambda: [current_frame_attention(**seg, heads=heads) for _ in range(calls)],
                                    device, replays) / calls * 1e3
        entry = {"ours_us": ours}
        if reference is not None:
            ref_current = _triton_attention.current_frame_attention
            theirs = _graph_ms_per_replay(lambda: [ref_current(**seg, heads=heads) for _ in range(calls)], device,
                                          replays) / calls * 1e3
            entry.update(reference_triton_us=theirs, speedup=theirs / ours)
        out["current_frame_120+240+32"] = entry
    return out


def projection_timings(device, geo, replays, layout=None):
    """Attention-side projections of one block at M = 392 rows (packed QKV
    3072 -> 9216, self-attention output, cross-attention query and output,
    3072 -> 3072): this library's plans against torch's F.linear (cuBLAS, what
    the reference calls, WAMInfer/blocks.py:204-240), 30 layers' worth of
    distinct weights so that every call streams its weights from HBM."""
    import torch.nn.functional as F

    from waminfer_b200.ffn import Plan, pack_weight

    g = torch.Generator(device=device).manual_seed(123)
    m, d, layers = geo.seq, geo.d, 30
    x = torch.randn(m, d, device=device, generator=g).to(torch.bfloat16)
    out = {}
    for name, n in (("qkv", 3 * d), ("self_out", d), ("cross_q", d), ("cross_out", d)):
        ws = [(torch.randn(n, d, device=device, generator=g) * 0.02).to(torch.bfloat16) for _ in range(layers)]
        b = (torch.randn(n, device=device, generator=g) * 0.01).to(torch.bfloat16)
        packed = [pack_weight(w) for w in ws]
        plan = Plan(x, packed[0], b, True, False)
        if layout is not None:
            plan.set_layout(*layout)

        def ours():
            for w in packed:
                plan.run(x, w, b)

        def torch_linear():
            for w in ws:
                F.linear(x, w, b)

        # NVTX range per projection: `ncu --nvtx --nvtx-include "ours_self_out/"` captures its launches.
        with torch.cuda.nvtx.range(f"ours_{name}"):
            t_ours = _graph_ms_per_replay(ours, device, replays) / layers * 1e3
        t_torch = _graph_ms_per_replay(torch_linear, device, replays) / layers * 1e3
        flops = 2 * m * n * d
        out[name] = {"ours_us": t_ours, "torch_us": t_torch, "speedup": t_torch / t_ours,
                     "ours_tflops": flops / (t_ours * 1e-6) / 1e12, **plan.layout()}
        plan.close()
        del ws, packed
    return out


def gpu_baselines(device, geo, weights, replays=5, lanes=1, ours_latency=None, ours_lanes=None):
    """Same-GPU baselines over one request's 60 layer passes (FFN GEMMs only,
    no norm / gather / scatter), CUDA-graph replayed:
    * torch native Linear -> GELU(tanh) -> Linear (what the reference runs on
      B200, WAMInfer/blocks.py:254-258);
    * the reference's own cuBLASLt prepared path (WAMInfer/ffn.py:96-107 over
      WAMInfer/_cublaslt_inference.cpp Plan, exhaustive tuning, col-major weight
      copies), built by baseline/build_reference_cublaslt.py."""
    import torch.nn.functional as F

    out = {}
    g = torch.Generator(device=device).manual_seed(99)
    rows = geo.request_rows()
    xs = {m: torch.randn(m, geo.d, device=device, generator=g).to(torch.bfloat16) for m in set(rows)}
    layers = len(weights)

    def native():
        for i, m in enumerate(rows):
            w = weights[i % layers]
            h = F.gelu(F.linear(xs[m], w.w_up, w.b_up), approximate="tanh")
            F.linear(h, w.w_down, w.b_down)

    out["torch_native_ms_per_request"] = _graph_ms_per_replay(native, device, replays)

    # The same GEMM-only work on this library's plans (up + bias + GELU, split-K
    # down + bias), for a like-for-like comparison of the GEMM engines.
    from waminfer_b200.ffn import Plan, pack_weight

    packed = [(pack_weight(w.w_up), pack_weight(w.w_down)) for w in weights]
    our_plans = {}
    for m in set(rows):
        hid = torch.empty(m, geo.h, device=device, dtype=torch.bfloat16)
        our_plans[m] = (Plan(xs[m], packed[0][0], weights[0].b_up, True, True),
                        Plan(hid, packed[0][1], weights[0].b_down, True, False))

    def ours_gemms():
        for i, m in enumerate(rows):
            w, (wu, wd) = weights[i % layers], packed[i % layers]
            up, down = our_plans[m]
            down.run(up.run(xs[m], wu, w.b_up), wd, w.b_down)

    out["ours_gemms_only_ms_per_request"] = _graph_ms_per_replay(ours_gemms, device, replays)
    try:
        out["projections_m392"] = projection_timings(device, geo, replays)
    except Exception as exc:  # reported, not fatal
        out["projections_error"] = f"{type(exc).__name__}: {exc}"
    try:
        out["modulated_norm_s392"] = norm_timings(device, geo, replays)
    except Exception as exc:  # reported, not fatal
        out["modulated_norm_error"] = f"{type(exc).__name__}: {exc}"
    for up, down in our_plans.values():
        up.close()
        down.close()
    del packed, our_plans
    ref_dir = ROOT / "baseline" / "_ref"
    if (ref_dir / "wam_infer_ffn_v1.so").exists():
        try:
            sys.path.insert(0, str(ref_dir))
            import wam_infer_ffn_v1 as ext  # noqa: F401

            col = [(w.w_up.T.contiguous().T, w.w_down.T.contiguous().T) for w in weights]
            plans = {}
            for m in set(rows):
                h = torch.randn(m, geo.h, device=device, generator=g).to(torch.bfloat16)
                plans[m] = (ext.Plan(xs[m], col[0][0], weights[0].b_up, True, True),
                            ext.Plan(h, col[0][1], weights[0].b_down, True, False))

            def cublaslt():
                for i, m in enumerate(rows):
                    w, (wu, wd) = weights[i % layers], col[i % layers]
                    up, down = plans[m]
                    down.run(up.run(xs[m], wu, w.b_up), wd, w.b_down)

            out["reference_cublaslt_ms_per_request"] = _graph_ms_per_replay(cublaslt, device, replays)
            out["reference_cublaslt_configs"] = {str(m): [list(p.selected_configuration()) for p in plans[m]]
                                                 for m in plans}
            del col, plans
        except Exception as exc:  # reported, not fatal: the product arm does not depend on it
            out["reference_cublaslt_error"] = f"{type(exc).__name__}: {exc}"
        try:
            phase = reference_ffn_phase_ms(device, geo, weights, replays, lanes, ours_latency, ours_lanes)
            out["reference_ffn_phase_ms_per_request"] = phase["latency_ms"]
            out["reference_ffn_phase_requests_back_to_back"] = phase["latency_requests_back_to_back"]
            if "ours_latency_ms" in phase:
                out["ours_paired_latency_ms_per_request"] = phase["ours_latency_ms"]
            if "lanes_ms_per_request" in phase:
                out["reference_ffn_phase_lanes_ms_per_request"] = phase["lanes_ms_per_request"]
                out["reference_ffn_phase_lanes"] = lanes
            if "ours_lanes_ms" in phase:
                out["ours_paired_lanes_ms_per_request"] = phase["ours_lanes_ms"]
        except Exception as exc:  # reported, not fatal
            out["reference_ffn_phase_error"] = f"{type(exc).__name__}: {exc}"
    else:
        out["reference_cublaslt_error"] = "baseline/_ref/wam_infer_ffn_v1.so not built"
    torch.cuda.synchronize(device)
    return out


def request_roofline_ms(geo, pk):
    """Sum over layer passes of max(FLOPs / bf16 peak, bytes / HBM bandwidth)."""
    total = 0.0
    for m in geo.request_rows():
        flops = 4 * m * geo.d * geo.h
        bytes_ = 2 * geo.d * geo.h * 2 + 2 * m * geo.d * 2 + 2 * m * geo.h * 2 + 2 * m * geo.d * 2
        total += max(flops / (pk["bf16_tflops_sustained"] * 1e12), bytes_ / (pk["hbm_gbs"] * 1e9))
    return total * 1e3


def run_ours(args, world, rank, local):
    from waminfer_b200 import _lib
    from waminfer_b200.stack import FFNStack, Geometry, Request, make_weights

    device = torch.device("cuda", local)
    torch.cuda.set_device(device)
    pk, pk_kind = peaks()
    geo = Geometry(layers=args.layers)
    weights = make_weights(geo.layers, geo.d, geo.h, device, seed=0)
    if args.lanes < 1:
        raise SystemExit("--lanes must be at least 1")
    stack = FFNStack(weights, geo, device, lanes=args.lanes)
    requests = [Request(geo, device, seed=rank * 100_000 + i) for i in range(args.requests)]
    stream = torch.cuda.Stream(device)
    handle = stream.cuda_stream
    # The dominant kernel alone, first: against the burst peak it needs the
    # clocks of a GPU that is not yet running into its power cap.
    roof = time_dominant_kernel(device, geo, pk)
    roof["peak_kind"] = f"{pk_kind} (burst bf16 GEMM)"

    def capture(lanes, splits, reqs=requests):
        # Eager warm-up (also checks the device status words), then capture the
        # R requests over `lanes` lanes into one graph.
        stack.set_down_splits(splits)
        with torch.cuda.stream(stream):
            stack.enqueue_requests(reqs, handle, lanes=lanes)
        torch.cuda.synchronize(device)
        status = stack.status()
        if status:
            raise RuntimeError(f"device status {status:#x} after warm-up")
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=stream):
            stack.enqueue_requests(reqs, handle, lanes=lanes)
        return g

    # Latency: one lane, requests back to back (each request's own duration).
    latency_graph = capture(1, 0)
    # Throughput (the headline): the same requests over the lanes.
    graph = capture(args.lanes, args.down_splits) if args.lanes > 1 else latency_graph
    with torch.cuda.stream(stream):
        for _ in range(args.warmup):
            graph.replay()
    torch.cuda.synchronize(device)

    uuid = None
    try:
        uuid = str(torch.cuda.get_device_properties(device).uuid)
    except Exception:
        pass
    barrier(world)
    torch.cuda.synchronize(device)
    with Clocks(uuid, enabled=rank == 0) as clocks, torch.cuda.stream(stream):
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        start.record(stream)
        for _ in range(args.steps):
            graph.replay()
        end.record(stream)
        end.synchronize()
    torch.cuda.synchronize(device)
    barrier(world)
    ms_step_local = start.elapsed_time(end) / args.steps
    ms_step = max_over_ranks(ms_step_local, world, device)
    flops_step = geo.request_flops() * args.requests * world
    value = flops_step / (ms_step * 1e-3) / 1e12
    ms_request = ms_step / args.requests
    clk = clocks.summary()

    # Per-request latency: the one-lane graph (heuristic split-K), same requests.
    latency_ms = ms_request
    if graph is not latency_graph:
        with torch.cuda.stream(stream):
            for _ in range(args.warmup):
                latency_graph.replay()
            s1, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            s1.record(stream)
            for _ in range(max(1, args.steps // 2)):
                latency_graph.replay()
            e1.record(stream)
            e1.synchronize()
        latency_ms = max_over_ranks(s1.elapsed_time(e1) / max(1, args.steps // 2), world, device) / args.requests

    # 4F schedule latency (the motion-adaptive schedule with small coarse motion): the
    # Transformer runs at updates 0, 3, 6 and 9, so a request is the reuse pass
    # of update 0 and three full passes, one request after another on one lane.
    stack.set_down_splits(0)
    four = requests[:min(8, len(requests))]

    def enqueue_4f():
        stack._keep.clear()
        for r in four:
            stack.enqueue_pass(r.x[0], r.out[0], r.time[0], handle, reuse=r)
            for _ in range(3):
                stack.enqueue_pass(r.x[1], r.out[1], r.time[1], handle)

    with torch.cuda.stream(stream):
        enqueue_4f()
    torch.cuda.synchronize(device)
    graph_4f = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph_4f, stream=stream):
        enqueue_4f()
    with torch.cuda.stream(stream):
        graph_4f.replay()
        s3, e3 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s3.record(stream)
        graph_4f.replay()
        e3.record(stream)
        e3.synchronize()
    latency_4f_ms = max_over_ranks(s3.elapsed_time(e3), world, device) / len(four)
    graph_4f.reset()

    # End to end: every step copies its R requests' inputs from pinned host
    # memory and its outputs back, around the same lanes graph.  Two sets of
    # request buffers alternate between steps so that the copies of one step
    # overlap the compute of its neighbours (a serving loop's double
    # buffering): inputs of step k go up on a copy stream while step k-1
    # computes, outputs of step k come down while step k+1 computes.  The
    # timed region runs from before the first input copy to after the last
    # output copy.
    e2e = None
    if not args.no_e2e:
        sets = [(requests, graph)]
        if args.steps > 1:
            other = [Request(geo, device, seed=rank * 100_000 + args.requests + i) for i in range(args.requests)]
            sets.append((other, capture(args.lanes, args.down_splits if args.lanes > 1 else 0, other)))
        host_in = [[r.x[0].cpu().pin_memory(), r.x[1].cpu().pin_memory(), r.indices.cpu().pin_memory()]
                   for r in requests]
        host_out = [[[torch.empty_like(r.out[0], device="cpu").pin_memory() for _ in range(2)] for r in reqs]
                    for reqs, _ in sets]
        h2d = sum(t.numel() * t.element_size() for hs in host_in for t in hs)
        d2h = sum(t.numel() * t.element_size() for hs in host_out[0] for t in hs)
        copy_in, copy_out = torch.cuda.Stream(device), torch.cuda.Stream(device)
        inputs_ready = [torch.cuda.Event() for _ in sets]
        computed = [torch.cuda.Event() for _ in sets]
        outputs_copied = [torch.cuda.Event() for _ in sets]

        def e2e_run(steps):
            begin = torch.cuda.Event()
            begin.record(stream)
            copy_in.wait_event(begin)
            for k in range(steps):
                j = k % len(sets)
                reqs, g = sets[j]
                with torch.cuda.stream(copy_in):
                    copy_in.wait_event(computed[j])       # the set's previous graph has read its inputs
                    for r, hi in zip(reqs, host_in):
                        r.x[0].copy_(hi[0], non_blocking=True)
                        r.x[1].copy_(hi[1], non_blocking=True)
                        r.indices.copy_(hi[2], non_blocking=True)
                    inputs_ready[j].record(copy_in)
                stream.wait_event(inputs_ready[j])
                stream.wait_event(outputs_copied[j])     # the set's previous outputs are on the host
                with torch.cuda.stream(stream):
                    g.replay()
                computed[j].record(stream)
                with torch.cuda.stream(copy_out):
                    copy_out.wait_event(computed[j])
                    for r, ho in zip(reqs, host_out[j]):
                        ho[0].copy_(r.out[0], non_blocking=True)
                        ho[1].copy_(r.out[1], non_blocking=True)
                    outputs_copied[j].record(copy_out)
            for ev in outputs_copied:
                stream.wait_event(ev)

        e2e_run(len(sets))
        torch.cuda.synchronize(device)
        barrier(world)
        s2, e2 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s2.record(stream)
        e2e_run(args.steps)
        e2.record(stream)
        e2.synchronize()
        barrier(world)
        ms_e2e = max_over_ranks(s2.elapsed_time(e2) / args.steps, world, device)
        e2e = {"value": flops_step / (ms_e2e * 1e-3) / 1e12, "unit": "TFLOP/s", "ms_per_step": ms_e2e,
               "ms_per_request": ms_e2e / args.requests, "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
               "copies": "double-buffered: a step's copies overlap its neighbours' compute" if len(sets) > 1
               else "serial"}
        for _, g in sets[1:]:
            g.reset()

    roof_ms = request_roofline_ms(geo, pk)

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        cpu = cpu_baseline(geo, args.cpu_seconds)
    baselines = None
    if rank == 0 and world == 1 and not args.no_gpu_baselines:
        # A one-lane graph of 8 back-to-back requests, timed in alternation
        # with the reference's FFN phase over as many requests.
        paired = requests[:8]
        stack.set_down_splits(0)
        paired_graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(paired_graph, stream=stream):
            stack.enqueue_requests(paired, handle, lanes=1)
        baselines = gpu_baselines(device, geo, weights, lanes=args.lanes,
                                  ours_latency=(paired_graph, stream, len(paired)),
                                  ours_lanes=(graph, stream, args.requests) if args.lanes > 1 else None)
        paired_graph.reset()
        if "reference_ffn_phase_ms_per_request" in baselines:
            baselines["reference_geometry"] = reference_geometry_timings(device, weights, stream)
        baselines["ours_ms_per_request"] = baselines.get("ours_paired_latency_ms_per_request", latency_ms)
        baselines["ours_lanes_ms_per_request"] = baselines.get("ours_paired_lanes_ms_per_request", ms_request)
        for key in ("torch_native", "reference_cublaslt"):
            if f"{key}_ms_per_request" in baselines:
                # GEMMs only on both sides (these baselines time no norm / gather / scatter).
                baselines[f"gemms_only_speedup_vs_{key}"] = (baselines[f"{key}_ms_per_request"] /
                                                             baselines["ours_gemms_only_ms_per_request"])
        if "reference_ffn_phase_ms_per_request" in baselines:
            # Whole FFN phase on both sides: norms, gather, GEMMs, scatter, gated residual.
            # Latency: one request at a time on both sides, timed in alternation.
            baselines["speedup_vs_reference_ffn_phase"] = (baselines["reference_ffn_phase_ms_per_request"] /
                                                           baselines["ours_ms_per_request"])
        if "reference_ffn_phase_lanes_ms_per_request" in baselines:
            # Throughput: the same number of concurrent lanes on both sides.
            baselines["lanes_speedup_vs_reference_ffn_phase"] = (
                baselines["reference_ffn_phase_lanes_ms_per_request"] / baselines["ours_lanes_ms_per_request"])

    launches = stack.launches_per_request() * args.requests * args.steps
    if rank == 0:
        line = {
            "metric": METRIC, "value": value, "unit": "TFLOP/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms_step, "ms_per_request": ms_request,
            "latency_ms_per_request": latency_ms, "latency_4f_ms_per_request": latency_4f_ms,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic (seeded N(0,1) activations, N(0,0.02) weights)",
            "config": config_dict(geo, args, world),
            "request_roofline_ms": roof_ms, "request_roofline_frac": roof_ms / ms_request,
            "roofline": roof, "cpu_baseline": cpu, "e2e": e2e, "clocks": clk, "gpu_baselines": baselines,
            "gpu_launches": launches, "launches_per_request": stack.launches_per_request(),
            "library_launches_total": _lib.launch_count(),
        }
    graph.reset()
    latency_graph.reset()
    stack.close()
    del stack, graph, latency_graph, requests, weights
    tp = None
    if world > 1 and not args.no_tp:
        # The secondary tensor-parallel mode on the same ranks, reported beside
        # the request-parallel headline with its own timing and clock record.
        torch.cuda.empty_cache()
        tp = run_tp(args, world, rank, local, requests=args.tp_requests, report=False)
    if rank == 0:
        line["tp"] = tp
        print(json.dumps(line), flush=True)


def run_tp(args, world, rank, local, requests: int | None = None, report: bool = True):
    """Tensor-parallel arm: the same requests on every rank, h split across
    the ranks, one all-reduce per layer.  Whole-job TFLOP/s counts each
    request's FLOPs once (strong scaling).  Returns rank 0's line (printed
    when `report`)."""
    import torch.distributed as dist

    from waminfer_b200.stack import Geometry, Request, make_weights
    from waminfer_b200.tp import TPStack, slice_weights

    device = torch.device("cuda", local)
    torch.cuda.set_device(device)
    geo = Geometry(layers=args.layers)
    weights = make_weights(geo.layers, geo.d, geo.h, device, seed=0)
    shards = slice_weights(weights, rank, world) if world > 1 else weights
    del weights
    if world > 1:
        stack = TPStack(shards, geo, device)
    else:
        from waminfer_b200.stack import FFNStack

        stack = FFNStack(shards, geo, device)
    n_requests = args.requests if requests is None else requests
    requests = [Request(geo, device, seed=i) for i in range(n_requests)]
    stream = torch.cuda.Stream(device)

    def step():
        for req in requests:
            if world > 1:
                stack.enqueue_pass(req.x[0], req.out[0], req.time[0], reuse=req)
                stack.enqueue_pass(req.x[1], req.out[1], req.time[1])
            else:
                stack.enqueue_request(req, stream.cuda_stream)

    with torch.cuda.stream(stream):
        step()
    torch.cuda.synchronize(device)
    status = stack.plan.status()
    if status:
        raise RuntimeError(f"device status {status:#x} after warm-up")
    # Collectives inside a captured graph when the backend allows it; eager otherwise.
    graph, mode = None, "eager"
    try:
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=stream):
            step()
        mode = "graph"
    except Exception as exc:  # noqa: BLE001 - reported in the line
        graph, mode = None, f"eager ({type(exc).__name__})"
        torch.cuda.synchronize(device)

    def run():
        if graph is not None:
            graph.replay()
        else:
            step()

    with torch.cuda.stream(stream):
        for _ in range(args.warmup):
            run()
    torch.cuda.synchronize(device)
    uuid = None
    try:
        uuid = str(torch.cuda.get_device_properties(device).uuid)
    except Exception:
        pass
    barrier(world)
    torch.cuda.synchronize(device)
    with Clocks(uuid, enabled=rank == 0) as clocks, torch.cuda.stream(stream):
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        start.record(stream)
        for _ in range(args.steps):
            run()
        end.record(stream)
        end.synchronize()
    torch.cuda.synchronize(device)
    barrier(world)
    ms_step = max_over_ranks(start.elapsed_time(end) / args.steps, world, device)
    flops_step = geo.request_flops() * n_requests
    line = None
    if rank == 0:
        line = {
            "metric": METRIC, "impl": "ours-tp", "value": flops_step / (ms_step * 1e-3) / 1e12, "unit": "TFLOP/s",
            "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms_step,
            "ms_per_request": ms_step / n_requests, "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None, "dtype": "bf16", "data": "synthetic (seeded N(0,1) activations, N(0,0.02) weights)",
            "config": dict(config_dict(geo, args, 1), parallelism=f"tp{world} (h split, one all-reduce per layer)",
                           requests_per_step=n_requests, requests_per_gpu_per_step=n_requests, capture=mode),
            "clocks": clocks.summary(),
            "gpu_launches": stack.launches_per_request() * n_requests * args.steps,
        }
        if report:
            print(json.dumps(line), flush=True)
    if graph is not None:
        graph.reset()
    del graph
    stack.close()
    if world > 1:
        dist.barrier()
    return line


def run_only(args):
    from waminfer_b200.stack import Geometry

    device = torch.device("cuda", 0)
    torch.cuda.set_device(device)
    geo = Geometry(layers=args.layers)
    if args.only == "norm":
        out = norm_timings(device, geo, 50)
    elif args.only == "attention":
        out = attention_timings(device, 20)
    elif args.only == "projections":
        layout = tuple(int(v) for v in args.proj_layout.lower().split("x")) if args.proj_layout else None
        out = projection_timings(device, geo, 20, layout)
    else:
        pk, kind = peaks()
        out = time_dominant_kernel(device, geo, pk)
    print(json.dumps({"only": args.only, **out}), flush=True)


def main():
    args = parse()
    if args.only:
        run_only(args)
        return
    world, rank, local = dist_setup(args.gpus)
    try:
        if args.impl == "reference":
            run_reference(args, world, rank)
        elif args.tp:
            run_tp(args, world, rank, local)
        else:
            run_ours(args, world, rank, local)
    finally:
        if world > 1:
            import torch.distributed as dist

            barrier(world)
            dist.destroy_process_group()


if __name__ == "__main__":
    main()
