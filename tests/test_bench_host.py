"""CPU: the benchmark's clock-record parsing (the contract's `clocks` key):
samples before the timed region are dropped, other GPUs' lines are ignored,
throttle reasons are reported by name, and a sampler that is off says so."""

import tempfile

import bench


def _clocks(lines, uuid, skip):
    c = bench.Clocks(uuid)
    c.file = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)
    c.file.write("\n".join(lines) + "\n")
    c.file.flush()
    c.proc = object()  # a sampler that ran
    c.skip = skip
    return c.summary()


def _line(uuid, mhz, power_cap="Not Active", hw="Not Active"):
    return f"0, GPU-{uuid}, {mhz}, 1965, 900.0, 0x4, {hw}, Not Active, Not Active, {power_cap}"


def test_summary_median_reasons_and_filtering():
    lines = [_line("aaaa", 1965), _line("aaaa", 1500, power_cap="Active"), _line("bbbb", 900),
             _line("aaaa", 1480, power_cap="Active"), _line("aaaa", 1520)]
    out = _clocks(lines, "aaaa", skip=1)  # the first line predates the timed region
    assert out["samples"] == 3
    assert out["sm_mhz"] == 1500.0 and out["sm_max_mhz"] == 1965.0
    assert out["reasons"] == ["sw_power_cap"]


def test_hardware_slowdown_is_reported():
    out = _clocks([_line("aaaa", 1100, hw="Active")], "aaaa", skip=0)
    assert out["reasons"] == ["hw_slowdown"]


def test_no_samples_and_disabled_sampler():
    assert _clocks([_line("bbbb", 1900)], "aaaa", skip=0)["reasons"] == ["no samples"]
    assert bench.Clocks("aaaa", enabled=False).summary()["reasons"] == ["sampled on rank 0 only"]
