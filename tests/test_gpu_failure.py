"""Failure detection without a GPU fault: a pipeline wait that can never
complete gives up after its limit, reports WAMFFN_DEV_TIMEOUT through the
device status word, releases the other waiter through the abort flag, and
leaves the context usable (``wamffn_selftest_wait_timeout``)."""

import time

import pytest
import torch

from waminfer_b200 import _lib

WAMFFN_DEV_TIMEOUT = 1
ABORT_SEEN = 0x100


def test_selftest_rejects_bad_arguments_without_a_gpu():
    lib = _lib.lib()
    assert lib.wamffn_selftest_wait_timeout(None, None, 10_000) == _lib.WAMFFN_ERR_INVALID
    assert lib.wamffn_selftest_wait_timeout(None, 256, 10) == _lib.WAMFFN_ERR_INVALID           # limit too short
    assert lib.wamffn_selftest_wait_timeout(None, 256, 10**10) == _lib.WAMFFN_ERR_INVALID       # limit too long
    assert lib.wamffn_selftest_wait_timeout(None, 258, 10_000) == _lib.WAMFFN_ERR_INVALID       # unaligned


@pytest.mark.gpu
def test_wait_timeout_reports_and_context_survives(cuda_device):
    from oracle import ffn as offn
    from waminfer_b200.ffn import Plan

    lib = _lib.lib()
    status = torch.zeros(1, dtype=torch.int32, device=cuda_device)
    stream = torch.cuda.current_stream(cuda_device).cuda_stream
    t0 = time.perf_counter()
    _lib.check(lib.wamffn_selftest_wait_timeout(stream, status.data_ptr(), 2_000_000))  # ~1 ms of SM cycles
    torch.cuda.synchronize(cuda_device)
    elapsed = time.perf_counter() - t0
    assert int(status.item()) == WAMFFN_DEV_TIMEOUT | ABORT_SEEN
    assert elapsed < 5.0
    # The context still runs work correctly afterwards.
    g = torch.Generator(device=cuda_device).manual_seed(5)
    x = torch.randn(64, 1024, device=cuda_device, generator=g).to(torch.bfloat16)
    w = (torch.randn(256, 1024, device=cuda_device, generator=g) * 0.02).to(torch.bfloat16)
    b = torch.zeros(256, device=cuda_device, dtype=torch.bfloat16)
    plan = Plan(x, w, b, exhaustive=False, gelu=False)
    out = plan.run(x, w, b)
    ok, msg = offn.check_close(out, offn.bf16(x.float() @ w.float().T))
    assert ok, msg
    assert plan.status() == 0
    plan.close()
