"""Allocation-free split-K linear (``wamffn_linear_run_static``) against the
plan-based entry point (``wamffn_linear_plan_create`` + ``wamffn_linear_run``).

Both go through the C ABI.  The file name sorts last so that the GPU test also
runs after every other test of the suite has used the device; it passes alone
in a fresh process as well (``pytest tests/test_zz_no_alloc.py``).
"""

from __future__ import annotations

import ctypes

import pytest
import torch

from oracle import ffn as offn
from waminfer_b200 import _lib

SCRATCH_BYTES = 16 << 20   # WAMFFN_STATIC_SCRATCH_BYTES
HEADER = 256               # status word in front of the partials


def _run_static(lib, device, stream, rows, n_out, k_in, splits, flags, x, w, b, out, status=None):
    return lib.wamffn_linear_run_static(device, stream, rows, n_out, k_in, splits, flags, x, w, b, out, status)


def test_static_rejects_what_does_not_fit_before_launching():
    """Validation happens on the host before any device call, so this runs without a GPU."""
    lib = _lib.lib()
    fake = 256  # non-null, 16-byte aligned: never dereferenced because the call is rejected first
    # 8 splits x 512 rows x 3072 outputs x 4 B = 48 MiB of partials > 16 MiB.
    assert 8 * 512 * 3072 * 4 + HEADER > SCRATCH_BYTES
    rc = _run_static(lib, 0, None, 512, 3072, 14336, 8, 0, fake, fake, fake, fake)
    assert rc == 1  # WAMFFN_ERR_INVALID
    assert b"static scratch" in lib.wamffn_last_error()
    # GELU is not offered (the split-K reduction applies the bias only).
    assert _run_static(lib, 0, None, 128, 3072, 14336, 4, _lib.LINEAR_GELU, fake, fake, fake, fake) == 1
    # Split counts outside [2, 16].
    assert _run_static(lib, 0, None, 128, 3072, 14336, 1, 0, fake, fake, fake, fake) == 1
    assert _run_static(lib, 0, None, 128, 3072, 14336, 17, 0, fake, fake, fake, fake) == 1
    # One row past the limit: 4 x 342 x 3072 x 4 B + 256 > 16 MiB (341 rows fit, the GPU test runs them).
    assert HEADER + 4 * 342 * 3072 * 4 > SCRATCH_BYTES >= HEADER + 4 * 341 * 3072 * 4
    assert _run_static(lib, 0, None, 342, 3072, 14336, 4, 0, fake, fake, fake, fake) == 1
    assert b"static scratch" in lib.wamffn_last_error()


@pytest.mark.gpu
@pytest.mark.parametrize("rows,packed,splits", [(1, True, None), (77, False, None), (128, True, None),
                                                (392, True, None), (392, False, None), (341, True, 4)])
def test_static_matches_plan_on_two_calls_in_a_row(cuda_device, rows, packed, splits):
    """Against the plan path and the fp32 oracle (x . W^T + b in fp32, rounded
    to bf16), two calls in a row with different inputs.  Row counts that are
    not a multiple of 16 leave padded token columns; 341 rows at 4 splits
    fill the scratch to within 17 KB of its size."""
    from waminfer_b200.ffn import pack_weight

    lib = _lib.lib()
    n_out, k_in = 3072, 14336  # the down projection of the FFN
    g = torch.Generator(device=cuda_device).manual_seed(rows)
    weight = (torch.randn(n_out, k_in, device=cuda_device, generator=g) * 0.02).bfloat16()
    bias = (torch.randn(n_out, device=cuda_device, generator=g) * 0.01).bfloat16()
    w = pack_weight(weight) if packed else weight
    flags = _lib.WEIGHTS_PACKED if packed else 0

    plan = ctypes.c_void_p()
    _lib.check(lib.wamffn_linear_plan_create(0, rows, n_out, k_in, flags, 0, ctypes.byref(plan)))
    try:
        values = (ctypes.c_uint32 * 7)()
        _lib.check(lib.wamffn_linear_configuration(plan, values, 7))
        # The plan's own split count when it fits the static scratch, else the largest that does.
        if splits is None:
            splits = max(2, int(values[4]))
            while splits > 2 and HEADER + splits * rows * n_out * 4 > SCRATCH_BYTES:
                splits -= 1
        assert splits >= 2 and HEADER + splits * rows * n_out * 4 <= SCRATCH_BYTES
        stream = torch.cuda.current_stream(cuda_device).cuda_stream
        status = torch.zeros(1, dtype=torch.int32, device=cuda_device)
        for call in range(2):
            # Different inputs on each call: nothing may leak from the previous one.
            x = torch.randn(rows, k_in, device=cuda_device, generator=g).bfloat16()
            ref = torch.empty(rows, n_out, device=cuda_device, dtype=torch.bfloat16)
            _lib.check(lib.wamffn_linear_run(plan, stream, x.data_ptr(), w.data_ptr(), bias.data_ptr(),
                                             ref.data_ptr()))
            out = torch.full((rows, n_out), float("nan"), device=cuda_device, dtype=torch.bfloat16)
            # First call reports device errors into a caller-owned word, the second into the shared one.
            word = status.data_ptr() if call == 0 else None
            _lib.check(_run_static(lib, 0, stream, rows, n_out, k_in, splits, flags, x.data_ptr(), w.data_ptr(),
                                   bias.data_ptr(), out.data_ptr(), word))
            torch.cuda.synchronize(cuda_device)
            ok, msg = offn.check_close(out, ref)
            assert ok, f"call {call}, splits {splits}: {msg}"
            oracle = offn.bf16(x.float() @ weight.float().T + bias.float())
            ok, msg = offn.check_close(out, oracle)
            assert ok, f"call {call}, splits {splits}, against the oracle: {msg}"
        assert int(status.item()) == 0
    finally:
        lib.wamffn_linear_plan_destroy(plan)
