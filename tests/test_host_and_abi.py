"""CPU: host logic against the reference's golden outputs, and the C ABI surface."""

import ctypes
import re
from pathlib import Path
from types import SimpleNamespace

import numpy as np
import pytest
import torch

ROOT = Path(__file__).resolve().parents[1]


def test_header_declares_exactly_the_exported_symbols():
    from waminfer_b200 import _lib

    header = (ROOT / "include" / "wamffn.h").read_text()
    declared = set(re.findall(r"\b(wamffn_[a-z_]+)\s*\(", header))
    assert declared == set(_lib.EXPORTED_SYMBOLS)


def test_library_loads_and_exports_every_symbol():
    from waminfer_b200 import _lib

    handle = _lib.lib()
    for name in _lib.EXPORTED_SYMBOLS:
        assert hasattr(handle, name), name
    assert handle.wamffn_abi_version() == 2


def test_abi_rejects_bad_arguments_without_a_gpu():
    """Argument validation happens before any CUDA call."""
    from waminfer_b200 import _lib

    lib = _lib.lib()
    out = ctypes.c_void_p()
    assert lib.wamffn_linear_plan_create(0, 0, 128, 64, 1, 0, ctypes.byref(out)) != 0
    assert lib.wamffn_linear_plan_create(0, 600, 128, 64, 1, 0, ctypes.byref(out)) != 0  # > 512 rows
    assert lib.wamffn_linear_plan_create(0, 16, 100, 64, 1, 0, ctypes.byref(out)) != 0   # n_out % 128
    assert b"n_out" in lib.wamffn_last_error()
    assert lib.wamffn_linear_run(None, None, None, None, None, None) == _lib.WAMFFN_ERR_INVALID
    assert lib.wamffn_linear_plan_set_layout(None, 2, 1) == _lib.WAMFFN_ERR_INVALID
    assert b"plan is null" in lib.wamffn_last_error()
    assert lib.wamffn_block_run(None, None, None) == _lib.WAMFFN_ERR_INVALID
    args = _lib.NormArgs(rows=4, dim=12, mode=0)
    assert lib.wamffn_modulated_norm(None, ctypes.byref(args)) == _lib.WAMFFN_ERR_INVALID
    sel = _lib.SelectArgs(n=120, dim=3072, count=120, seq=392)
    assert lib.wamffn_select_tokens(None, ctypes.byref(sel)) == _lib.WAMFFN_ERR_INVALID
    with pytest.raises(_lib.WamffnError):
        _lib.check(lib.wamffn_block_run(None, None, None))
    # Stack entry points: null plan / arguments, and the tensor-parallel hook is required.
    stack = _lib.StackArgs(layers=1)
    assert lib.wamffn_stack_run(None, None, ctypes.byref(stack)) == _lib.WAMFFN_ERR_INVALID
    assert lib.wamffn_stack_run_tp(None, None, ctypes.byref(stack), None, _lib.ALLREDUCE_FN(), None) == \
        _lib.WAMFFN_ERR_INVALID
    assert b"allreduce" in lib.wamffn_last_error()


def test_token_reuse_capacity_and_history(golden):
    from waminfer_b200.approximation import TokenReuse

    g = golden("token_reuse.pt")
    history = TokenReuse((1, 2, 3, 4))
    inputs = dict(latents=torch.zeros(1, 4, 3, 4, 4))
    image = np.zeros((8, 8, 3), dtype=np.uint8)
    reuse, observation = history.begin(image, inputs, "task", (1, 2, 2))
    assert reuse["count"] == g["small_first_count"] == 4
    previous = torch.ones(1, 4, 8)
    history.commit(observation, previous, previous.unsqueeze(0))
    image[:4, 4:] = 30
    reuse, _ = history.begin(image, inputs, "task", (1, 2, 2))
    assert reuse["count"] == g["small_second_count"]
    assert reuse["mandatory"].tolist() == g["small_second_mandatory"].tolist()
    torch.testing.assert_close(history.features, previous)
    assert history.begin(image, inputs, "new task", (1, 2, 2))[0]["count"] == 4  # key change resets


def test_token_reuse_rgb_threshold(golden):
    from waminfer_b200.approximation import TokenReuse

    g = golden("token_reuse.pt")
    base = g["rgb_base"].numpy()
    lat = dict(latents=torch.zeros(1, 4, 3, 24, 20))
    for (dtype, change), (mask, count) in g["rgb_masks"].items():
        history = TokenReuse((32, 64, 96, 120))
        before = base.astype(dtype)
        _, observation = history.begin(before, lat, "task", (1, 2, 2))
        history.commit(observation, torch.empty(1, 120, 1), torch.empty(1, 1, 120, 1))
        before[:] = 0  # the caller recycles its buffer; the snapshot must not change
        current = (base.astype(np.float64) + change).astype(dtype)
        reuse, _ = history.begin(current, lat, "task", (1, 2, 2))
        assert reuse["mandatory"].tolist() == mask.tolist(), (dtype, change)
        assert reuse["count"] == count


def test_token_reuse_rejects_bad_inputs():
    from waminfer_b200.approximation import TokenReuse

    with pytest.raises(ValueError):
        TokenReuse(())
    with pytest.raises(ValueError):
        TokenReuse((0, 4))
    history = TokenReuse((32,))
    with pytest.raises(ValueError):
        history.begin(np.zeros((8, 8)), dict(latents=torch.zeros(1, 4, 3, 4, 4)), "t", (1, 2, 2))
    with pytest.raises(ValueError):
        history.begin(np.zeros((8, 8, 3)), dict(latents=torch.zeros(1, 4, 1, 4, 4)), "t", (1, 2, 2))


def test_motion_refinement_matches_reference(golden):
    from waminfer_b200.approximation import MotionRefinement

    schedule = [(1000 - i * 100,) * 2 for i in range(11)]
    for motion, steps in golden("token_reuse.pt")["motion_full_steps"].items():
        gate = MotionRefinement(lambda actions, m=motion: m, 0.08, schedule)
        got = [i for i in range(4) if gate.full(i)]
        gate.decide(np.zeros((32, 7)))
        got += [i for i in range(4, 10) if gate.full(i)]
        assert got == steps
    with pytest.raises(ValueError, match="motion_metric"):
        MotionRefinement(None, 0.08, schedule)
    with pytest.raises(ValueError, match="10 Euler"):
        MotionRefinement(lambda x: 0.1, 0.08, schedule[:5])
    gate = MotionRefinement(lambda x: float("nan"), 0.08, schedule)
    with pytest.raises(ValueError):
        gate.decide(None)


def test_select_tokens_full_refresh_needs_no_kernel():
    from waminfer_b200.approximation import select_tokens

    features = torch.randn(1, 12, 8)
    state = SimpleNamespace(extras=dict(token_reuse=dict(n=4, count=4)))
    select_tokens(state, features)
    assert "token_indices" not in state.extras
    torch.testing.assert_close(state.extras["token_features"], features[:, :4])


def test_request_geometry_and_flops():
    from waminfer_b200.stack import Geometry

    geo = Geometry()
    assert geo.seq == 392 and geo.reuse_rows == 304
    rows = geo.request_rows()
    assert len(rows) == 60 and rows[0] == 392 and rows[1] == 304 and rows[30:] == [392] * 30
    assert geo.request_flops() == 4 * 3072 * 14336 * (392 + 29 * 304 + 30 * 392)


def test_euler_schedule_matches_oracle_schedule():
    """2F runs the stack at updates 0 and 3; 4F adds 6 and 9 (decided after
    update 3 from the coarse motion against the 0.05 m threshold)."""
    from oracle import euler as oeuler
    from waminfer_b200.approximation import MotionRefinement
    from waminfer_b200.euler import MOTION_THRESHOLD_M, SCHEDULE, UPDATES

    assert SCHEDULE == oeuler.SCHEDULE and UPDATES == oeuler.UPDATES == 10
    for amplitude, nfe in ((0.1, 2), (0.05, 4), (0.02, 4), (0.0501, 2)):
        r = MotionRefinement(lambda clean: amplitude, MOTION_THRESHOLD_M, SCHEDULE)
        fresh = []
        for k in range(UPDATES):
            if r.full(k):
                fresh.append(k)
            if k == 3:
                r.decide(None)
        assert r.nfe == nfe and fresh == oeuler.fresh_updates(nfe)


def test_attention_abi_rejects_before_launching():
    """Argument checks of wamffn_masked_attention run on the host, before any device call."""
    import ctypes

    from waminfer_b200 import _lib

    lib = _lib.lib()
    fake = 256
    args = _lib.AttentionArgs(q=fake, q_row_stride=3072, q_batch_stride=3072 * 392, k=fake, k_row_stride=3072,
                              k_batch_stride=3072 * 392, v=fake, v_row_stride=3072, v_batch_stride=3072 * 392,
                              out=fake, batch=1, nq=392, nk=392, heads=24, head_dim=64)
    assert lib.wamffn_masked_attention(None, ctypes.byref(args)) == 3  # head_dim 64: unsupported
    args.head_dim = 128
    args.q_batch_stride = 3072 * 391  # rows not at one stride across batches
    assert lib.wamffn_masked_attention(None, ctypes.byref(args)) == 1
    assert b"q strides" in lib.wamffn_last_error()
    args.q_batch_stride = 3072 * 392
    args.key_split = 3  # the key split is 1, 2 or 4 CTAs (0: automatic)
    assert lib.wamffn_masked_attention(None, ctypes.byref(args)) == 1
    assert b"key_split" in lib.wamffn_last_error()


def test_structured_attention_abi_rejects_before_launching():
    """Argument checks of wamffn_joint_first_frame_attention and
    wamffn_current_frame_attention run on the host, before any device call."""
    import ctypes

    from waminfer_b200 import _lib

    lib = _lib.lib()
    fake = 256
    view = lambda rows: _lib.RowsView(data=fake, row_stride=3072, batch_stride=3072 * rows)  # noqa: E731
    joint = _lib.JointAttentionArgs(q=view(392), k=view(392), v=view(392), out=fake, batch=1, count=392, video=360,
                                    first=393, heads=24, head_dim=128)
    assert lib.wamffn_joint_first_frame_attention(None, ctypes.byref(joint)) == 1  # first > count
    assert b"first" in lib.wamffn_last_error()
    joint.first, joint.head_dim = 120, 64
    assert lib.wamffn_joint_first_frame_attention(None, ctypes.byref(joint)) == 3  # head_dim 64: unsupported
    joint.head_dim, joint.k = 128, _lib.RowsView(data=fake + 2, row_stride=3072, batch_stride=3072 * 392)
    assert lib.wamffn_joint_first_frame_attention(None, ctypes.byref(joint)) == 1  # k not 16-byte aligned
    assert b"aligned" in lib.wamffn_last_error()

    cur = _lib.CurrentFrameArgs(qv=view(240), qa=view(32), ck=view(120), kv=view(240), ka=view(32), cv=view(120),
                                vv=view(240), va=view(32), ov=fake, oa=fake, batch=1, nc=120, nv=0, na=0, heads=24,
                                head_dim=128)
    assert lib.wamffn_current_frame_attention(None, ctypes.byref(cur)) == 1  # no query rows
    cur.nv, cur.na, cur.key_split = 240, 32, 3
    assert lib.wamffn_current_frame_attention(None, ctypes.byref(cur)) == 1  # key split 3
    assert b"key_split" in lib.wamffn_last_error()
    cur.key_split, cur.oa = 0, None
    assert lib.wamffn_current_frame_attention(None, ctypes.byref(cur)) == 1  # action output missing
    cur.oa, cur.vv = fake, _lib.RowsView(data=fake, row_stride=3072, batch_stride=3072 * 239)
    assert lib.wamffn_current_frame_attention(None, ctypes.byref(cur)) == 1  # vv rows not at one stride
    assert b"vv strides" in lib.wamffn_last_error()
