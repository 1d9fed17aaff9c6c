"""Generates the golden fixtures in this folder by running the reference's own code.

Run from the repository root, in a checkout that has the WAMInfer sources:

    PYTHONDONTWRITEBYTECODE=1 python tests/golden/make_golden.py /path/to/WAMInfer-checkout

The reference package is imported through a stub parent module (its
``__init__`` imports the upstream ``openwam`` model, which is not needed for
these functions).  Captured, all on CPU:

* ``modulated_norm.pt`` -- the ``_modulated_norm`` Triton kernel
  (WAMInfer/_triton_inference.py:130-176) in the Triton interpreter, all four
  MODEs, shared and per-token time rows.  The interpreter truncates fp32->bf16
  casts, while compiled Triton rounds to nearest even; the cast is patched to
  round to nearest even so the fixtures hold what the GPU kernel computes.
* ``ffn_phase.pt`` -- ``VideoAdapter.ffn_at_layer_for_compile``
  (WAMInfer/blocks.py:246-272) with the native FFN (``vb.ffn = None``), with and
  without token reuse, on a middle and the last layer, in bf16.
* ``token_reuse.pt`` -- ``TokenReuse.begin`` masks/counts and ``select_tokens``
  indices (WAMInfer/approximation.py) on seeded features, plus the motion
  schedule of ``MotionRefinement``.

Nothing here runs at test time; the tests only load the saved tensors.
"""

from __future__ import annotations

import os
import sys
import types
from pathlib import Path
from types import SimpleNamespace

os.environ.setdefault("TRITON_INTERPRET", "1")

import numpy as np  # noqa: E402
import torch  # noqa: E402

HERE = Path(__file__).resolve().parent


def import_reference(checkout: str):
    stub = types.ModuleType("WAMInfer")
    stub.__path__ = [str(Path(checkout) / "WAMInfer")]
    sys.modules["WAMInfer"] = stub
    import WAMInfer._triton_inference as tri
    import WAMInfer.approximation as approx
    import WAMInfer.blocks as blocks
    return tri, approx, blocks


def float32_to_bf16_bits(values: np.ndarray) -> np.ndarray:
    """IEEE round-to-nearest-even of float32 to bfloat16, returned as uint16 bits."""
    bits = np.ascontiguousarray(values, dtype=np.float32).view(np.uint32).astype(np.uint64)
    rounded = (bits + 0x7FFF + ((bits >> 16) & 1)) >> 16
    nan = np.isnan(values)
    out = rounded.astype(np.uint16)
    out[nan] = ((bits[nan] >> 16) | 0x40).astype(np.uint16)  # keep NaNs quiet NaNs
    return out


def patch_interpreter_rounding():
    """Round fp32->bf16 casts to nearest even in the Triton interpreter (its
    default cast truncates, unlike compiled Triton)."""
    from triton.runtime import interpreter as interp
    import triton.language as tl

    original = interp.InterpreterBuilder.cast_impl

    def cast_impl(self, src, dst_type):
        if src.dtype.scalar == tl.float32 and dst_type.scalar == tl.bfloat16:
            return interp.TensorHandle(float32_to_bf16_bits(src.data), dst_type.scalar)
        return original(self, src, dst_type)

    interp.InterpreterBuilder.cast_impl = cast_impl


def run_norm(tri, x, update, mod, previous, time, weight, bias, mode, eps):
    import triton

    y = torch.empty_like(x)
    norm = torch.empty_like(x)
    ts = time.stride(1) if time.ndim == 4 and time.shape[1] != 1 else 0
    tri._modulated_norm[(x.shape[1],)](
        x, update, mod, previous, time, weight, bias, y, norm,
        x.shape[-1], x.stride(1), 0 if update is None else update.stride(1), ts, mode, eps,
        triton.next_power_of_2(x.shape[-1]), num_warps=4, enable_fp_fusion=False,
    )
    return y, norm


def make_norm_cases(tri):
    g = torch.Generator().manual_seed(11)
    cases = []
    for dim, rows, per_token in ((128, 12, True), (3072, 6, True), (3072, 5, False)):
        def rnd(*shape, scale=1.0):
            return (torch.randn(*shape, generator=g) * scale).to(torch.bfloat16)

        x = rnd(1, rows, dim)
        update = rnd(1, rows, dim)
        mod = rnd(1, 6, dim, scale=0.1)
        previous = rnd(1, 6, dim, scale=0.1)
        time = rnd(1, rows, 6, dim, scale=0.1) if per_token else rnd(1, 6, dim, scale=0.1)
        weight = rnd(dim, scale=0.5) + 1
        bias = rnd(dim, scale=0.1)
        for mode in (0, 1, 2, 3):
            y, norm = run_norm(tri, x, None if mode == 0 else update, mod, previous if mode == 3 else None, time,
                               weight if mode == 1 else None, bias if mode == 1 else None, mode, 1e-6)
            cases.append(dict(dim=dim, rows=rows, mode=mode, per_token=per_token, x=x, update=update, mod=mod,
                              previous=previous, time=time, weight=weight, bias=bias, eps=1e-6, y=y, norm=norm))
    return cases


def make_ffn_cases(blocks_mod):
    cases = []
    g = torch.Generator().manual_seed(5)
    configs = [
        # (d, h, seq, n, indices or None, layer_id, num_layers)
        (128, 512, 12, 4, [0, 3, *range(4, 12)], 1, 3),
        (128, 512, 12, 4, [0, 3, *range(4, 12)], 2, 3),
        (256, 512, 40, 16, None, 1, 3),
        (256, 512, 40, 16, "random", 1, 2),
        (128, 512, 20, 0, None, 0, 2),
    ]
    for d, h, seq, n, idx, layer_id, num_layers in configs:
        torch.manual_seed(1000 + len(cases))
        blocks = []
        for _ in range(num_layers):
            ffn = torch.nn.Sequential(torch.nn.Linear(d, h), torch.nn.GELU(approximate="tanh"), torch.nn.Linear(h, d))
            ffn = ffn.to(torch.bfloat16).eval()
            modulation = torch.nn.Parameter((torch.randn(1, 6, d) * 0.1).to(torch.bfloat16), requires_grad=False)
            blocks.append(SimpleNamespace(ffn=ffn, modulation=modulation))
        native = SimpleNamespace(dit=SimpleNamespace(blocks=blocks), num_layers=num_layers)
        vb = blocks_mod.VideoAdapter(native)
        vb.ffn = None
        x = torch.randn(1, seq, d, generator=g).to(torch.bfloat16)
        normalized = torch.randn(1, seq, d, generator=g).to(torch.bfloat16)
        time_mod = (torch.randn(1, seq, 6, d, generator=g) * 0.1).to(torch.bfloat16)
        extras = {}
        indices = None
        cache = None
        if n > 0:
            if idx == "random":
                count = 6
                chosen = torch.randperm(n, generator=g)[:count].sort().values
                indices = torch.cat((chosen, torch.arange(n, seq)))
            elif idx is not None:
                indices = torch.tensor(idx)
                count = indices.numel() - (seq - n)
            else:
                count = n
            cache = (torch.randn(num_layers - 1, 1, n, d, generator=g)).to(torch.bfloat16)
            extras = dict(token_reuse=dict(n=n, count=count, cache=cache), token_outputs=[])
            if indices is not None:
                extras["token_indices"] = indices
        state = SimpleNamespace(time_mod=time_mod, extras=extras, hidden_states=None)
        with torch.no_grad():
            vb.ffn_at_layer_for_compile(layer_id, state, normalized, x)
        pending = state.extras.get("_inference_ffn_residual")
        case = dict(d=d, h=h, seq=seq, n=n, layer_id=layer_id, num_layers=num_layers, x=x, normalized=normalized,
                    time_mod=time_mod, modulation=blocks[layer_id].modulation.detach().clone(),
                    w_up=blocks[layer_id].ffn[0].weight.detach().clone(),
                    b_up=blocks[layer_id].ffn[0].bias.detach().clone(),
                    w_down=blocks[layer_id].ffn[2].weight.detach().clone(),
                    b_down=blocks[layer_id].ffn[2].bias.detach().clone(),
                    indices=indices, cache=None if cache is None else cache[layer_id - 1].clone(),
                    hidden_states=state.hidden_states,
                    output=None if pending is None else pending[0],
                    token_outputs=state.extras.get("token_outputs"))
        cases.append(case)
    return cases


def make_reuse_cases(approx):
    out = {}
    # Reference test re-expressed: capacity rounding, mandatory token, ties -> smaller index.
    history = approx.TokenReuse((1, 2, 3, 4))
    inputs = dict(latents=torch.zeros(1, 4, 3, 4, 4))
    image = np.zeros((8, 8, 3), dtype=np.uint8)
    reuse, observation = history.begin(image, inputs, "task", (1, 2, 2))
    out["small_first_count"] = reuse["count"]
    previous = torch.ones(1, 4, 8)
    history.commit(observation, previous, previous.unsqueeze(0))
    image[:4, 4:] = 30
    reuse, _ = history.begin(image, inputs, "task", (1, 2, 2))
    out["small_second_count"] = reuse["count"]
    out["small_second_mandatory"] = reuse["mandatory"].clone()
    state = SimpleNamespace(extras=dict(token_reuse=reuse))
    current = torch.ones(1, 12, 8)
    current[:, 2:4] = 5
    approx.select_tokens(state, current)
    out["small_indices"] = state.extras["token_indices"].clone()

    # RGB threshold boundary on the default geometry (384x320 -> 12x10 patches).
    rng = np.random.default_rng(9)
    base = rng.integers(0, 240, (384, 320, 3), dtype=np.uint8)
    masks = {}
    for dtype in (np.uint8, np.float32, np.float64):
        history = approx.TokenReuse((32, 64, 96, 120))
        lat = dict(latents=torch.zeros(1, 4, 3, 24, 20))
        before = base.astype(dtype)
        _, observation = history.begin(before, lat, "task", (1, 2, 2))
        history.commit(observation, torch.empty(1, 120, 1), torch.empty(1, 1, 120, 1))
        for change in (4.999999, 5.0, 5.000001, 9.0):
            current = (base.astype(np.float64) + change).astype(dtype)
            reuse, _ = history.begin(current, lat, "task", (1, 2, 2))
            masks[(np.dtype(dtype).name, change)] = (reuse["mandatory"].clone(), reuse["count"])
    out["rgb_masks"] = masks
    out["rgb_base"] = torch.from_numpy(base)

    # Partial-patch changes: a few patches change by more than 5.
    history = approx.TokenReuse((32, 64, 96, 120))
    lat = dict(latents=torch.zeros(1, 4, 3, 24, 20))
    _, observation = history.begin(base, lat, "task", (1, 2, 2))
    history.commit(observation, torch.empty(1, 120, 1), torch.empty(1, 1, 120, 1))
    changed = base.copy()
    changed[0:64, 0:96] = 255 - changed[0:64, 0:96]
    reuse, _ = history.begin(changed, lat, "task", (1, 2, 2))
    out["patch_change_image"] = torch.from_numpy(changed)
    out["patch_change_mandatory"] = reuse["mandatory"].clone()
    out["patch_change_count"] = reuse["count"]

    # select_tokens on seeded first-layer features at the default geometry.
    g = torch.Generator().manual_seed(21)
    selections = []
    # select_tokens reads only the first n rows; the sequence length sets the future rows.
    for count, dim, seq in ((32, 3072, 392), (64, 768, 360), (96, 768, 136)):
        before = torch.randn(1, 120, dim, generator=g).to(torch.bfloat16)
        now = (before.float() + torch.randn(1, 120, dim, generator=g) * torch.rand(1, 120, 1, generator=g)).to(
            torch.bfloat16)
        features = torch.cat((now, torch.zeros(1, seq - 120, dim).to(torch.bfloat16)), dim=1)
        mandatory = torch.rand(120, generator=g) < 0.1
        reuse = dict(n=120, count=count, mandatory=mandatory, features=before)
        state = SimpleNamespace(extras=dict(token_reuse=reuse))
        approx.select_tokens(state, features)
        selections.append(dict(count=count, before=before, features=features[:, :120].clone(), seq=seq,
                               mandatory=mandatory,
                               indices=state.extras["token_indices"].clone()))
    out["selections"] = selections

    # Motion-adaptive 2F/4F schedule (threshold 0.08 m).
    schedule = [(1000 - i * 100,) * 2 for i in range(11)]
    motion = {}
    for m in (0.081, 0.08, 0.005, 0.15, 0.05):
        gate = approx.MotionRefinement(lambda actions, m=m: m, 0.08, schedule)
        before_decision = [i for i in range(4) if gate.full(i)]
        gate.decide(np.zeros((32, 7)))
        motion[m] = before_decision + [i for i in range(4, 10) if gate.full(i)]
    out["motion_full_steps"] = motion
    return out


def main(checkout: str) -> None:
    patch_interpreter_rounding()
    tri, approx, blocks_mod = import_reference(checkout)
    torch.save(make_norm_cases(tri), HERE / "modulated_norm.pt")
    torch.save(make_ffn_cases(blocks_mod), HERE / "ffn_phase.pt")
    torch.save(make_reuse_cases(approx), HERE / "token_reuse.pt")
    for name in ("modulated_norm.pt", "ffn_phase.pt", "token_reuse.pt"):
        print(name, (HERE / name).stat().st_size)


if __name__ == "__main__":
    if len(sys.argv) != 2:
        raise SystemExit("usage: make_golden.py <directory holding the WAMInfer package>")
    main(sys.argv[1])
