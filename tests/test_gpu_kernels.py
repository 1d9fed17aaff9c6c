"""GPU parity of the sm_100a kernels against the fp32 oracle.

Tolerance (made well-posed for bf16): every output
element within max(2e-2, one bf16 ulp of the fp32-oracle value) and the mean
relative error within 5e-3; indices, cache positions and rows served from the
cache are bit-exact.
"""

import pytest
import torch

from oracle import ffn as offn

pytestmark = pytest.mark.gpu

D, H = 3072, 14336


def close(actual, expected, what=""):
    """Elementwise within max(2e-2, one bf16 ulp of the reference); mean relative
    error within 5e-3 (oracle.ffn.check_close)."""
    ok, msg = offn.check_close(actual, expected)
    assert ok, f"{what}: {msg}"


@pytest.fixture(scope="module")
def weights(cuda_device):
    torch.backends.cuda.matmul.allow_tf32 = False
    g = torch.Generator(device=cuda_device).manual_seed(1234)

    def rnd(*shape, std):
        return (torch.randn(*shape, device=cuda_device, generator=g) * std).to(torch.bfloat16)

    return dict(
        w_up=rnd(H, D, std=0.02), b_up=rnd(H, std=0.01), w_down=rnd(D, H, std=0.02), b_down=rnd(D, std=0.01),
        mod=rnd(1, 6, D, std=0.1), gen=g,
    )


def randn(shape, device, g, std=1.0):
    return (torch.randn(*shape, device=device, generator=g) * std).to(torch.bfloat16)


def test_pack_weight_is_the_tile_permutation(cuda_device, weights):
    from waminfer_b200.ffn import pack_weight

    for w in (weights["w_up"], weights["w_down"]):
        n, k = w.shape
        packed = pack_weight(w)
        expected = w.view(n // 128, 128, k // 64, 64).permute(0, 2, 1, 3).contiguous()
        assert torch.equal(packed, expected)


@pytest.fixture(scope="module")
def packed(weights):
    from waminfer_b200.ffn import pack_weight

    return {"w_up": pack_weight(weights["w_up"]), "w_down": pack_weight(weights["w_down"])}


@pytest.mark.parametrize("layout", ["packed", "rowmajor"])
@pytest.mark.parametrize("rows", [1, 16, 17, 100, 240, 257, 272, 304, 336, 360, 392, 512])
def test_up_projection_gelu(cuda_device, weights, packed, rows, layout):
    from waminfer_b200.ffn import Plan

    x = randn((rows, D), cuda_device, weights["gen"])
    w = packed["w_up"] if layout == "packed" else weights["w_up"]
    plan = Plan(x, w, weights["b_up"], exhaustive=False, gelu=True)
    out = plan.run(x, w, weights["b_up"])
    ref = offn.bf16(offn.gelu_tanh(x.float() @ weights["w_up"].float().T + weights["b_up"].float()))
    close(out, ref)
    assert plan.status() == 0
    plan.close()


@pytest.mark.parametrize("rows", [16, 128])
def test_tuned_gelu_plan_never_splits_k(cuda_device, weights, packed, rows):
    """The split-K reduction applies the bias only, so tuning must keep GELU
    plans at one split (the tuner times the candidates on the device)."""
    from waminfer_b200.ffn import Plan

    x = randn((rows, D), cuda_device, weights["gen"])
    plan = Plan(x, packed["w_up"], weights["b_up"], exhaustive=True, gelu=True)
    assert plan.selected_configuration()[4] == 1
    out = plan.run(x, packed["w_up"], weights["b_up"])
    ref = offn.bf16(offn.gelu_tanh(x.float() @ weights["w_up"].float().T + weights["b_up"].float()))
    close(out, ref)
    plan.close()


@pytest.mark.parametrize("layout", ["packed", "rowmajor"])
@pytest.mark.parametrize("rows", [1, 17, 240, 272, 304, 360, 392, 512])
def test_down_projection_split_k(cuda_device, weights, packed, rows, layout):
    from waminfer_b200.ffn import Plan

    h = randn((rows, H), cuda_device, weights["gen"], std=0.5)
    w = packed["w_down"] if layout == "packed" else weights["w_down"]
    plan = Plan(h, w, weights["b_down"], exhaustive=True, gelu=False)
    out = plan.run(h, w, weights["b_down"])
    ref = offn.bf16(h.float() @ weights["w_down"].float().T + weights["b_down"].float())
    close(out, ref)
    assert plan.selected_configuration()[-1] == 1  # tuned
    assert plan.status() == 0
    plan.close()


@pytest.mark.parametrize("rows,n_out", [(392, 3072), (392, 9216), (304, 3072), (100, 3072), (17, 640), (513 - 1, 384)])
def test_linear_layouts_split_k_and_token_groups(cuda_device, rows, n_out):
    """Every layout the tuner may pick -- split-K x token groups (grid.z) --
    against the fp32 oracle, for the attention projections' shapes (d x d and
    the packed QKV 3d x d at the DiT's row counts) and odd ones; one bf16
    rounding of the same fp32 sum, so the layouts agree with each other
    within one bf16 ulp."""
    from waminfer_b200.ffn import Plan, pack_weight

    g = torch.Generator(device=cuda_device).manual_seed(rows * 7 + n_out)
    x = randn((rows, D), cuda_device, g)
    w = (torch.randn(n_out, D, device=cuda_device, generator=g) * 0.02).to(torch.bfloat16)
    bias = (torch.randn(n_out, device=cuda_device, generator=g) * 0.01).to(torch.bfloat16)
    ref = offn.bf16(x.float() @ w.float().T + bias.float())
    pw = pack_weight(w)
    plan = Plan(x, pw, bias, exhaustive=True, gelu=False)
    tuned = plan.layout()
    close(plan.run(x, pw, bias), ref, f"tuned {tuned}")
    for split_k, groups in ((1, 1), (6, 1), (3, 2), (2, 3), (1, 2), (1, 4), (2, 2), (4, 1)):
        if (rows + groups - 1) // groups > 512:
            continue
        plan.set_layout(split_k, groups)
        assert plan.layout() == {"split_k": split_k, "token_groups": groups, "streamk_groups": 0}
        out = plan.run(x, pw, bias)
        close(out, ref, f"split_k={split_k} groups={groups}")
        assert plan.status() == 0
    plan.close()


@pytest.mark.parametrize("rows", [100, 300, 392])
def test_gelu_plan_token_groups(cuda_device, weights, packed, rows):
    """The GELU epilogue with the rows cut into token groups (no split-K)."""
    from waminfer_b200.ffn import Plan

    x = randn((rows, D), cuda_device, weights["gen"])
    ref = offn.bf16(offn.gelu_tanh(x.float() @ weights["w_up"].float().T + weights["b_up"].float()))
    plan = Plan(x, packed["w_up"], weights["b_up"], exhaustive=False, gelu=True)
    for groups in (2, 3, 4):
        plan.set_layout(1, groups)
        close(plan.run(x, packed["w_up"], weights["b_up"]), ref, f"groups={groups}")
        assert plan.status() == 0
    with pytest.raises(RuntimeError, match="never splits K"):
        plan.set_layout(2, 1)
    with pytest.raises(RuntimeError, match="groups=5"):
        plan.set_layout(1, 5)
    plan.close()


@pytest.mark.parametrize("gelu", [False, True])
@pytest.mark.parametrize("rows,n_out,k_in", [(1, 384, 256), (100, 384, 1024), (300, 640, 512), (512, 128, 3072)])
def test_single_cta_tiles(cuda_device, rows, n_out, k_in, gelu):
    """An odd number of 128-feature tiles runs one CTA per tile (no UMMA pair),
    with one UMMA up to 256 rows and two above (rows 300, 512); with and
    without tuned split-K, against the fp32 oracle."""
    from waminfer_b200.ffn import Plan, pack_weight

    g = torch.Generator(device=cuda_device).manual_seed(rows + n_out + k_in)
    x = randn((rows, k_in), cuda_device, g)
    w = (torch.randn(n_out, k_in, device=cuda_device, generator=g) * 0.02).to(torch.bfloat16)
    bias = (torch.randn(n_out, device=cuda_device, generator=g) * 0.01).to(torch.bfloat16)
    pre = x.float() @ w.float().T + bias.float()
    ref = offn.bf16(offn.gelu_tanh(pre) if gelu else pre)
    for weight in (w, pack_weight(w)):
        for exhaustive in (False, True):
            plan = Plan(x, weight, bias, exhaustive=exhaustive, gelu=gelu)
            assert plan.selected_configuration()[0] == 128  # one CTA per 128-feature tile
            close(plan.run(x, weight, bias), ref)
            assert plan.status() == 0
            plan.close()


def _block_inputs(cuda_device, weights, seq, per_token=True):
    g = weights["gen"]
    x = randn((1, seq, D), cuda_device, g)
    update = randn((1, seq, D), cuda_device, g)
    time = randn((1, seq, 6, D), cuda_device, g, std=0.1) if per_token else randn((1, 6, D), cuda_device, g, std=0.1)
    return x, update, time


def _oracle_block(x, update, normalized, mod, time, weights, indices, cache, n):
    t = time[0].float()
    return offn.ffn_block(
        x[0].float(), None if update is None else update[0].float(),
        None if normalized is None else normalized[0].float(), mod[0].float(), t,
        weights["w_up"], weights["b_up"], weights["w_down"], weights["b_down"],
        None if indices is None else indices.cpu(), None if cache is None else cache.reshape(-1, D).float(), n,
        1e-6, ffn=lambda a, wu, bu, wd, bd: offn.prepared_ffn(a.to(wu.device), wu, bu, wd, bd).cpu())


def _run_block(plan_id, x, update, normalized, mod, time, weights, indices, cache, n, want_output=True, packed=None):
    from waminfer_b200.blocks import ffn_block

    w_up = weights["w_up"] if packed is None else packed["w_up"]
    w_down = weights["w_down"] if packed is None else packed["w_down"]
    return ffn_block(x, update, normalized, mod, time, w_up, weights["b_up"], w_down,
                     weights["b_down"], indices, cache, n, plan_id, 1e-6, want_output)


@pytest.fixture(scope="module")
def block_plan(cuda_device):
    from waminfer_b200.blocks import BlockPlan, register_block_plan, release_block_plan

    plan_id = register_block_plan(BlockPlan(cuda_device, 512, 512, D, H))
    yield plan_id
    release_block_plan(plan_id)


def _cpu(t):
    return t.detach().float().cpu()


def check_residual(x_next, output, x, update, mod, time):
    """The gated residual is elementwise bf16 arithmetic: given the kernel's FFN
    output it must equal the oracle's fold bit for bit."""
    y, _ = offn.modulated_norm(_cpu(x)[0], None if update is None else _cpu(update)[0], _cpu(mod)[0], None,
                               _cpu(time)[0], None, None, offn.CROSS_RESIDUAL, 1e-6)
    expected = offn.gate_residual(y, _cpu(output)[0], _cpu(mod)[0], _cpu(time)[0])
    assert torch.equal(_cpu(x_next)[0], expected), "x_next differs from the residual fold of the output"


@pytest.mark.parametrize("seq,per_token", [(392, True), (360, True), (240, False), (33, True)])
def test_block_full_refresh(cuda_device, weights, block_plan, seq, per_token):
    x, update, time = _block_inputs(cuda_device, weights, seq, per_token)
    x_next, output, clean = _run_block(block_plan, x, update, None, weights["mod"], time, weights, None, None, 0)
    rx, rout, _, _ = _oracle_block(_cpu(x), _cpu(update), None, _cpu(weights["mod"]), _cpu(time), weights, None,
                                   None, 0)
    close(output[0], rout, "output")
    check_residual(x_next, output, x, update, weights["mod"], time)
    assert clean.numel() == 0


@pytest.mark.parametrize("count,index_dtype", [(32, torch.int64), (64, torch.int32), (96, torch.int64)])
def test_block_token_reuse_reference_mode(cuda_device, weights, packed, block_plan, count, index_dtype):
    """Reference semantics: n = 120 current rows, `count` recomputed, 240 future
    + 32 action rows always fresh; non-selected rows come from the cache."""
    n, seq = 120, 392
    g = torch.Generator().manual_seed(count)
    chosen = torch.randperm(n, generator=g)[:count].sort().values
    indices = torch.cat((chosen, torch.arange(n, seq))).to(index_dtype).to(cuda_device)
    x, update, time = _block_inputs(cuda_device, weights, seq)
    cache = randn((1, n, D), cuda_device, weights["gen"])
    x_next, output, clean = _run_block(block_plan, x, update, None, weights["mod"], time, weights, indices, cache, n,
                                       packed=packed)
    rx, rout, rclean, _ = _oracle_block(_cpu(x), _cpu(update), None, _cpu(weights["mod"]), _cpu(time), weights,
                                        indices.long(), _cpu(cache), n)
    kept = sorted(set(range(n)) - set(chosen.tolist()))
    # Rows served from the cache are bit-exact copies, in the output and the new history.
    assert torch.equal(output[0, kept].cpu(), cache[0, kept].cpu())
    assert torch.equal(clean[0, kept].cpu(), cache[0, kept].cpu())
    close(output[0], rout, "output")
    close(clean[0], rclean, "clean")
    assert torch.equal(clean[0], output[0, :n])
    check_residual(x_next, output, x, update, weights["mod"], time)


def test_block_baseline_mode_with_pads(cuda_device, weights, block_plan):
    """Per-frame selection over 3 latent frames (cache of 360 rows) with pad
    entries (-1) that are computed on zeros and never scattered."""
    n, seq, k, cap = 360, 392, 16, 32
    g = torch.Generator().manual_seed(7)
    entries = []
    for f in range(3):
        rows = (torch.randperm(120, generator=g)[:k].sort().values + 120 * f).tolist()
        entries += rows + [-1] * (cap - k)
    indices = torch.tensor(entries + list(range(n, seq)), dtype=torch.int32, device=cuda_device)
    x, update, time = _block_inputs(cuda_device, weights, seq)
    cache = randn((n, D), cuda_device, weights["gen"])
    x_next, output, clean = _run_block(block_plan, x, update, None, weights["mod"], time, weights, indices, cache, n)
    rx, rout, rclean, _ = _oracle_block(_cpu(x), _cpu(update), None, _cpu(weights["mod"]), _cpu(time), weights,
                                        indices.long(), _cpu(cache), n)
    selected = {r for r in entries if r >= 0}
    kept = sorted(set(range(n)) - selected)
    assert torch.equal(output[0, kept].cpu(), cache[kept].cpu())
    close(output[0], rout, "output")
    close(clean[0], rclean, "clean")
    assert torch.equal(clean[0], output[0, :n])
    check_residual(x_next, output, x, update, weights["mod"], time)


def test_block_pre_normalized_matches_fused(cuda_device, weights, block_plan):
    """ffn_at_layer_for_compile's form (normalized given) equals the fused norm."""
    from waminfer_b200.norm import CROSS_RESIDUAL, modulated_norm

    seq, n, count = 392, 120, 32
    indices = torch.cat((torch.arange(0, 120, 120 // count)[:count], torch.arange(n, seq))).to(cuda_device)
    x, update, time = _block_inputs(cuda_device, weights, seq)
    cache = randn((1, n, D), cuda_device, weights["gen"])
    y, normalized = modulated_norm(x, update, weights["mod"], None, time, None, None, CROSS_RESIDUAL, 1e-6)
    a = _run_block(block_plan, x, update, None, weights["mod"], time, weights, indices, cache, n)
    b = _run_block(block_plan, y, None, normalized, weights["mod"], time, weights, indices, cache, n)
    for u, v in zip(a, b):
        assert torch.equal(u, v)


def test_modulated_norm_matches_reference_kernel(cuda_device, golden):
    from waminfer_b200.norm import modulated_norm

    for c in golden("modulated_norm.pt"):
        dev = lambda t: None if t is None else t.to(cuda_device)  # noqa: E731
        mode = c["mode"]
        y, n = modulated_norm(dev(c["x"]), dev(c["update"]) if mode else None, dev(c["mod"]),
                              dev(c["previous"]) if mode == 3 else None, dev(c["time"]),
                              dev(c["weight"]) if mode == 1 else None, dev(c["bias"]) if mode == 1 else None,
                              mode, c["eps"])
        assert torch.equal(y.cpu(), c["y"]), (c["dim"], mode)
        norm_close(n.cpu(), c["norm"], (c["dim"], mode))


def norm_close(n, ref, what):
    """The residual y is exact; the normalised row may differ from the Triton
    kernel by reduction order and rsqrt rounding, which can flip one bf16
    rounding of an intermediate (|n * scale| < 8): at most one ulp there
    (2^-5), on at most 1% of the elements."""
    diff = (n.float() - ref.float()).abs()
    assert float(diff.max()) <= 2.0**-5, (what, float(diff.max()))
    assert float((diff > 0).float().mean()) <= 0.01, (what, float((diff > 0).float().mean()))


def test_streamk_gelu_plans_follow_oracle(cuda_device, tmp_path):
    """Stream-K GELU plans (WAMFFN_STREAMK=1, read once per process, so in a
    child interpreter): single-CTA tiles (odd tile counts) with up to four
    helper pieces per owner tile, and the FFN up projection on UMMA pairs,
    against the fp32 oracle; the plans report their stream-K grid."""
    import os
    import subprocess
    import sys

    script = tmp_path / "sk.py"
    script.write_text(
        "import torch\n"
        "from oracle import ffn as offn\n"
        "from waminfer_b200.ffn import Plan\n"
        "dev = torch.device('cuda', 0)\n"
        "torch.backends.cuda.matmul.allow_tf32 = False\n"
        "g = torch.Generator(device=dev).manual_seed(5)\n"
        "for rows, n_out, k_in in ((1, 384, 256), (100, 384, 1024), (300, 640, 512), (512, 128, 3072),\n"
        "                          (392, 14336, 3072), (304, 14336, 3072), (77, 14336, 3072)):\n"
        "    x = torch.randn(rows, k_in, device=dev, generator=g).bfloat16()\n"
        "    w = (torch.randn(n_out, k_in, device=dev, generator=g) * 0.02).bfloat16()\n"
        "    b = (torch.randn(n_out, device=dev, generator=g) * 0.01).bfloat16()\n"
        "    plan = Plan(x, w, b, exhaustive=False, gelu=True)\n"
        "    import ctypes\n"
        "    from waminfer_b200 import _lib\n"
        "    vals = (ctypes.c_uint32 * 8)()\n"
        "    _lib.check(_lib.lib().wamffn_linear_configuration(plan._handle, vals, 8))\n"
        "    assert vals[7] > 0, (rows, n_out, k_in, list(vals))\n"
        "    for _ in range(2):\n"
        "        out = plan.run(x, w, b)\n"
        "        ref = offn.bf16(offn.gelu_tanh(x.float() @ w.float().T + b.float()))\n"
        "        ok, msg = offn.check_close(out, ref)\n"
        "        assert ok, (rows, n_out, k_in, msg)\n"
        "    assert plan.status() == 0\n"
        "    plan.close()\n"
        "print('ok')\n")
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    env = dict(os.environ, WAMFFN_STREAMK="1", PYTHONPATH=root)
    out = subprocess.run([sys.executable, str(script)], env=env, cwd=root, timeout=600, capture_output=True, text=True)
    assert out.returncode == 0, out.stdout + out.stderr


def test_register_norm_is_bit_identical_to_row_kernel(cuda_device, tmp_path):
    """The standalone op's register-resident kernel (4 warps per row) and the
    shared-memory row kernel that the stack's first layer and the layer
    boundary share compute the same bits, every mode, per-token and shared
    time rows, strided inputs (WAMFFN_NORM_REG is read once per process, so
    each kernel runs in its own child interpreter)."""
    import os
    import subprocess
    import sys

    script = tmp_path / "norm.py"
    script.write_text(
        "import sys, torch\n"
        "from waminfer_b200.norm import modulated_norm\n"
        "dev = torch.device('cuda', 0)\n"
        "g = torch.Generator(device=dev).manual_seed(3)\n"
        "out = {}\n"
        "for dim, rows in ((3072, 392), (1024, 77), (256, 5)):\n"
        "    r = lambda *s, std=1.0: (torch.randn(*s, device=dev, generator=g) * std).bfloat16()\n"
        "    x = r(1, rows, dim + 8)[:, :, 8:]\n"
        "    upd, mod, prev = r(1, rows, dim), r(1, 6, dim, std=0.1), r(1, 6, dim, std=0.1)\n"
        "    w, b = r(dim, std=0.1), r(dim, std=0.1)\n"
        "    for shared in (False, True):\n"
        "        time = r(1, 1, 6, dim, std=0.1) if shared else r(1, rows, 6, dim, std=0.1)\n"
        "        for mode in range(4):\n"
        "            y, n = modulated_norm(x, upd if mode else None, mod, prev if mode == 3 else None, time,\n"
        "                                  w if mode == 1 else None, b if mode == 1 else None, mode, 1e-6)\n"
        "            out[(dim, shared, mode)] = (y.cpu(), n.cpu())\n"
        "torch.save(out, sys.argv[1])\n")
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    results = []
    for flag in ("1", "0"):
        env = dict(os.environ, WAMFFN_NORM_REG=flag, PYTHONPATH=root)
        path = tmp_path / f"norm{flag}.pt"
        subprocess.run([sys.executable, str(script), str(path)], check=True, env=env, cwd=root, timeout=600)
        results.append(torch.load(path))
    assert results[0].keys() == results[1].keys()
    for key in results[0]:
        for a, b in zip(results[0][key], results[1][key]):
            assert torch.equal(a, b), key
