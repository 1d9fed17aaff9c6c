"""A synthetic OpenWAM-shaped model for driving the reference's own joint loop
(test infrastructure only).

The reference's ``ParallelJointLoop`` (WAMInfer/joint.py:24-156) schedules the
Video and Action DiT branches of OpenWAM over two CUDA streams through the
reference's adapters (``VideoAdapter`` / ``ActionAdapter``,
WAMInfer/blocks.py:85-272) and its ``JointDriver`` (joint.py:159-165).  The
model itself comes from the absent ``openwam`` package, so this module builds
blocks with exactly the attributes those adapters read, at the video shapes
of the default request (d = 3072, h = 14336, 24 heads x 128, 3 latent frames
of 120 tokens, a 512-token text context) and an action branch of half the
width (the reference's own test fixture, tests/helpers.py:35-46) whose
attention projects to the shared 24 x 128 heads.  Weights are seeded
synthetic values; everything runs in bf16 on the GPU with the reference's
Triton kernels (Q/K RMSNorm + RoPE, modulated norms, masked attention).

The reference package is imported from baseline/_ref through the stub parent
package of baseline/reference_phase.py; ``reference_graphs`` adds the
reference's CUDA-graph wrapper.
"""

from __future__ import annotations

import sys
from pathlib import Path
from types import ModuleType, SimpleNamespace

import torch
from torch import nn

D, H, HEADS, HEAD_DIM = 3072, 14336, 24, 128
DA, HA = 1536, 6144
FRAMES, TOKENS_PER_FRAME, ACTION_ROWS, CONTEXT = 3, 120, 32, 512
SEQ = FRAMES * TOKENS_PER_FRAME


def reference():
    sys.path.insert(0, str(Path(__file__).resolve().parents[1] / "baseline"))
    import reference_phase as rp

    reason = rp.missing(cuda=True)
    if reason:
        return None, reason
    ns = rp.import_reference(cuda=True)
    from WAMInfer import joint

    ns.joint = joint
    return ns, None


def reference_graphs():
    """The reference's ``WAMInfer.graphs`` (``CudaGraphForward``, graphs.py:30-128).
    The module imports ``openwam``'s ``CausalConv3d`` for its VAE graph only; a
    stand-in class under that module path lets it import without openwam.  Its
    input guard is the reference's own C++ extension, built on first use by
    ``graphs.extension()`` (torch.utils.cpp_extension, g++)."""
    names = ["openwam", "openwam.model", "openwam.model.video_backbone", "openwam.model.video_backbone.wan",
             "openwam.model.video_backbone.wan.models", "openwam.model.video_backbone.wan.models.vae"]
    for name in names:
        sys.modules.setdefault(name, ModuleType(name))
    vae = sys.modules[names[-1]]
    if not hasattr(vae, "CausalConv3d"):
        vae.CausalConv3d = type("CausalConv3d", (nn.Conv3d,), {})
    from WAMInfer import graphs

    return graphs


class _Attention(nn.Module):
    def __init__(self, dim: int):
        super().__init__()
        inner = HEADS * HEAD_DIM
        self.q, self.k, self.v = nn.Linear(dim, inner), nn.Linear(dim, inner), nn.Linear(dim, inner)
        self.o = nn.Linear(inner, dim)
        self.norm_q, self.norm_k = nn.RMSNorm(inner, eps=1e-6), nn.RMSNorm(inner, eps=1e-6)
        self.num_heads = HEADS


class _VideoBlock(nn.Module):
    def __init__(self):
        super().__init__()
        self.modulation = nn.Parameter(torch.empty(1, 6, D))
        self.norm1 = nn.LayerNorm(D, eps=1e-6, elementwise_affine=False)
        self.self_attn = _Attention(D)
        self.norm3 = nn.LayerNorm(D, eps=1e-6)
        self.cross_attn = _Attention(D)
        self.norm2 = nn.LayerNorm(D, eps=1e-6, elementwise_affine=False)
        self.ffn = nn.Sequential(nn.Linear(D, H), nn.GELU(approximate="tanh"), nn.Linear(H, D))


class _ActionBlock(nn.Module):
    def __init__(self):
        super().__init__()
        self.modulation = nn.Parameter(torch.empty(1, 6, DA))
        self.self_attn_norm = nn.LayerNorm(DA, eps=1e-6, elementwise_affine=False)
        self.self_attn = _Attention(DA)
        self.cross_attn = _Attention(DA)
        self.context_attn_norm = nn.LayerNorm(DA, eps=1e-6)
        self.ffn_norm = nn.LayerNorm(DA, eps=1e-6, elementwise_affine=False)
        self.ffn = nn.Sequential(nn.Linear(DA, HA), nn.GELU(approximate="tanh"), nn.Linear(HA, DA))


def _init(module: nn.Module, g: torch.Generator) -> nn.Module:
    """Seeded synthetic parameters: linear weights N(0, 0.02), biases and
    modulation N(0, 0.01) / N(0, 0.1), norm weights 1 + N(0, 0.05)."""
    with torch.no_grad():
        for name, p in module.named_parameters():
            if name.endswith("modulation"):
                p.copy_(torch.randn(p.shape, generator=g) * 0.1)
            elif "norm" in name and name.endswith("weight"):
                p.copy_(1 + torch.randn(p.shape, generator=g) * 0.05)
            elif name.endswith("weight"):
                p.copy_(torch.randn(p.shape, generator=g) * 0.02)
            else:
                p.copy_(torch.randn(p.shape, generator=g) * 0.01)
    return module


def _rope(rows: int, device) -> torch.Tensor:
    positions = torch.arange(rows, dtype=torch.float64)[:, None]
    inv = 10000.0 ** (-torch.arange(HEAD_DIM // 2, dtype=torch.float64) / (HEAD_DIM // 2))
    angles = (positions * inv)[:, None, :]
    return torch.polar(torch.ones_like(angles), angles).to(torch.complex64).to(device)


class JointModel:
    """Video and action branches of `layers` blocks, the reference's adapters
    over them, and the reference's driver."""

    def __init__(self, ref, layers: int, device, seed: int = 0):
        self.ref, self.layers, self.device = ref, layers, torch.device(device)
        g = torch.Generator().manual_seed(seed)
        self.video_blocks = [_init(_VideoBlock(), g).to(device=device, dtype=torch.bfloat16).eval()
                             for _ in range(layers)]
        self.action_blocks = [_init(_ActionBlock(), g).to(device=device, dtype=torch.bfloat16).eval()
                              for _ in range(layers)]
        for b in self.video_blocks + self.action_blocks:
            b.requires_grad_(False)
        with torch.no_grad():
            for b in self.video_blocks + self.action_blocks:
                ref.blocks.prepare_packed_weights(b.self_attn, "qkv")
        native_video = SimpleNamespace(dit=SimpleNamespace(blocks=self.video_blocks), num_layers=layers, training=False)
        native_action = SimpleNamespace(blocks=self.action_blocks, num_heads=HEADS, training=False)
        self.vb = ref.blocks.VideoAdapter(native_video)
        self.vb.ffn = None
        self.ab = ref.blocks.ActionAdapter(native_action)
        native_driver = SimpleNamespace(
            num_heads=HEADS, num_layers=layers, attention_mask_mode="mutual",
            _video_tokens_per_frame=lambda state: TOKENS_PER_FRAME,
            _build_attention_mask=lambda **kw: None)
        self.driver = ref.joint.JointDriver(native_driver, self.vb, self.ab)
        self.arch = SimpleNamespace(mot_driver=self.driver, device=self.device)
        # Request inputs (seeded): video latents after patch embedding, per-token
        # time modulation, the text context's K/V per layer for both branches.
        gd = torch.Generator(device=device).manual_seed(seed + 1)

        def rnd(*shape, std=1.0):
            return (torch.randn(*shape, device=device, generator=gd) * std).to(torch.bfloat16)

        self.video = rnd(1, SEQ, D)
        self.video_time = rnd(1, SEQ, 6, D, std=0.1)
        self.action = rnd(1, ACTION_ROWS, DA)
        self.action_time = rnd(1, 6, DA, std=0.1)
        self.context_mask = torch.ones(1, CONTEXT, dtype=torch.bool, device=device)
        self.context_mask[:, 400:] = False  # a padded text prompt
        self.video_kv = [(rnd(1, CONTEXT, HEADS * HEAD_DIM), rnd(1, CONTEXT, HEADS * HEAD_DIM)) for _ in range(layers)]
        self.action_kv = [(rnd(1, CONTEXT, HEADS * HEAD_DIM), rnd(1, CONTEXT, HEADS * HEAD_DIM))
                          for _ in range(layers)]
        self.video_rope, self.action_rope = _rope(SEQ, device), _rope(ACTION_ROWS, device)
        # Token reuse: the previous observation's current-frame features, the
        # FFN history of layers 1.. and the RGB-mandatory rows.
        self.features = rnd(1, TOKENS_PER_FRAME, D)
        self.history = rnd(layers - 1, 1, TOKENS_PER_FRAME, D) if layers > 1 else None
        mg = torch.Generator().manual_seed(seed + 2)
        self.mandatory = (torch.rand(TOKENS_PER_FRAME, generator=mg) < 0.05).to(device)

    def states(self, reuse_count: int | None = None, video: torch.Tensor | None = None,
               action: torch.Tensor | None = None):
        """Fresh video / action states of the request (the loop mutates them).
        With reuse_count, token reuse with that capacity (runtime.py:244-246);
        video / action replace the request's hidden states (used as they are)."""
        extras = {"_inference_context_kv": self.video_kv, "action_only": False, "record_first_frame": False}
        if reuse_count is not None:
            extras.update(token_reuse=dict(n=TOKENS_PER_FRAME, count=reuse_count, mandatory=self.mandatory,
                                           features=self.features, cache=self.history),
                          token_outputs=[])
        video = self.ref.blocks.VideoState(
            hidden_states=self.video.clone() if video is None else video, time_mod=self.video_time, rope_freqs=self.video_rope,
            context_mask=self.context_mask, grid_frames=FRAMES, grid_height=12, grid_width=10, extras=extras)
        action = self.ref.blocks.ActionState(
            x_action=self.action.clone() if action is None else action, t_mod=self.action_time, action_freqs=self.action_rope,
            context_mask=self.context_mask, context_kv=self.action_kv)
        return video, action

    def loop(self, compiled: bool):
        """The reference's ParallelJointLoop; with compiled=False its phases
        run eagerly (torch.compile replaced by the identity while it is built,
        the scheduling and stream joins unchanged)."""
        if compiled:
            return self.ref.joint.ParallelJointLoop(self.arch)
        real = torch.compile
        torch.compile = lambda fn, **kw: fn
        try:
            return self.ref.joint.ParallelJointLoop(self.arch)
        finally:
            torch.compile = real
