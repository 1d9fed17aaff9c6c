"""Motion-adaptive Euler schedule over the FFN stack (2F / 4F).

The reference denoises the action latents with 10 Euler updates
(``WAMInfer/runtime.py:157-201``): the Transformer runs only at the "fresh"
updates of ``MotionRefinement`` (0 and 3, plus 6 and 9 when the coarse motion
decided at update 3 is small, ``WAMInfer/approximation.py:70-84``), records
its residual there and replays the cached residual at the other updates.
Here the Transformer is its FFN stack, so one update is

    x_k = [video rows; a_k]                                   (seq rows)
    fresh:  out_k = FFNStack(x_k)   (update 0 with token reuse), residual = out_k - x_k
    cached: out_k = x_k + residual
    v_k   = out_k[action rows]
    a_k+1 = a_k + (t_k+1 - t_k) v_k                           (Euler step)

with t_k = 1 - k / 10.  The action scheduler's ``flow_step`` and the action
decoder are not part of the reference sources (they come from the absent
openwam package), so the step above is this harness's own definition (the
plain flow-matching Euler update), and the motion metric is the caller's:
a drawn coarse displacement in metres, 2F above the 0.05 m threshold.  The
clean estimate handed to the metric at update 3 is ``a - t v``
(``WAMInfer/runtime.py:184``).
"""

from __future__ import annotations

from dataclasses import dataclass

import torch

from waminfer_b200.approximation import MotionRefinement
from waminfer_b200.stack import FFNStack, Geometry, Request

UPDATES = 10
SCHEDULE = [1.0 - k / UPDATES for k in range(UPDATES + 1)]
MOTION_THRESHOLD_M = 0.05


@dataclass
class EulerResult:
    actions: torch.Tensor   # [action, d] bf16 latents after the last update
    fresh: list[int]        # updates that ran the FFN stack
    nfe: int                # 2 or 4


def time_modulation(geo: Geometry, update: int, device, seed: int = 0) -> torch.Tensor:
    """Seeded per-token time modulation [seq, 6, d] of one update."""
    g = torch.Generator(device=device).manual_seed(30_000 + 97 * seed + update)
    return (torch.randn(geo.seq, 6, geo.d, device=device, generator=g) * 0.1).to(torch.bfloat16)


def run_euler(stack: FFNStack, req: Request, actions: torch.Tensor, amplitude_m: float,
              seed: int = 0) -> EulerResult:
    """Runs the 10 updates on the device, on the current stream.  `req`
    supplies the video rows (``req.x[0]`` rows before the action rows), the
    gather list and the history of the token-reuse update 0; `actions`
    [action, d] bf16."""
    geo = stack.geo
    device = stack.device
    stream = torch.cuda.current_stream(device).cuda_stream
    n_video = geo.seq - geo.action
    video = req.x[0][:n_video].clone()
    a = actions.to(device=device, dtype=torch.bfloat16).clone()
    refinement = MotionRefinement(lambda clean: amplitude_m, MOTION_THRESHOLD_M, SCHEDULE)
    residual = None
    fresh_steps = []
    x = torch.empty(geo.seq, geo.d, device=device, dtype=torch.bfloat16)
    out = torch.empty_like(x)
    for k in range(UPDATES):
        t, t_next = SCHEDULE[k], SCHEDULE[k + 1]
        x[:n_video] = video
        x[n_video:] = a
        if refinement.full(k):
            fresh_steps.append(k)
            stack.enqueue_pass(x, out, time_modulation(geo, k, device, seed), stream, reuse=req if k == 0 else None)
            y = out
            residual = (y.float() - x.float()).to(torch.bfloat16)
        else:
            y = (x.float() + residual.float()).to(torch.bfloat16)
        v = y[n_video:].float()
        if k == 3:
            refinement.decide(a.float() - t * v)
        a = (a.float() + (t_next - t) * v).to(torch.bfloat16)
    return EulerResult(a, fresh_steps, refinement.nfe)
