"""CPU restatement of the 2F/4F Euler schedule over the FFN stack -- TEST
INFRASTRUCTURE ONLY (the checker of ``waminfer_b200.euler``).

Schedule and residual replay follow ``WAMInfer/runtime.py:157-201`` and
``WAMInfer/approximation.py:70-84``: the stack runs at updates 0 and 3, plus 6
and 9 when the motion decided after update 3 is at most the threshold; fresh
updates record ``out - x``, the others replay it.  Update 0 gathers the
request's indices and reads its history from layer 1 on
(``WAMInfer/blocks.py:246-264``).  The Euler step ``a + (t_next - t) v`` with
t_k = 1 - k/10 and the clean estimate ``a - t v`` at update 3
(``WAMInfer/runtime.py:184``) are the harness's definitions (the upstream
``flow_step`` is not part of the reference sources).
"""

from __future__ import annotations

import torch

from oracle import ffn as offn

UPDATES = 10
SCHEDULE = [1.0 - k / UPDATES for k in range(UPDATES + 1)]


def fresh_updates(nfe: int) -> list[int]:
    return [0, 3] if nfe == 2 else [0, 3, 6, 9]


def stack_pass(x, time, weights, indices=None, history=None, cache_rows=0, eps=1e-6, device="cpu"):
    """All layers of one pass on the fp32 oracle; layer 0 recomputes every
    row, later layers gather `indices` and read history[layer - 1].  The fp32
    arithmetic runs on `device` (a GPU holding the weights keeps a 30-layer
    oracle fast; matmuls there must run without TF32)."""
    x = x.float().to(device)
    time = time.float().to(device)
    for layer, w in enumerate(weights):
        reuse = indices is not None and layer > 0
        cache = history[layer - 1].float().to(device) if reuse else None
        x, _, _, _ = offn.ffn_block(
            x, None, None, w.mod[0].float().to(device), time, w.w_up, w.b_up, w.w_down, w.b_down,
            indices if reuse else None, cache, cache_rows if reuse else 0, eps,
            ffn=lambda a, wu, bu, wd, bd: offn.prepared_ffn(a, wu.to(device), bu.to(device), wd.to(device),
                                                            bd.to(device)))
    return offn.bf16(x)


def run_euler(weights, video, actions, times, indices, history, cache_rows, amplitude_m, threshold_m=0.05,
              eps=1e-6, device="cpu", pass_fn=None):
    """times: {update: [seq, 6, d]} for the fresh updates.  Returns
    (actions after update 10, fresh updates, nfe) on `device`.

    pass_fn(x, time, indices, history, cache_rows) -> y replaces the oracle's
    FFN stack (default: ``stack_pass`` over `weights`); a test passes another
    implementation's stack to run the same schedule on it."""
    if pass_fn is None:
        def pass_fn(x, time, idx, hist, n):
            return stack_pass(x, time, weights, idx, hist, n, eps, device)
    a = offn.bf16(actions.float().to(device))
    video = video.float().to(device)
    nfe = 2
    residual = None
    fresh = []
    for k in range(UPDATES):
        t, t_next = SCHEDULE[k], SCHEDULE[k + 1]
        x = torch.cat((video, a))
        if k in fresh_updates(nfe):
            fresh.append(k)
            y = pass_fn(x, times[k].float(), indices if k == 0 else None, history if k == 0 else None,
                        cache_rows if k == 0 else 0).float().to(device)
            residual = offn.bf16(y - x)
        else:
            y = offn.bf16(x + residual)
        v = y[video.shape[0]:]
        if k == 3:
            nfe = 2 if amplitude_m > threshold_m else 4
        a = offn.bf16(a + (t_next - t) * v)
    return a, fresh, nfe
