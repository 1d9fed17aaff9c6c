"""The 2F/4F Euler schedule over the FFN stack (the motion-adaptive workload): the action
latents after 10 updates from the device stack against the CPU oracle's
schedule, within the FFN tolerance, for a large (2F) and a small (4F) coarse
motion."""

import pytest
import torch

from oracle import euler as oeuler
from oracle import ffn as offn

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("amplitude_m,nfe", [(0.10, 2), (0.02, 4)])
def test_euler_actions_follow_oracle(cuda_device, amplitude_m, nfe):
    from waminfer_b200.euler import run_euler, time_modulation
    from waminfer_b200.stack import FFNStack, Geometry, Request, make_weights

    torch.backends.cuda.matmul.allow_tf32 = False
    geo = Geometry(layers=3)
    weights = make_weights(geo.layers, geo.d, geo.h, cuda_device, seed=31)
    stack = FFNStack(weights, geo, cuda_device)
    req = Request(geo, cuda_device, seed=32)
    g = torch.Generator(device=cuda_device).manual_seed(33)
    actions = torch.randn(geo.action, geo.d, device=cuda_device, generator=g).to(torch.bfloat16)

    result = run_euler(stack, req, actions, amplitude_m, seed=5)
    torch.cuda.synchronize()
    assert stack.plan.status() == 0
    assert result.nfe == nfe
    assert result.fresh == oeuler.fresh_updates(nfe)

    n_video = geo.seq - geo.action
    times = {k: time_modulation(geo, k, cuda_device, 5).cpu() for k in result.fresh}
    ref, fresh, ref_nfe = oeuler.run_euler(weights, req.x[0][:n_video].cpu(), actions.cpu(), times,
                                           req.indices.cpu(), req.history_in.cpu(), geo.current, amplitude_m)
    assert (fresh, ref_nfe) == (result.fresh, result.nfe)
    ok, msg = offn.check_close(result.actions, ref)
    assert ok, f"actions after 10 updates: {msg}"
    stack.close()
