"""GPU: the per-layer FFN phase inside the reference's branch-overlap pattern.

``ParallelJointLoop._run`` (``WAMInfer/joint.py:116-146``) runs the Action
branch on a side stream while the Video FFN runs on the main stream, joining
the streams at every layer, and ``CudaGraphForward`` replays the whole loop
as one CUDA graph.  Here the video FFN phase is this library's op
(``wam_ffn::ffn_block``, token reuse and history included) and a stand-in
action branch (a narrower torch FFN over 32 rows, the action width being half
the video width in the reference's fixtures) runs on the side stream with the
same waits.  The FFN outputs must not depend on the overlap: eager serial,
eager overlapped and graph-replayed overlapped runs are bit-identical.
"""

import pytest
import torch
import torch.nn.functional as F

pytestmark = pytest.mark.gpu

D, H, SEQ, N, COUNT, LAYERS = 3072, 14336, 392, 120, 32, 3
DA, HA, ROWS_A = 1536, 6144, 32


def test_ffn_phase_under_joint_loop_overlap(cuda_device):
    from waminfer_b200.blocks import _BLOCK_PLANS, BlockPlan, ffn_block, register_block_plan, release_block_plan
    from waminfer_b200.ffn import pack_weight

    g = torch.Generator(device=cuda_device).manual_seed(90)

    def rnd(*shape, std=1.0):
        return (torch.randn(*shape, device=cuda_device, generator=g) * std).to(torch.bfloat16)

    layers = [dict(w_up=pack_weight(rnd(H, D, std=0.02)), b_up=rnd(H, std=0.01), w_down=pack_weight(rnd(D, H, std=0.02)),
                   b_down=rnd(D, std=0.01), mod=rnd(1, 6, D, std=0.1)) for _ in range(LAYERS)]
    action = [(rnd(HA, DA, std=0.02), rnd(DA, HA, std=0.02)) for _ in range(LAYERS)]
    x0, time = rnd(1, SEQ, D), rnd(1, SEQ, 6, D, std=0.1)
    a0 = rnd(1, ROWS_A, DA)
    chosen = torch.randperm(N, generator=torch.Generator().manual_seed(3))[:COUNT].sort().values
    indices = torch.cat((chosen, torch.arange(N, SEQ))).to(cuda_device)
    caches = [rnd(1, N, D) for _ in range(LAYERS)]
    plan_id = register_block_plan(BlockPlan(cuda_device, SEQ, SEQ, D, H))
    main = torch.cuda.Stream(cuda_device)
    side = torch.cuda.Stream(cuda_device)
    main.wait_stream(torch.cuda.current_stream(cuda_device))  # inputs were made on the default stream

    def run(overlap):
        x, a, history = x0, a0, []
        side.wait_stream(main)
        for layer, w in enumerate(layers):
            main.wait_stream(side)  # the joint attention consumes both branches
            if overlap:
                side.wait_stream(main)
                with torch.cuda.stream(side):  # the action branch overlaps the video FFN
                    wu, wd = action[layer]
                    a = a + F.linear(F.gelu(F.linear(a, wu), approximate="tanh"), wd)
            reuse = layer > 0
            x, _, clean = ffn_block(x, None, None, w["mod"], time, w["w_up"], w["b_up"], w["w_down"], w["b_down"],
                                    indices if reuse else None, caches[layer] if reuse else None,
                                    N if reuse else 0, plan_id, 1e-6, False)
            history.append(clean)
            if not overlap:
                wu, wd = action[layer]
                a = a + F.linear(F.gelu(F.linear(a, wu), approximate="tanh"), wd)
        main.wait_stream(side)
        return x, history, a

    try:
        with torch.no_grad(), torch.cuda.stream(main):
            serial = run(False)
            overlapped = run(True)
            torch.cuda.synchronize()
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(graph, stream=main):
                captured = run(True)
            graph.replay()
            torch.cuda.synchronize()
        for other in (overlapped, captured):
            assert torch.equal(other[0], serial[0])
            for h_other, h_serial in zip(other[1], serial[1]):
                assert torch.equal(h_other, h_serial)
        assert _BLOCK_PLANS[plan_id].status() == 0
        graph.reset()
    finally:
        release_block_plan(plan_id)

