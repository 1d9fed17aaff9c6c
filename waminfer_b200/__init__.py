"""B200-native (sm_100a) implementation of WAMInfer's video-DiT FFN hot path.

Modules mirror the reference's host interface for the path:

* ``waminfer_b200.ffn``     -- ``PreparedFFN``, ``Plan`` and the
  ``wam_ffn::prepared_ffn_linear_v1`` op (reference ``WAMInfer/ffn.py``);
* ``waminfer_b200.norm``    -- ``modulated_norm`` op (reference
  ``WAMInfer/_triton_inference.py``);
* ``waminfer_b200.blocks``  -- the fused FFN phase ``VideoFFN`` and the
  ``wam_ffn::ffn_block`` op (reference ``WAMInfer/blocks.py``);
* ``waminfer_b200.approximation`` -- token reuse and the 2F/4F schedule
  (reference ``WAMInfer/approximation.py``);
* ``waminfer_b200.stack``   -- the 30-layer FFN stack of one request, and
  concurrent request lanes (``FFNStack(lanes=k).enqueue_requests``);
* ``waminfer_b200.tp``      -- the same stack with the hidden dimension split
  across the ranks of a process group (one all-reduce per layer);
* ``waminfer_b200.euler``   -- the 10-update Euler schedule over the stack;
* ``waminfer_b200.projections`` -- attention-side projections on the same GEMM;
* ``waminfer_b200.trace``   -- per-CTA phase timelines of the library's kernels.

All GPU work runs in ``libwamffn.so`` (``waminfer_b200/csrc``); importing an op
module does not load it, calling one does (and raises if it is missing).
"""

__version__ = "0.1.0"
