"""CPU oracle of WAMInfer's video-DiT FFN hot path -- TEST INFRASTRUCTURE ONLY.

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline /
reference arm may import this package, and only as the checker or the timed CPU
baseline.  The product (``waminfer_b200``) never calls it: its ops run on the
sm_100a library or raise.

* ``oracle.ffn``    -- torch fp32 restatement of the FFN path with the
                       reference's bf16 rounding points (modulated norm, prepared
                       and native FFN, gather / scatter / gated residual).
* ``oracle.reuse``  -- numpy restatement of TokenReuse (RGB mandatory mask,
                       capacity bucket) and select_tokens (score, stable top-k).
* ``oracle.euler``  -- the 2F/4F Euler schedule over the FFN stack (fresh
                       updates, cached residual replay, Euler step) on the
                       fp32 FFN restatement.

Parity pinning: both are checked against golden vectors produced by running the
reference's own code in this container (``tests/golden/make_golden.py``:
``VideoAdapter.ffn_at_layer_for_compile``, ``PreparedFFN``'s native fallback,
``TokenReuse``, ``select_tokens`` and the ``_modulated_norm`` Triton kernel in the
Triton interpreter with round-to-nearest-even casts) and against the known
answers of the reference's tests (``WAMInfer/tests/test_approximation.py``).
"""
