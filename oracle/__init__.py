"""CPU oracle of the rollout-cache path: TEST INFRASTRUCTURE, not product code.

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py`` (its CPU
baseline and ``--impl reference`` arm) may import this package, and only as a
checker or as the timed CPU baseline. The product path in ``shellsmith_b200``
never imports it and has no CPU fallback.

Modules:
  gdn        -- gated-delta-net recurrence: float64 sequential form, the one-token
                step (fp32 and the reference's bf16 rounding points) and the
                chunk-64 WY/UT form with its inter-chunk scan.
  attention  -- causal GQA attention with a query offset, split-K partials and
                their (out, lse) combine, and the paged-pool gather.
  scheduler  -- the continuous batcher and the prefix snapshot cache, restated
                for CPU timing and trace checks.

Parity pins: every restatement is checked against golden vectors produced by
the reference's own code (``tests/golden/make_golden.py``) and against the
reference tests' known answers.
"""
