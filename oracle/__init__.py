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
  front      -- the GDN layer glue around the recurrence: causal conv taps,
                SiLU, q/k norms, the gates from their logits and the gated
                RMS norm, with the reference's bf16 rounding points.
  cpu_step   -- the timed CPU baseline: one decode step of sampled sequences
                through every layer on the host cores.
The scheduler, prefix cache, request lifecycle and byte admission are pinned
by traces of the reference's own classes and functions (tests/golden/), not
restated here.

Parity pins: every restatement is checked against golden vectors produced by
the reference's own code (``tests/golden/make_golden.py``) and against the
reference tests' known answers.
"""
