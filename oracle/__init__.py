"""CPU oracle for the scene-packed attention path — TEST INFRASTRUCTURE ONLY.

This package restates, on the CPU, what the OneReel reference computes on its hot path, so that the CUDA product can be
checked against it:

  oracle.layout_oracle     scene layout, Algorithm 1 partition, exchange sets, Eq. 2 and the packed segment order
                           (reference: src/onereel/layout.py, src/onereel/parallel/comm.py,
                           src/onereel/models/hunyuan15.py `_segments`, src/onereel/models/wan.py `ranges`)
  oracle.attention_oracle  per-segment softmax attention in float32/float64 numpy, the log-sum-exp, the LSE merge and
                           the scene processors' outputs (reference: src/onereel/attention.py, which calls
                           flash-attn 2.8.3.post1 `flash_attn_varlen_func`; its published algorithm is exact softmax
                           attention, restated here directly)
  oracle.frame_memory_oracle per-frame pooling and the cosine k-means choice of representative frames in float64
                           numpy (reference: src/onereel/frame_memory.py)

Only `tests/`, `__graft_entry__.smoke()` and `bench.py`'s CPU-baseline leg may import this package, and only as the
checker or the timed CPU baseline. The product (`onereel_b200`) never imports it and has no CPU fallback.

Parity pinning: the restatement is checked against golden vectors produced by running the reference's own Python code
(tests/golden/make_golden.py, committed with its outputs) and against the known-answer tests of the reference's
tests/test_onereel_layout.py and tests/test_onereel_frame_memory.py.
"""
