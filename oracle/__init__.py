"""CPU oracle for the GQA attention core -- TEST INFRASTRUCTURE ONLY.

Nothing in the product package imports this.  Only ``tests/``,
``__graft_entry__.smoke()`` and the CPU-baseline / reference legs of
``bench.py`` use it, and only as the checker or as the timed CPU baseline.

* ``oracle.golden``  -- ctypes wrapper over ``gqa_oracle.c``: the bf16-staged
  stage arithmetic of the reference's golden model
  (llama3_attention_golden_model.py:124-190), pinned bit-exactly against the
  reference's committed hex golden vectors (tests/golden/).
* ``oracle.cpu_port`` -- NumPy restatement of CPU_Baseline's fp32 GQA core
  (CPU_Baseline/cpu_baseline/attention.py:11-84, bf16.py:6-14,
  config.py:19-91, metrics.py:22-40) used as the fp32 reference and as the
  timed CPU baseline.
"""
