"""CPU oracle of the talker decode step — TEST INFRASTRUCTURE ONLY.

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg import
this package, and only as the checker or the timed CPU baseline.  The product
(sglang-omni_b200/omni_b200) never imports it.

- ``oracle.sampler``: ctypes binding of omni_oracle.c (integer, packing and
  sampling arithmetic, bit-exact specification).
- ``oracle.model``: fp32 PyTorch-CPU restatement of the talker layer, paged
  attention, MoE and the code-predictor loop.
"""
