"""CPU oracle for the AOA-KV / Quest sparse-decode path — TEST INFRASTRUCTURE.

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py`` (its
``cpu_baseline`` leg and ``--impl reference`` arm) may import this package,
and only as the checker or the timed CPU baseline. The product path
(``aoa_kv_b200``) never imports it and has no CPU fallback.

Two restatements, in numpy, of the reference's arithmetic:

* ``oracle.sim``          — semantics A, the reference's PyTorch simulation
  (filtering/filter_util.py driven by the decode branch of
  evaluation/quest_attention.py). Pinned against golden vectors produced by
  importing the reference's own filter_util.py (tests/golden/make_golden.py).
* ``oracle.kernel_tree``  — semantics B, what the reference's CUDA tree
  computes (kernels/aoa_kv/...), pinned against golden vectors produced by the
  reference's own CPU test references (quest/tests/test_estimate.py,
  test_approx_attention.py, test_v_log_norm_prefill_claude.py).
"""
