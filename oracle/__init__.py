"""CPU oracle for the HeatKV hot path - TEST INFRASTRUCTURE ONLY.

This package restates, in numpy, what the reference computes on its hot path so that the CUDA
implementation in ``heatkv_b200`` can be checked against it:

* ``oracle.attention`` - flat-slab segmented attention, after ``_flat_segmented_attention_reference``
  (real_pruning_fused_attention.py:312-361) and the Triton kernel it stands in for (:76-267).
* ``oracle.pack`` - the slab compaction copy, after ``_pack_flat_segments_kv_kernel`` (:33-73)
  and the ``index_select`` route of ``_segmented_flat_static_copy_precomputed_runs``
  (enable_real_pruning_fast.py:763-869).

The oracle is pinned against fixtures produced by running the reference itself
(tests/golden/make_golden.py). Only ``tests/``, ``__graft_entry__.smoke()`` and the CPU-baseline
leg of ``bench.py`` may import it; the product package never does.
"""
