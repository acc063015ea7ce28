"""CPU oracle for lorafusion's fused multi-adapter LoRA path.

TEST INFRASTRUCTURE ONLY.  Nothing in the shipped package imports this
directory; only ``tests/``, ``__graft_entry__.smoke()`` and the CPU-baseline
leg of ``bench.py`` use it, and only as the checker or as the timed CPU
reference arm.

* :mod:`oracle.mock_oracle` restates ``lorafusion/ops/mock_ops.py`` in numpy.
* :mod:`oracle.scheduler_oracle` restates the integer layout logic of
  ``lorafusion/scheduler`` in plain Python.

Both are pinned against golden fixtures produced by running the reference
itself (``tests/golden/make_golden.py``), see ``tests/test_oracle_golden.py``.
"""
