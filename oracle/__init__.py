"""Test-infrastructure oracle for the InnerQ decode hot path.

``quant_ref`` restates ``src/innerq/quant.py`` and ``cache_ref`` restates
``src/innerq/cache.py`` of mthcom/innerq in numpy, with the reference's
per-op rounding to the input dtype.  Both are pinned against golden vectors
produced by running the reference itself (``tests/golden/make_golden.py``).

This package is the CHECKER, never the thing measured or shipped: only
``tests/``, ``__graft_entry__.smoke()`` and the CPU-baseline legs of
``bench.py`` may import it.  The ``innerq_b200`` product never does.
"""
