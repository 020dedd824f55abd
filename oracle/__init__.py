"""CPU oracle for the BiGEMM hot path -- TEST INFRASTRUCTURE ONLY.

This package restates, in plain Python and numpy, the reference algorithm of
QuackPhuc/omniwave (package ``omniweave``) for the BiGEMM operator:

* ``oracle.routing`` -- route plans (``omniweave/models/routing.py``), written
  as the same nested loops the reference uses so it is independent of the
  vectorised builder in ``omniwave_b200.routing``.
* ``oracle.bigemm`` -- pack/unpack, the forward delta, its analytic backward
  and the RMSNorm block wrapper (``omniweave/ops/reference.py``,
  ``omniweave/models/block.py``).

Only ``tests/``, ``__graft_entry__.smoke()`` and the CPU-baseline leg of
``bench.py`` may import it, and only as the checker or the timed CPU
baseline.  The product package never imports it.

Parity is pinned: ``tests/test_oracle_golden.py`` checks this oracle against
golden vectors produced by running the reference itself
(``tests/golden/make_golden.py``).
"""
