"""CPU oracle for the CRESSO5 optimizer step (test infrastructure only).

This package restates, in plain torch/numpy, the arithmetic of the reference
PyTorch path (``cresso_v5.CRESSO5`` with ``cuda_ops='off'``) so that the CUDA
product path can be checked against it.  It is imported only by ``tests/``,
``__graft_entry__.smoke()`` and the ``cpu_baseline`` / ``--impl reference``
legs of ``bench.py``.  The product package ``cresso_b200`` never imports it.

Parity pin: ``tests/golden/`` holds vectors produced by the reference code
itself (``tests/golden/make_golden.py``); ``tests/test_oracle_golden.py``
checks this restatement against them.
"""
