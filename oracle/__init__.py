"""Oracle: CPU restatement of the reference's sequential scan paths (test infrastructure).

This package is the checker, never the product. Only ``tests/``,
``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline / reference legs may import
it. It restates, in plain PyTorch on the CPU (any dtype; the parity tests use float64),
the reference's own materialised implementations of the three layers on the hot path:

* ``oracle.selective_lru`` — SelectiveLRU / SelectiveLRUMIMO and ``_selective_recurrence``
  (models/selective_lru/selective_lru.py).
* ``oracle.linoss`` — LinOSS and ``_linoss_recurrence`` (models/linoss/linoss.py).

Gradients come from PyTorch autograd through these restatements. The restatements are
pinned against golden vectors produced by running the reference itself
(``tests/golden/make_golden.py``; checked by ``tests/test_oracle_golden.py``).
"""
