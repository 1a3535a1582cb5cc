"""CPU oracle for the tensorgrad training step (test infrastructure only).

This package is the checker, never the product: only ``tests/``, ``__graft_entry__.smoke()``
and the ``cpu_baseline`` / ``--impl reference`` legs of ``bench.py`` import it. It restates,
in float64 NumPy, the algorithm of the reference tensorgrad 0.2.0 training step (forward,
``loss.backward()``, ``clip_grad_norm_`` and ``AdamW.step()``); each function cites the
reference file:line (paths inside the tensorgrad project) that it follows.

Parity is pinned: ``tests/golden/make_golden.py`` imports the reference itself, runs it in
float64 on seeded inputs and commits its outputs as fixtures under ``tests/golden/``;
``tests/test_oracle_golden.py`` checks this restatement against those fixtures and against
the known-answer values of the reference's own tests.
"""

from oracle import gpt, ops  # noqa: F401
