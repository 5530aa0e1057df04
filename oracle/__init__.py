"""CPU oracle of the B200 decode path: a restatement of the reference's NumPy specification
(harness/numpy_ref.py) and of the operator order its graph runs (fleet/graph_plan.py), with the
summation order and exp/log made deterministic (oracle/detmath.py).

TEST INFRASTRUCTURE. This package is the checker, never the product: only ``tests/``,
``__graft_entry__.smoke()`` and ``bench.py`` (its ``cpu_baseline`` leg and ``--impl reference``)
may import it. The product path (``fleet-amd-task_b200/``) never imports it and fails loudly
when its CUDA library is missing.

Pinned by: the reference's own NumPy functions run on the same inputs and the reference's HF
modules (tiny random model) run here, both captured as fixtures in tests/golden/ by
tests/golden/make_golden.py (tests/test_oracle_pins.py).
"""
