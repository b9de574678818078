"""CPU oracle for the FADE tiered-KV hot path -- TEST INFRASTRUCTURE ONLY.

A numpy restatement of the reference's arithmetic (fade-kv 1.1.0), used by
``tests/``, ``__graft_entry__.smoke()`` and the ``cpu_baseline`` / reference
arm of ``bench.py`` as the checker and the timed CPU baseline.  Nothing in the
``fade_b200`` package imports it; the product path has no CPU fallback.

Pinned against golden vectors produced by the reference itself
(``tests/golden/make_golden.py`` imports the reference and writes
``tests/golden/*.npz``; ``tests/test_oracle_golden.py`` checks this module
against them bit-for-bit for the integer/byte outputs).
"""

from oracle.numerics import bf16_round, f16_round, rnd  # noqa: F401
