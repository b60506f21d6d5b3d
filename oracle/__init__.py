"""CPU oracle for the LongSpark drafting round -- TEST INFRASTRUCTURE ONLY.

This package restates, in numpy, the reference algorithm of every function on
the drafting hot path (view refresh, drafter pass, Markov argmax, accept
check).  It exists to check the CUDA path, never to stand in for it: only
``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s ``cpu_baseline`` /
``--impl reference`` legs may import it.  The product package
(``longspark_b200``) must never import anything from here.

Pinning: ``tests/golden/make_golden.py`` runs the unmodified reference
(``vendor/specforge`` + ``vendor/sglang`` of LongSpark, imported from a
read-only checkout) on seeded inputs and stores inputs and outputs as small
``.npz`` fixtures; ``tests/test_oracle_golden.py`` checks this restatement
against every fixture.
"""

from .drafter import *  # noqa: F401,F403
