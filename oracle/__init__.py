"""CPU oracle for the CROSS (jaxite_word) CKKS hot path.

TEST INFRASTRUCTURE ONLY.  Nothing in the ``cross_b200`` product imports,
links or executes this package.  It may be used by ``tests/``, by
``__graft_entry__.smoke()`` (to verify one small GPU invocation) and
by ``bench.py`` (the ``cpu_baseline`` leg and ``--impl reference``).

``cross_oracle`` is a numpy restatement of the reference's integer
algorithms; every function cites the file:line of
EfficientPPML/CROSS/jaxite_word it follows.  It is pinned against the
reference's own golden vectors (OpenFHE-produced, embedded in the reference
test files) that ``tests/golden/make_golden.py`` extracts into
``tests/golden/*.json``.
"""

from . import cross_oracle  # noqa: F401
