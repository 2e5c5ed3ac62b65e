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
``tests/golden/*.json``, and, at sizes those vectors do not reach (up to
HE-Mult and HE-Rotate at N = 2^16, L = 24), against digests of the
reference's own outputs on seeded inputs (``tests/golden/shim_digests.json``,
recorded by ``tests/golden/make_golden_shim.py`` with the reference's code
run on a numpy stand-in for jax).
"""

from . import cross_oracle  # noqa: F401
