"""CPU oracle for the NKIPy -> B200 execution path.

TEST INFRASTRUCTURE ONLY.  Nothing in ``nkipy_b200`` imports this package; only
``tests/``, ``__graft_entry__.smoke()`` and the CPU-baseline leg of
``bench.py`` use it, and only as the checker / the timed CPU reference.

The reference's own CPU path for every kernel is the NumPy direct call of the
kernel body (README.md:118-133 of shaojiex-aws/nkipy).  ``numpy_ref`` restates
that computation per benchmark configuration, citing the reference lines it
follows.  The restatements are pinned against fixtures produced by running the
reference's own functions (``tests/golden/make_golden.py``).
"""
