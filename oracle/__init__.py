"""CPU oracle for the Gated DeltaNet token mixer (test infrastructure only).

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py`` (CPU baseline and
the ``--impl reference`` arm) import this package.  The product package
``visionstack_b200`` never does.
"""
