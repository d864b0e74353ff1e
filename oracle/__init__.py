"""CPU oracle for the Pairformer pair path (test infrastructure only).

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline leg
may import this package, and only as the checker. The product path in
``fireprot_b200`` never imports it.
"""
