"""CPU oracle for the DSALT sparse-attention hot path.

Test infrastructure only: imported by ``tests/``, by ``__graft_entry__.smoke()``
and by the CPU-baseline leg of ``bench.py`` as the checker.  The shipped package
(``dsalt-library_b200/dsalt``) never imports it and has no CPU fallback.
"""
