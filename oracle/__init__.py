"""CPU oracle for the packed refresh executor (test infrastructure only).

Nothing in the product package imports this directory. Only ``tests/``,
``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline / reference arm use
it, and only as the checker or as the timed CPU restatement of the reference.
"""
