"""Test-infrastructure oracle package (CPU restatement of the reference's hot path).

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline legs may import
this package.  The product (``neurocell_b200``) never does.
"""
