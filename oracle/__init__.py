"""CPU oracle of the packed binary low-rank linear -- test infrastructure only.

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline
legs may import this package; the product path never does.
"""
