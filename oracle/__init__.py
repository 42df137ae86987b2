"""Oracle package — TEST INFRASTRUCTURE ONLY (checks the product, never part of it).

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline /
reference leg may import it.
"""
