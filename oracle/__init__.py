"""Oracle package — TEST INFRASTRUCTURE ONLY (the checker, never the product).

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline /
reference leg may import it.
"""
