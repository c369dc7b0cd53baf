"""CPU oracle for the MoE expert path: test infrastructure, never the product.

Only ``tests/``, ``__graft_entry__.smoke()`` and the ``cpu_baseline`` /
``--impl reference`` legs of ``bench.py`` may import this package.
"""
