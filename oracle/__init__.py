"""CPU oracle for the OABF path: TEST INFRASTRUCTURE ONLY.

Only ``tests/``, ``__graft_entry__.smoke()`` and the CPU-baseline leg of
``bench.py`` may import this package, and only as the checker. The product
package ``flashbfp_b200`` never imports it.
"""
