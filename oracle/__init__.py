"""CPU oracle for qi_b200 (TEST INFRASTRUCTURE ONLY).

Imported only by ``tests/``, ``__graft_entry__.smoke()`` and the CPU-baseline
leg of ``bench.py``; the product path (``qi_b200``) never imports it.
"""
