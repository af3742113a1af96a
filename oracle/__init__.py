"""TEST INFRASTRUCTURE ONLY: the CPU oracle (parity checker and timed CPU baseline).

Imported by ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py`` only.
"""
