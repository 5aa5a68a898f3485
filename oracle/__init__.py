"""CPU oracle of the ShadowKV decode step -- test infrastructure only.

Used by tests/, by ``__graft_entry__.smoke()`` as the checker and by
``bench.py`` as the timed CPU baseline.  The ``shadowkv_b200`` product never
imports it.
"""
