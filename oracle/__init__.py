"""CPU oracle of the corrected sparse attention operator - test infrastructure only.

Imported by ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU baseline and
reference legs; never by the ``recap_b200`` package.
"""
