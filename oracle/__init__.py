"""CPU oracle for the LVSA block-sparse attention path.

TEST INFRASTRUCTURE ONLY.  Nothing in the shipped package imports this
directory; only ``tests/``, ``__graft_entry__.smoke()`` and the
``cpu_baseline`` / ``--impl reference`` legs of ``bench.py`` use it, and
always as the checker or the timed CPU baseline, never as the product path.
"""
