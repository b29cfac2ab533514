"""Test infrastructure: CPU restatements of the reference's numeric goldens.

Nothing in the ``aipu_b200`` library imports this package. Only ``tests/``,
``__graft_entry__.smoke()`` and the CPU legs of ``bench.py`` use it, and only as the checker
(or as the timed CPU baseline), never as the thing measured for the GPU path.
"""
