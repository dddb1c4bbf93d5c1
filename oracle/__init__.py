"""CPU oracle for the packed-TCQ decode path.

TEST INFRASTRUCTURE, NOT PRODUCT CODE: a numpy restatement of the reference
(godsonj64/turbopress) arithmetic used only as the checker by ``tests/``,
``__graft_entry__.smoke()`` and the CPU-baseline legs of ``bench.py``.  The
``turbopress_b200`` package never imports it.
"""
