"""CPU oracle for com.microsoft.MatMulNBits.

TEST INFRASTRUCTURE ONLY. Nothing in the product path (``xrgpu_b200``) may
import, link or execute anything in this directory; only ``tests/``,
``__graft_entry__.smoke()`` and the CPU-baseline / reference legs of
``bench.py`` use it, and there only as the checker or the timed CPU baseline.
"""
