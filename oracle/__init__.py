"""CPU oracle for the W4G64 QuantLinear forward.

Test infrastructure only: imported by ``tests/``, ``__graft_entry__.smoke()``
and the CPU-baseline legs of ``bench.py``. The CUDA product path never calls
into this package.
"""
