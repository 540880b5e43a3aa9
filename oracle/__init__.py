"""CPU oracle for the elastic sparse attention hot path.

TEST INFRASTRUCTURE ONLY.  Nothing in the shipped package imports this
directory: only ``tests/``, ``__graft_entry__.smoke()`` and the CPU-baseline
leg of ``bench.py`` may use it, and only as the checker (or as the timed CPU
stand-in for the reference), never as the thing that is measured or shipped.

Contents
--------
pattern      numpy float32 restatement of the index/mask generator
             (reference ``elastic_sparse_attention.py:470-535``), plus the
             dense-mask expansion (``:537-572``).
pattern_c    ctypes binding of ``pattern_ref.c``, the same recipe in plain C,
             used where numpy would be too slow (L up to 2^20).
naive        chunked fp32 torch restatement of the "naive" forward
             (``:624-680``) and its autograd backward.
holes        receptive-field ("attention hole") restatement of
             ``check_attn_hole.py:53-180``.

Parity pins (see ``tests/test_oracle_pins.py``): the restatements are checked
against fixtures produced by importing the reference module itself
(``tests/golden/make_golden.py``) and against the known answers of the
reference's own validation script.
"""
