"""CPU oracle for the frozen-linear hot path — TEST INFRASTRUCTURE ONLY.

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline leg
(including ``bench.py --impl reference``) may import this package.  The product
package ``spilltune_b200`` never imports it, never falls back to it, and fails
loudly when its CUDA library is missing.

Parity pin: ``codec_oracle.c`` is checked bit-for-bit against golden vectors
produced by importing the reference itself (``tests/golden/make_golden.py``)
and against the reference's own known-answer test
(``tests/test_quantization.py:73-81``: int4 payload bytes ``[0x61,0x88,0xfa]``).
"""
