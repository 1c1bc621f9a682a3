"""CPU oracle for the exactkv hot path — TEST INFRASTRUCTURE ONLY.

Numpy restatements of the reference algorithms, used as the checker by
tests/, by __graft_entry__.smoke() and by bench.py's CPU-baseline and
reference arms. Nothing in the exactkv_b200 package imports this package, and
the product never runs it.

Pinning: the codec restatement is checked byte for byte against golden
vectors produced by the reference's own exactkv/codec.py (encode_reference,
decode_reference) and its Triton page encoder run under TRITON_INTERPRET=1
(tests/golden/make_golden.py); the attention restatement is checked against
the reference test's float64 einsum (tests/test_exactkv.py:75-77) stored in
the same fixtures. The reference has no CPU attention kernel, so the fp32
attention restatement itself is pinned only through that float64 bound.
"""
