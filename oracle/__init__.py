"""CPU oracle of the packed draft-KV path -- TEST INFRASTRUCTURE ONLY.

A numpy restatement of the reference algorithm (kv_reduce/packed_kv_cache.py
and the attention semantics of kv_reduce/triton_packed_kv_attention.py),
used as the checker for the CUDA kernels.  Only tests/, the graft entry's
smoke() and bench.py's CPU-baseline leg may import it; the product package
kv_reduce_b200 never does.

Pinning: tests/test_oracle_golden.py checks this oracle bit-exactly against
golden vectors that tests/golden/make_golden.py produced by running the
reference's own packed_kv_cache.py (and its fp32 unpack + torch SDPA).
"""
