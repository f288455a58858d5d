"""CPU oracle for the okc_b200 decode path — TEST INFRASTRUCTURE ONLY.

A restatement, in plain PyTorch fp32 on the CPU and numpy for the bit-exact integer and
ordering work, of the reference's own PyTorch reference path for the three decode
operators (tommyyliu/okc: muse_prefill_layer/submission.py, muse_attention_decode/
tools/bench_tail.py, muse_decode_layer/decode/nvfp4_gemv.py, muse_moe_w4a16/
submission.py).  Every function cites the reference file:line it follows.

Only tests/, __graft_entry__.smoke() and bench.py's cpu_baseline / --impl reference legs
may import this package, and only as the checker or the timed CPU baseline: the product
path (okc_b200) never calls it and has no CPU fallback.

Parity pins: tests/golden/ holds fixtures produced by running the reference's own code in
this container (tests/golden/make_golden.py): the NVFP4 nibble decoder of
muse_decode_layer/decode/nvfp4_gemv.py:9-18, the `_route` permutation kernel of
muse_moe_w4a16/submission.py:274-291 (under Triton's CPU interpreter), and the
`rms`/`rope`/`attention`/`route` functions of muse_prefill_layer/submission.py.
"""
