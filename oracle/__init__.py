"""CPU oracle for the quantized-linear hot path — TEST INFRASTRUCTURE ONLY.

This package restates, in numpy, the reference's own CPU algorithms for the three paths the
B200 library replaces (each function cites the reference file:line it follows):

  * gptq.py — webtorch/_core.py:4046-4072 (`_gptq_matmul_np`), the exact unpack
    (`_core.py:4060-4069`, `quantize.py:32-43`), the quantiser/packers
    (`_core.py:3782-3824`, `quantize.py:80-106`), and desc_act (`g_idx`) as the same
    formula with g = g_idx[k] (the reference has no desc_act path).
  * q4k.py — webtorch/ggufload.py:116-131,190-202 (GGUF Q4_K super-block decode).
  * moe.py — webtorch/lm_engine.py:294-333 (`moe_mlp`, `_softmax_rows`).

Parity is pinned: tests/test_oracle_golden.py checks every function here against golden
vectors produced by the reference itself (tests/golden/make_golden.py imports the reference
package and runs its CPU path).

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline / reference arm may import
this package, and only as a checker or as the timed CPU baseline. The product
(webpytorch_b200) never imports it.
"""
