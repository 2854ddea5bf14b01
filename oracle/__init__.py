"""TEST INFRASTRUCTURE ONLY -- the CPU oracle for the quantized decode path.

This package restates, on the CPU, the reference's algorithm for the four ops (COMP's `quant_q8_0`, `quant_q8_K`,
`q4_0_gemv`, `tq2_0_gemv`) and KURN's exact reference dot, plus the GEMVs of the two weight formats the product
adds beyond the reference (ggml Q8_0 and IQ4_NL, against q8_0 activations). It is the checker, never the product:
only `tests/`, `__graft_entry__.smoke()` and `bench.py`'s CPU-baseline / reference arm may import or run it. The
product (`comp_b200`) never imports it and has no CPU path.

  oracle.ref     numpy restatement (bit-exact quantizer bytes, exact int64 block dots, f64 reference dot in
                 KURN's order); also the seeded input generators.
  oracle.native  ctypes binding of oracle/c/oracle.c, the same math in C with OpenMP (timed CPU baseline and
                 full-size checks). Built by `python -m oracle.build` into oracle/_build/.

Parity is pinned: tests/test_oracle_golden.py checks both restatements against golden vectors produced by the
reference itself (COMP's kernels run under TRITON_INTERPRET=1, tests/golden/make_golden.py) and against gguf-py's
Q8_0 quantizer and Q4_0/TQ2_0/Q8_0/IQ4_NL dequantizers (the two extensions have no reference golden vectors, so
gguf-py's codecs pin them).
"""
