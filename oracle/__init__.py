"""TEST INFRASTRUCTURE ONLY -- the CPU oracle for the soinfer decode hot path.

This package restates, on the CPU, the reference algorithms of
sparse-offload-infer for every op on the path (numpy for the vectorisable
parts, plain C in oracle/csrc for the serial selector scan and a fused
dequant GEMV).  It is the checker the parity tests compare the sm_100a
kernels against, and the CPU baseline bench.py times; it is never part of
the product path (soinfer/ has no import of it and no CPU fallback).

Pinning: the quantize/pack restatement is checked against fixtures produced
by importing the reference's own python/soinfer/quant (tests/golden/
make_golden.py); the selector, GEMV, sparse-accumulate and attention
restatements are checked against outputs of the reference's own CUDA kernels
compiled from its sources (oracle/Makefile -> oracle/_ref) and run on a B200
(tests/golden/make_golden_gpu.py).
"""
