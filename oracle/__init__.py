"""CPU oracle for the skinny-GEMM path - TEST INFRASTRUCTURE ONLY.

This package restates, on the CPU, the algorithms the reference (0c33/mi50-vllm-lab) uses to
check and to time its kernels:

* ``skinny_oracle``: Exllama/GPTQ nibble packing, the float64 dequantize-then-matmul reference of
  kernels/check_w4.py:11-21, the fp16 GEMM reference of kernels/bench_skinny.py:44, the fixed
  rank-order all-reduce of kernels/hostar.cu:107, seeded input generators for the configurations
  of the benchmark, and the tolerance check.
* ``cpu_baseline``: the reference's torch dequantize-then-matmul on the host cores, timed.

Only ``tests/``, ``__graft_entry__.smoke()`` and the ``cpu_baseline`` / ``--impl reference`` legs of
``bench.py`` may import it, and only to check or to time the reference's CPU path. The product
(the CUDA kernels behind ``gfx906_skinny`` and ``libb2skinny.so``) never calls into it.

Parity is pinned: ``tests/golden/`` holds outputs produced by executing the reference's own
reference lines (kernels/check_w4.py:11-18,21 and kernels/bench_skinny.py:44) on seeded inputs,
and ``tests/test_oracle.py`` checks this oracle against them.
"""
