"""Command-line drivers with the reference's flags, grids, exit codes and
CSV schemas, running the sm_100a kernels through the C ABI:

* ``python -m gb300_microbench_b200.cli.memory_paths {ldgsts,tma} ...``
  (the reference binaries ``memory_paths/ldgsts``, ``memory_paths/tma``);
* ``python -m gb300_microbench_b200.cli.umma {umma_1sm,umma_2sm} ...``
  (``umma_throughput/umma_1sm``, ``umma_2sm``);
* ``python -m gb300_microbench_b200.cli.sweeps {memory,umma} ...``
  (``memory_paths/benchmark.py``, ``umma_throughput/benchmark.py``);
* ``python -m gb300_microbench_b200.cli.gemm_comparison ...``
  (``gemm_comparison/gemm_comparison.py``).

stdout carries CSV only; diagnostics go to stderr. Exit codes: 0 success,
1 validation / CUDA / self-test failure, 2 usage error.
"""
