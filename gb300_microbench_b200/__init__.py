"""B200-native (sm_100a) rebuild of the gb300-microbench hot path.

* :mod:`.gemm`      persistent warp-specialised BF16 GEMM (tcgen05 + TMA)
* :mod:`.streaming` HBM->SMEM streaming kernels (LDGSTS and 2D TMA)
* :mod:`.umma`      tcgen05 UMMA issue-throughput probes
* :mod:`.inputs`    seeded input generators of both input modes

All kernels live in ``lib/libb200bench.so`` behind the C ABI of
``include/b200bench.h``; :mod:`._native` is the ctypes shim. PyTorch is used
for device allocation and streams only.
"""
__all__ = ["gemm", "streaming", "umma", "inputs"]
__version__ = "0.1.0"
