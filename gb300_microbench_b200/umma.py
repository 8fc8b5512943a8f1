"""Python face of the tcgen05 UMMA throughput probes.

Replaces run_once / validate_d of the reference probes
(umma_throughput/umma_1sm.cu:1006-1083, umma_2sm.cu): launch one probe,
read back D and the cycle count, check D.
"""
from __future__ import annotations

import torch

from . import _native as nat

N_VALUES = (64, 128, 256)
REFERENCE_DEPTHS = (4, 16, 64, 256)
BASELINE_DEPTHS = (16, 32, 64, 128, 256)
ALL_DEPTHS = (4, 16, 32, 64, 128, 256)
K = 16


def m_of(cta_group: int) -> int:
    return 128 * cta_group


def kernel_name(cta_group: int, n: int, depth: int) -> str:
    name = nat.bench_lib().bb_umma_kernel_name(cta_group, n, depth)
    if not name:
        raise ValueError(f"no probe for cta_group={cta_group} n={n} depth={depth}")
    return name.decode()


def flops_per_umma(cta_group: int, n: int) -> int:
    """2*M*N*K (umma_1sm.cu:1153-1154)."""
    return 2 * m_of(cta_group) * n * K


class UmmaProbe:
    def __init__(self, cta_group: int, n: int, depth: int, a: torch.Tensor, b: torch.Tensor, stream=None,
                 handshake: bool = False):
        """handshake=True (CTA pairs only): the reference's per-iteration
        cluster handshake inside the timed loop (umma_2sm.cu:617-659)."""
        if a.shape != (m_of(cta_group), K) or b.shape != (n, K):
            raise ValueError(f"operands must be A {(m_of(cta_group), K)} and B {(n, K)}")
        if a.dtype != torch.bfloat16 or b.dtype != torch.bfloat16 or not a.is_cuda or not b.is_cuda:
            raise ValueError("operands must be CUDA bfloat16 tensors")
        if a.device != b.device:
            raise ValueError(f"A on {a.device}, B on {b.device}: both must be on one device")
        if handshake and cta_group != 2:
            raise ValueError("the handshake loop is a CTA-pair (cta_group 2) form")
        self.cta_group, self.n, self.depth = cta_group, n, depth
        self.handshake = bool(handshake)
        self.name = kernel_name(cta_group, n, depth)
        self.a, self.b = a.contiguous(), b.contiguous()
        dev = a.device
        self.d = torch.empty(m_of(cta_group), n, dtype=torch.float32, device=dev)
        self.cycles = torch.zeros(1, dtype=torch.int64, device=dev)
        self.launch_ok = torch.zeros(2, dtype=torch.int32, device=dev)
        self.status = torch.zeros(1, dtype=torch.int32, device=dev)
        self.stream = stream if stream is not None else torch.cuda.current_stream(dev)
        self._lib = nat.bench_lib()

    def launch(self, iterations: int, timed: bool = True) -> None:
        self.launch_ok.zero_()
        nat.check("bb_umma_run_ex", self._lib.bb_umma_run_ex(
            self.cta_group, self.n, self.depth, iterations, 1 if timed else 0, 1 if self.handshake else 0,
            self.a.data_ptr(), self.b.data_ptr(), self.d.data_ptr(), self.cycles.data_ptr(),
            self.launch_ok.data_ptr(), self.status.data_ptr(), self.stream.cuda_stream))

    def result(self) -> tuple[torch.Tensor, int]:
        """(D on the host, elapsed cycles); raises on a launch or wait failure."""
        self.stream.synchronize()
        ok = self.launch_ok.cpu().tolist()[: self.cta_group]
        st = int(self.status.item())
        if st != 0:
            raise nat.NativeCallError(self.name, nat.BB_ERR_TIMEOUT, f"device status 0x{st:x}")
        if ok != [1] * self.cta_group:
            raise nat.NativeCallError(self.name, nat.BB_ERR_INTERNAL, f"launch contract not confirmed: {ok}")
        return self.d.cpu(), int(self.cycles.item())
