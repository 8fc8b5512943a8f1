"""UMMA probes on the GPU: exact known answers (reference mode) and
N(0,1) operands against the double-precision oracle (baseline mode)."""
import numpy as np
import pytest
import torch

import oracle
from gb300_microbench_b200 import inputs, umma

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("cta_group,handshake", ((1, False), (2, False), (2, True)))
@pytest.mark.parametrize("n", umma.N_VALUES)
@pytest.mark.parametrize("depth", umma.ALL_DEPTHS)
def test_pattern_exact(cuda_device, cta_group, handshake, n, depth):
    """Both 2-SM loop forms (with the reference's per-iteration CTA-pair
    handshake, and without) give the exact known answer."""
    a, b = inputs.umma_pattern_operands(cta_group, n)
    probe = umma.UmmaProbe(cta_group, n, depth, a.to(cuda_device), b.to(cuda_device), handshake=handshake)
    probe.launch(iterations=2, timed=True)
    d, cycles = probe.result()
    want = oracle.umma_reference_d(cta_group, n, depth)
    assert np.array_equal(d.numpy().astype(np.float64), want)
    assert cycles > 0


@pytest.mark.parametrize("cta_group", (1, 2))
@pytest.mark.parametrize("n", umma.N_VALUES)
@pytest.mark.parametrize("depth", umma.BASELINE_DEPTHS)
def test_random_operands(cuda_device, cta_group, n, depth):
    a, b = inputs.umma_random_operands(cta_group, n)
    probe = umma.UmmaProbe(cta_group, n, depth, a.to(cuda_device), b.to(cuda_device))
    probe.launch(iterations=3)
    d, _ = probe.result()
    want = oracle.umma_expected(a.view(torch.int16).numpy().view(np.uint16),
                                b.view(torch.int16).numpy().view(np.uint16), depth)
    err = np.linalg.norm(d.numpy() - want) / np.linalg.norm(want)
    assert err <= 1e-5, err


def test_wait_timeout_is_reported_not_hung(cuda_device):
    """Waits that nothing completes (single thread, warp-wide spinning,
    warp-wide with the suspend hint) give up after their budget and report
    through their status words; the context stays usable afterwards."""
    from gb300_microbench_b200 import _native as nat

    status = torch.zeros(3, dtype=torch.int32, device=cuda_device)
    nat.call("bb_test_wait_timeout", 2_000_000, status.data_ptr(), torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    assert status.tolist() == [0x106, 0x106, 0x106]
    x = torch.ones(4, device=cuda_device)
    assert float((x * 2).sum().item()) == 8.0
