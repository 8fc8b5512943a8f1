"""Streaming kernels on the GPU: bit-exact against the oracle's checksums
and the SplitMix64 pattern, for every configuration of both grids."""
import numpy as np
import pytest
import torch

import oracle
from gb300_microbench_b200 import streaming

pytestmark = pytest.mark.gpu

ALL_STAGES = (2, 3, 4, 8)


def _small_ws(sm_count: int, multiples: int = 8) -> int:
    # The reference's self-test working set: 8 x sm_count x 32 KiB
    # (ldgsts.cu:69, 467-471).
    return multiples * sm_count * 32 * 1024


@pytest.mark.parametrize("method", ["ldgsts", "tma"])
@pytest.mark.parametrize("stages", ALL_STAGES)
@pytest.mark.parametrize("bif", streaming.BIF_KIB)
def test_pattern_validate_and_checksums(cuda_device, method, stages, bif):
    sm = torch.cuda.get_device_properties(0).multi_processor_count
    nbytes = _small_ws(sm)
    buf = torch.empty(nbytes // 4, dtype=torch.int32, device=cuda_device)
    streaming.fill_pattern(buf)
    run = streaming.StreamingRun(method, stages, bif, buf, row_bytes=256)
    assert run.validate() == 0
    words = oracle.pattern_words(0, nbytes // 16)
    assert np.array_equal(buf.cpu().numpy().view(np.uint32), words)
    want = oracle.copy_checksums(words, run.info["stage_bytes"], run.info["grid_ctas"])
    assert np.array_equal(np.array(run.checksums(), dtype=np.uint32), want)
    for passes, rotation in ((3, 1), (2, 5)):
        run.run(passes=passes, rotation=rotation)
        want = oracle.copy_checksums(words, run.info["stage_bytes"], run.info["grid_ctas"], passes)
        assert np.array_equal(np.array(run.checksums(), dtype=np.uint32), want)
    run.check_status()


@pytest.mark.parametrize("method,row_bytes", [("ldgsts", 256), ("tma", 128)])
@pytest.mark.parametrize("stages", (2, 3, 4))
def test_uniform_buffer_ragged_size(cuda_device, method, row_bytes, stages):
    """Seeded uniform u32 buffer of a size that is no multiple of the tile
    or of the SM count: last tile short, unequal tile counts per CTA."""
    nbytes = 37 * 1024 * 1024 + 3 * 256
    buf = torch.empty(nbytes // 4, dtype=torch.int32, device=cuda_device)
    streaming.fill_uniform_u32(buf, seed=0)
    words = oracle.uniform_u32(nbytes // 4, seed=0)
    assert np.array_equal(buf.cpu().numpy().view(np.uint32), words)
    for bif in streaming.BIF_KIB:
        run = streaming.StreamingRun(method, stages, bif, buf, row_bytes=row_bytes)
        run.run()
        got = np.array(run.checksums(), dtype=np.uint32)
        want = oracle.copy_checksums(words, run.info["stage_bytes"], run.info["grid_ctas"])
        assert np.array_equal(got, want), (bif, run.info)
        assert int(np.bitwise_xor.reduce(got)) == oracle.xor_all(words)


def test_full_size_4gib_checksum_of_checksums(cuda_device):
    """Config 1 at full size: 4 GiB seeded uniform u32 read once; the XOR of
    the per-CTA checksums equals the XOR of the whole buffer, which the
    oracle computes from its own draw."""
    nbytes = 4 << 30
    buf = torch.empty(nbytes // 4, dtype=torch.int32, device=cuda_device)
    streaming.fill_uniform_u32(buf, seed=0)
    want = oracle.xor_all(oracle.uniform_u32(nbytes // 4, seed=0))
    for method, row_bytes in (("ldgsts", 256), ("tma", 128)):
        run = streaming.StreamingRun(method, 4, 64, buf, row_bytes=row_bytes)
        run.run()
        got = np.bitwise_xor.reduce(np.array(run.checksums(), dtype=np.uint32))
        assert int(got) == want, method
    del buf
    torch.cuda.empty_cache()


@pytest.mark.parametrize("method,row_bytes,nbytes", [("ldgsts", 256, 16), ("ldgsts", 256, 4096),
                                                     ("ldgsts", 256, 8192 + 16), ("tma", 256, 256),
                                                     ("tma", 128, 3 * 128), ("tma", 128, 8192 + 128)])
def test_tiny_buffers(cuda_device, method, row_bytes, nbytes):
    """Buffers of one short tile or barely more: most CTAs get no tile, the
    one or two that do stop at the buffer's end (checksums bit-exact)."""
    buf = torch.empty(nbytes // 4, dtype=torch.int32, device=cuda_device)
    streaming.fill_uniform_u32(buf, seed=3)
    words = oracle.uniform_u32(nbytes // 4, seed=3)
    for stages in (2, 4):
        run = streaming.StreamingRun(method, stages, 16, buf, row_bytes=row_bytes)
        run.run(passes=2)
        got = np.array(run.checksums(), dtype=np.uint32)
        want = oracle.copy_checksums(words, run.info["stage_bytes"], run.info["grid_ctas"], 2)
        assert np.array_equal(got, want), (stages, run.info)
        run.check_status()


@pytest.mark.parametrize("pipe", ["0", "1"])
@pytest.mark.parametrize("stages,bif", [(2, 64), (4, 32), (8, 16)])
def test_ldgsts_pipeline_forms_same_checksums(cuda_device, monkeypatch, pipe, stages, bif):
    """Both LDGSTS pipeline forms (classic: reduce a landed tile, then issue
    into the freed slot; refill: each position refilled right after it was
    read; BB_COPY_PIPE) read the same words over several passes with
    rotation, on a buffer whose last tile is short."""
    monkeypatch.setenv("BB_COPY_PIPE", pipe)
    nbytes = 9 * 1024 * 1024 + 512
    buf = torch.empty(nbytes // 4, dtype=torch.int32, device=cuda_device)
    streaming.fill_uniform_u32(buf, seed=3)
    words = oracle.uniform_u32(nbytes // 4, seed=3)
    run = streaming.StreamingRun("ldgsts", stages, bif, buf, row_bytes=256)
    for passes, rotation in ((1, 0), (3, 2)):
        run.run(passes=passes, rotation=rotation)
        want = oracle.copy_checksums(words, run.info["stage_bytes"], run.info["grid_ctas"], passes)
        assert np.array_equal(np.array(run.checksums(), dtype=np.uint32), want)
    run.check_status()
