"""Failure detection on one GPU, without a GPU fault: a bounded device wait
that runs out returns, records its bit in the device error word, and leaves the
context usable.

The peer all-gather (mllb_q8_1_quantize_allgather) waits for every rank's
arrival on its counters.  Here world = 2 with both "ranks'" buffers and
counters in this GPU's memory and only rank 0 launching, so the arrival of
rank 1 never comes: CTA 0 polls for ~1 s (the wait's time limit), records
kErrPeerWaitTimeout (bit 6) and returns.  Nothing here touches another GPU.
"""
import ctypes as C
import time

import pytest
import torch

from mojo_llm_lab_b200 import formats as F
from mojo_llm_lab_b200 import ops
from mojo_llm_lab_b200._lib import PeerGather, check, lib

PEER_WAIT_TIMEOUT = 1 << 6


def _gather(x, k, rank, world, buffers, flags, count):
    pg = PeerGather()
    pg.rank, pg.world = rank, world
    for r in range(world):
        pg.buffers[r] = buffers[r].data_ptr()
        pg.flags[r] = flags[r].data_ptr()
    pg.count = count.data_ptr()
    stream = torch.cuda.current_stream().cuda_stream
    check(lib().mllb_q8_1_quantize_allgather(x.data_ptr(), k, C.byref(pg), 0, stream), "allgather")


@pytest.mark.gpu
def test_peer_gather_gives_up_when_a_rank_never_arrives():
    torch.cuda.set_device(0)
    k = 2560
    slice_bytes = F.q8_1_bytes(k)
    x = torch.randn(k, device="cuda")
    ref = ops.quantize_q8_1(x)
    assert ops.device_error() == 0
    buffers = [torch.zeros(2 * slice_bytes, dtype=torch.uint8, device="cuda") for _ in range(2)]
    flags = [torch.zeros(2, dtype=torch.int32, device="cuda") for _ in range(2)]
    count = torch.zeros(1, dtype=torch.int32, device="cuda")
    torch.cuda.synchronize()

    t0 = time.perf_counter()
    _gather(x, k, 0, 2, buffers, flags, count)
    torch.cuda.synchronize()
    waited = time.perf_counter() - t0
    assert 0.5 < waited < 30.0, f"the wait returned after {waited:.3f} s"
    assert ops.device_error(clear=False) & PEER_WAIT_TIMEOUT
    assert ops.device_error(clear=True) & PEER_WAIT_TIMEOUT
    assert ops.device_error() == 0, "clearing the word did not clear it"

    # What rank 0 did before the wait stands: its slice in both buffers,
    # its arrival counted in both counter arrays, its own gather counted.
    for r in range(2):
        assert torch.equal(buffers[r][:slice_bytes], ref)
        assert not buffers[r][slice_bytes:].any()
    grid = flags[0][0].item()
    assert grid > 0 and flags[1][0].item() == grid
    assert flags[0][1].item() == 0 and count.item() == 1

    # The context is usable: a gather that completes (one rank) succeeds.
    buf = torch.zeros(slice_bytes, dtype=torch.uint8, device="cuda")
    flag = torch.zeros(1, dtype=torch.int32, device="cuda")
    cnt = torch.zeros(1, dtype=torch.int32, device="cuda")
    t0 = time.perf_counter()
    _gather(x, k, 0, 1, [buf], [flag], cnt)
    torch.cuda.synchronize()
    assert time.perf_counter() - t0 < 0.5
    assert ops.device_error() == 0
    assert torch.equal(buf, ref)
