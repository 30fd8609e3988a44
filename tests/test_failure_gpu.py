"""Failure detection on the device without a GPU fault: a cross-GPU wait whose peer never
signals gives up after its bounded spin (about a second of %globaltimer), records an
error code in the status word that the host reads, and leaves the context usable.  Both
"ranks" are buffers on one GPU: the peer's flag is simply never written, and no second
kernel waits on this one."""

import time

import pytest
import torch

pytestmark = pytest.mark.gpu


def test_peer_wait_gives_up_and_reports():
    from myk_llm_b200.ops import ext

    mine = torch.zeros(8, dtype=torch.int32, device="cuda")
    silent_peer = torch.zeros(8, dtype=torch.int32, device="cuda")
    ptrs = torch.tensor([mine.data_ptr(), silent_peer.data_ptr()], dtype=torch.int64, device="cuda")
    ext().take_status()
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    ext().peer_barrier(ptrs, 0, 2, 1)  # rank 0 of 2; rank 1 never arrives
    torch.cuda.synchronize()
    waited = time.perf_counter() - t0
    assert ext().take_status() != 0
    assert 0.5 < waited < 30
    assert int(silent_peer[0]) == 1  # this rank's arrival was still delivered to the peer
    # the context is intact, and a barrier whose peer has arrived passes at once
    assert float(torch.ones(16, device="cuda").sum()) == 16.0
    mine[1] = 2  # rank 1 arrived at epoch 2
    t0 = time.perf_counter()
    ext().peer_barrier(ptrs, 0, 2, 2)
    torch.cuda.synchronize()
    assert ext().take_status() == 0
    assert time.perf_counter() - t0 < 0.5
