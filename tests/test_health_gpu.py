"""Bounded device-side waits: a peer barrier whose peer never arrives (a flag that nothing sets)
gives up after its ~1 s budget, records an error code that the host reads, and leaves the
context usable. One GPU; the "peer" is a local buffer that nobody writes."""
import pytest
import torch

pytestmark = pytest.mark.gpu


def test_peer_barrier_times_out_with_error_status():
    from appcorr_b200.ops.native import check_errors, err_word, lib

    dev = torch.device("cuda", 0)
    mine = torch.zeros(16, dtype=torch.int32, device=dev)   # 8 rank slots + the epoch counter
    ghost = torch.zeros(16, dtype=torch.int32, device=dev)  # the absent rank's flags
    err = err_word(dev)
    lib().tp_barrier([mine.data_ptr(), ghost.data_ptr()], 0, err)
    torch.cuda.synchronize()
    with pytest.raises(RuntimeError, match="peer"):
        check_errors(dev)
    # this rank's arrival was still published to both flag arrays
    assert int(ghost[0].item()) == 1 and int(mine[0].item()) == 1
    assert int(mine[8].item()) == 1  # the device-side epoch advanced
    # the context still works
    x = torch.ones(1024, device=dev)
    assert float((x * 2).sum().item()) == 2048.0
    check_errors(dev)
