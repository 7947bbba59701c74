"""The bounded flag exchange of the p2p camera-sharded mode (s4d_peer_signal_wait) on one GPU.

Two cases that need no second GPU: the epoch the other rank would publish is already in this
GPU's slot (the launch publishes its own epoch in the other rank's slot array and returns at
once), and nothing ever publishes it (the wait gives up after its limit, sets
S4D_FLAG_PEER_TIMEOUT and returns; the context stays usable).  The "other rank's" slot array is
a second buffer on the same GPU.  The exchange between two GPUs is tested in test_gpu_multi.py."""
import ctypes

import pytest
import torch

from sparse4d_tt_b200 import _lib as L

pytestmark = pytest.mark.gpu


def _signal(own, other, rank, epoch, limit_ns, flag):
    arr = (ctypes.c_void_p * 8)()
    arr[1 - rank] = other.data_ptr()
    st = L.lib().s4d_peer_signal_wait(own.data_ptr(), ctypes.cast(arr, ctypes.c_void_p), rank, 2, epoch, limit_ns,
                                      flag.data_ptr(), torch.cuda.current_stream().cuda_stream)
    L.check("peer_signal_wait", st)


def test_signal_publishes_and_returns_when_the_epoch_is_there(cuda_device):
    own = torch.zeros(8, dtype=torch.int32, device="cuda:0")
    other = torch.zeros(8, dtype=torch.int32, device="cuda:0")
    flag = torch.zeros(1, dtype=torch.int32, device="cuda:0")
    own[1] = 5  # rank 1 has published epoch 5
    for epoch in (3, 5):  # an older or equal epoch needs no wait
        _signal(own, other, 0, epoch, 10_000_000_000, flag)
        torch.cuda.synchronize()
        assert other[0].item() == epoch and flag.item() == 0
    # epochs compare modulo 2^32: 0xFFFFFFFF is older than 5
    _signal(own, other, 0, 0xFFFFFFFF, 10_000_000_000, flag)
    torch.cuda.synchronize()
    assert flag.item() == 0 and other[0].item() == -1
    own[0] = 9  # rank 1's own call (slot 0 written by rank 0)
    _signal(own, other, 1, 9, 10_000_000_000, flag)
    torch.cuda.synchronize()
    assert other[1].item() == 9 and flag.item() == 0


def test_signal_wait_gives_up_and_the_context_stays_usable(cuda_device):
    own = torch.zeros(8, dtype=torch.int32, device="cuda:0")
    other = torch.zeros(8, dtype=torch.int32, device="cuda:0")
    flag = torch.zeros(1, dtype=torch.int32, device="cuda:0")
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record()
    _signal(own, other, 0, 1, 2_000_000, flag)  # nothing publishes epoch 1 in own[1]: 2 ms limit
    end.record()
    torch.cuda.synchronize()
    assert flag.item() & L.S4D_FLAG_PEER_TIMEOUT
    assert other[0].item() == 1  # its own epoch was still published
    assert 1.5 <= start.elapsed_time(end) < 1000.0
    x = torch.arange(1000, device="cuda:0", dtype=torch.float32)
    assert float(x.sum().item()) == 499500.0
