"""The bounded flag exchange of the p2p camera-sharded mode (s4d_peer_signal_wait and its
device-epoch form s4d_peer_signal_wait_counter) on one GPU.

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


def _signal_counter(own, other, rank, counter, advance, limit_ns, flag):
    arr = (ctypes.c_void_p * 8)()
    arr[1 - rank] = other.data_ptr()
    st = L.lib().s4d_peer_signal_wait_counter(own.data_ptr(), ctypes.cast(arr, ctypes.c_void_p), rank, 2,
                                              counter.data_ptr(), advance, limit_ns, flag.data_ptr(),
                                              torch.cuda.current_stream().cuda_stream)
    L.check("peer_signal_wait_counter", st)


def test_device_epoch_advances_per_launch_and_per_graph_replay(cuda_device):
    """The epoch is read from the device counter when the launch runs: eager launches and the
    replays of a graph that captured one launch each move it on by one."""
    own = torch.zeros(8, dtype=torch.int32, device="cuda:0")
    other = torch.zeros(8, dtype=torch.int32, device="cuda:0")
    counter = torch.zeros(1, dtype=torch.int32, device="cuda:0")
    flag = torch.zeros(1, dtype=torch.int32, device="cuda:0")
    own[1] = 1000  # the other rank is far ahead: no wait
    for e in (1, 2):
        _signal_counter(own, other, 0, counter, 1, 10_000_000_000, flag)
        torch.cuda.synchronize()
        assert counter.item() == e and other[0].item() == e and flag.item() == 0
    _signal_counter(own, other, 0, counter, 0, 10_000_000_000, flag)  # advance 0: publish the current epoch
    torch.cuda.synchronize()
    assert counter.item() == 2 and other[0].item() == 2
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=s):
        _signal_counter(own, other, 0, counter, 1, 10_000_000_000, flag)
    torch.cuda.synchronize()
    assert counter.item() == 2  # capturing runs nothing
    for e in (3, 4, 5):
        g.replay()
        torch.cuda.synchronize()
        assert counter.item() == e and other[0].item() == e and flag.item() == 0
    del g


def test_device_epoch_wait_gives_up(cuda_device):
    own = torch.zeros(8, dtype=torch.int32, device="cuda:0")
    other = torch.zeros(8, dtype=torch.int32, device="cuda:0")
    counter = torch.full((1,), 7, dtype=torch.int32, device="cuda:0")
    flag = torch.zeros(1, dtype=torch.int32, device="cuda:0")
    own[1] = 7  # the other rank has published epoch 7, never 8
    _signal_counter(own, other, 0, counter, 1, 2_000_000, flag)
    torch.cuda.synchronize()
    assert flag.item() & L.S4D_FLAG_PEER_TIMEOUT
    assert counter.item() == 8 and other[0].item() == 8
