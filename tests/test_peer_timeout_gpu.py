"""The peer exchange's bounded wait running out, on one GPU.

aspida_attn_exchange_merge waits for every rank's step-tagged flag in its
own receive buffer. Here rank 1 is absent: its slot is a second, local,
zero-filled buffer in which no flag is ever raised, so rank 0's wait must run
out (after a short, test-set number of polls), the kernel must return, and
the failure must be visible through the device status word, through the
caller's host-mapped failure word, and (PeerExchange) as a ShardError that
also refuses every later step. Nothing faults or hangs: the only failure is
a flag that nobody sets.
"""
import ctypes as C
import os
import socket

import pytest
import torch

pytestmark = pytest.mark.gpu


def _alloc_peer_buffer(lib, nbytes):
    ptr = C.c_void_p()
    handle = (C.c_char * 64)()
    assert lib.aspida_attn_peer_alloc(nbytes, C.byref(ptr), handle) == 0
    return ptr.value


def test_exchange_wait_runs_out():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    import aspida_b200 as ab
    from aspida_b200 import _lib

    lib = _lib.load()
    assert ab.device_status() == 0
    rows, hd, world = 64, 128, 2
    nbytes = lib.aspida_attn_peer_buffer_size(world, rows, hd)
    own = _alloc_peer_buffer(lib, nbytes)
    absent = _alloc_peer_buffer(lib, nbytes)       # stands in for rank 1: no flag ever arrives
    try:
        part = torch.randn(rows * (hd + 2), device="cuda")
        part[:rows] = 0.0                           # m
        part[rows:2 * rows] = 1.0                   # l
        out = torch.full((rows, hd), 7.0, device="cuda")
        fail = torch.zeros(1, dtype=torch.int32).pin_memory()
        table = (C.c_void_p * world)(own, absent)
        rc = lib.aspida_attn_exchange_merge_ex(
            part.data_ptr(), table, world, 0, 1, None, out.data_ptr(), rows, hd,
            fail.data_ptr(), 2000, torch.cuda.current_stream().cuda_stream)
        assert rc == 0
        torch.cuda.synchronize()                    # the call returned: the wait gave up
        assert int(fail[0]) != 0
        assert lib.aspida_attn_device_status_where() == 60
        assert ab.device_status() == ab.ASPIDA_ERR_DEVICE
        assert ab.device_status() == 0              # read-and-clear
        ab.last_error()
        # no output was merged from a missing partial
        assert torch.all(out == 7.0)
        # a rank that is present completes with the default limit: give the
        # stand-in buffer rank 1's flag for step 2 by running rank 1's send
        # first, then rank 0's step (sequential launches, no mutual wait)
        fail.zero_()
        table1 = (C.c_void_p * world)(own, absent)
        # "rank 1" sends into slot 1 of own; its own wait (on `absent`) runs out fast
        rc = lib.aspida_attn_exchange_merge_ex(
            part.data_ptr(), table1, world, 1, 2, None, out.data_ptr(), rows, hd,
            None, 2000, torch.cuda.current_stream().cuda_stream)
        assert rc == 0
        torch.cuda.synchronize()
        assert ab.device_status() == ab.ASPIDA_ERR_DEVICE
        ab.last_error()
        rc = lib.aspida_attn_exchange_merge_ex(
            part.data_ptr(), table, world, 0, 2, None, out.data_ptr(), rows, hd,
            fail.data_ptr(), 0, torch.cuda.current_stream().cuda_stream)
        assert rc == 0
        torch.cuda.synchronize()
        assert int(fail[0]) == 0
        assert ab.device_status() == 0
        # both slots hold the same partial with m = 0, l = 1: the merge is o
        ref = part[2 * rows:].reshape(rows, hd)
        torch.testing.assert_close(out, ref, rtol=1e-6, atol=1e-6)
    finally:
        torch.cuda.synchronize()
        lib.aspida_attn_peer_free(own)
        lib.aspida_attn_peer_free(absent)


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def test_peer_exchange_object_raises_and_stays_failed():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    import torch.distributed as dist
    import aspida_b200 as ab
    from aspida_b200 import _lib, shard

    lib = _lib.load()
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(_free_port()))
    own_group = not dist.is_initialized()
    if own_group:
        dist.init_process_group("nccl", rank=0, world_size=1,
                                device_id=torch.device("cuda", torch.cuda.current_device()))
    rows, hd = 32, 128
    absent = None
    px = shard.PeerExchange(rows, hd, wait_limit=2000)
    try:
        # turn the 1-rank exchange into a 2-rank one whose second rank never arrives
        # (both buffers sized for the 2-rank layout)
        absent = _alloc_peer_buffer(lib, lib.aspida_attn_peer_buffer_size(2, rows, hd))
        px.world = 2
        own2 = _alloc_peer_buffer(lib, lib.aspida_attn_peer_buffer_size(2, rows, hd))
        lib.aspida_attn_peer_free(px._own)
        px._own = own2
        px.table = (C.c_void_p * 2)(own2, absent)
        part = torch.zeros(rows * (hd + 2), device="cuda")
        out = torch.empty(rows, hd, device="cuda")
        px(part, out)
        with pytest.raises(shard.ShardError):
            px.check()
        with pytest.raises(shard.ShardError):
            px(part, out)                            # refuses further steps
        assert ab.device_status() == ab.ASPIDA_ERR_DEVICE
        ab.last_error()
    finally:
        torch.cuda.synchronize()
        px._mapped = []
        px.close(barrier=False)
        if absent is not None:
            lib.aspida_attn_peer_free(absent)
        if own_group:
            dist.destroy_process_group()
