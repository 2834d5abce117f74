"""Sequence-parallel decode on 2 GPUs (skipped with fewer), at config 5a's
length (one 131072-key sequence, 64/8 heads, hd 128): each rank attends
its KV chunk of one long sequence, the (m, l, o) partials are exchanged
(NVLink peer stores fused with the merge, or an NCCL all-gather) and merged;
every rank's output must match the CPU oracle, on every one of several
consecutive steps (the peer exchange alternates its two buffer banks)."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

from tests.util import assert_parity

pytestmark = pytest.mark.gpu


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, ret, transport):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    import datetime
    import torch.distributed as dist
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev,
                            timeout=datetime.timedelta(seconds=60))
    from aspida_b200 import shard
    nq, nkv, hd, L = 64, 8, 128, 131072
    g = torch.Generator().manual_seed(7)
    K = torch.randn(L, nkv * hd, generator=g).half()
    V = torch.randn(L, nkv * hd, generator=g).half()
    q = torch.randn(1, nq * hd, generator=g)
    lo, hi = shard.kv_chunks(L, world)[rank]
    op = shard.SeqParallelDecode([K[lo:hi].to(dev)], [V[lo:hi].to(dev)], hi - lo, nq, nkv, hd,
                                 transport=transport)
    outs = []
    qd = q.to(dev)
    for step in range(3):
        outs.append(op(qd).clone())
    torch.cuda.synchronize()
    import aspida_b200 as ab
    assert ab.device_status() == 0
    op.close()
    ret[rank] = [o.cpu().numpy() for o in outs]
    dist.destroy_process_group()


@pytest.mark.parametrize("transport", ["p2p", "nccl"])
def test_seq_parallel_decode(oracle, transport):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    world = 2
    ret = mp.Manager().dict()
    mp.start_processes(_worker, args=(world, _free_port(), ret, transport), nprocs=world,
                       join=True, start_method="spawn")
    nq, nkv, hd, L = 64, 8, 128, 131072
    g = torch.Generator().manual_seed(7)
    K = torch.randn(L, nkv * hd, generator=g).half().float().numpy()
    V = torch.randn(L, nkv * hd, generator=g).half().float().numpy()
    q = torch.randn(1, nq * hd, generator=g).numpy()
    ref = oracle.decode_batch(q, [K], [V], [L - 1], nq, nkv, hd)
    for r in range(world):
        for step, o in enumerate(ret[r]):
            assert_parity(o, ref, what=f"{transport} rank {r} step {step}")
