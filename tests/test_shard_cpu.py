"""Host-side multi-rank logic on CPU with gloo (world size 2): planning, the
(m, l, o) exchange + merge of sequence-parallel decode (partials from the
CPU oracle's definitions, merge by the oracle), and failure of the exchange
when a peer leaves."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from aspida_b200 import shard


def test_plan_sequences_balances_and_covers():
    lens = [8192, 512, 700, 4000, 4100, 3000, 6000, 1000]
    plan = shard.plan_sequences(lens, 3)
    assert sorted(i for r in plan for i in r) == list(range(len(lens)))
    loads = [sum(lens[i] for i in r) for r in plan]
    assert max(loads) - min(loads) <= max(lens)
    assert shard.plan_sequences([5, 5], 4)[2:] == [[], []]


def test_kv_chunks_cover_aligned():
    for L, W in [(131072, 8), (100, 3), (17, 4), (0, 2)]:
        ch = shard.kv_chunks(L, W)
        assert ch[0][0] == 0 and ch[-1][1] == L
        for (a, b), (c, d) in zip(ch, ch[1:]):
            assert b == c and a <= b
        assert all(lo % 16 == 0 for lo, _ in ch)


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _partial_np(q, K, V, nq, nkv, hd, scale):
    """Split-KV partial (m, l, o) of one chunk, natural-log units."""
    rep = nq // nkv
    m = np.empty(nq, np.float32)
    l = np.empty(nq, np.float32)
    o = np.empty((nq, hd), np.float32)
    for h in range(nq):
        kv = h // rep
        s = (K[:, kv * hd:(kv + 1) * hd] @ q[h * hd:(h + 1) * hd]) * scale
        if s.size == 0:
            m[h], l[h], o[h] = -3.402823466e38, 0.0, 0.0
            continue
        m[h] = s.max()
        p = np.exp(s - m[h])
        l[h] = p.sum()
        o[h] = p @ V[:, kv * hd:(kv + 1) * hd]
    return m, l, o


def _worker(rank, world, port, q, K, V, nq, nkv, hd, ret, leave_early):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    import datetime
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=10))
    try:
        if leave_early and rank == 1:
            return                     # a rank that never joins the exchange
        lo, hi = shard.kv_chunks(K.shape[0], world)[rank]
        m, l, o = _partial_np(q, K[lo:hi], V[lo:hi], nq, nkv, hd, 1 / np.sqrt(hd))
        try:
            M, L, O = shard.exchange_partials(torch.from_numpy(m)[None], torch.from_numpy(l)[None],
                                              torch.from_numpy(o)[None])
        except shard.ShardError:
            ret[rank] = "shard_error"
            return
        import oracle
        ret[rank] = oracle.merge(M.numpy(), L.numpy(), O.numpy())
    finally:
        if not (leave_early and rank == 1):
            dist.destroy_process_group()


def _run(world, leave_early=False):
    rng = np.random.RandomState(3)
    nq, nkv, hd, L = 8, 2, 64, 500
    q = rng.standard_normal(nq * hd).astype(np.float32)
    K = rng.standard_normal((L, nkv * hd)).astype(np.float32)
    V = rng.standard_normal((L, nkv * hd)).astype(np.float32)
    ret = mp.Manager().dict()
    port = _free_port()
    mp.start_processes(_worker, args=(world, port, q, K, V, nq, nkv, hd, ret, leave_early),
                       nprocs=world, join=True, start_method="spawn")
    return q, K, V, nq, nkv, hd, L, dict(ret)


def test_seq_parallel_exchange_and_merge_gloo(oracle):
    q, K, V, nq, nkv, hd, L, ret = _run(2)
    ref = oracle.decode_batch(q[None], [K], [V], [L - 1], nq, nkv, hd)[0]
    for r in range(2):
        np.testing.assert_allclose(ret[r].reshape(-1), ref, atol=2e-6, rtol=1e-5)


def test_exchange_fails_cleanly_when_a_rank_leaves():
    *_, ret = _run(2, leave_early=True)
    assert ret.get(0) == "shard_error"
