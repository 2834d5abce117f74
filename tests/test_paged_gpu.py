"""GPU tests of the paged KV path (block tables over shared pools, the KV_Pool
layout of src/llm/kv_pool.ads): appending through block tables, prefill and
decode reading through them. Paged results must equal the contiguous-cache
results on the same rows (bit-exact: same kernels, same tiles) and the
oracle."""
import numpy as np
import pytest
import torch

from tests.util import assert_parity

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def ab():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    import aspida_b200
    return aspida_b200


def scattered_tables(nseq, nblk, total, seed):
    """Per-sequence block ids drawn without replacement from a shuffled pool."""
    perm = np.random.RandomState(seed).permutation(total)
    table = np.zeros((nseq, max(nblk)), np.int32)
    k = 0
    for b, n in enumerate(nblk):
        table[b, :n] = perm[k:k + n]
        k += n
    return table


def gather_rows(pool, table_row, bs, L):
    rows = np.concatenate([np.arange(t * bs, t * bs + bs) for t in table_row])[:L]
    return pool[torch.from_numpy(rows).long().to(pool.device)]


def test_prep_paged_matches_contiguous(ab):
    """One sequence, P tokens crossing block boundaries, at pos_start > 0."""
    nq, nkv, hd, bs, P, ps = 8, 2, 128, 16, 40, 29
    g = torch.Generator(device="cuda").manual_seed(3)
    q = torch.randn(P, nq * hd, generator=g, device="cuda")
    k = torch.randn(P, nkv * hd, generator=g, device="cuda")
    v = torch.randn(P, nkv * hd, generator=g, device="cuda")
    rope = ab.RopeParams(dim=hd, freq_base=500000.0)
    cache = ab.KVCache(ps + P, nkv, hd, nq)
    q_ref = ab.prep(q, k, v, cache.K, cache.V, ps, nq, nkv, hd, rope)
    nb = (ps + P + bs - 1) // bs
    total = nb + 5
    table = scattered_tables(1, [nb], total, 4)[0]
    Kp = torch.zeros(total * bs, nkv * hd, dtype=torch.half, device="cuda")
    Vp = torch.zeros_like(Kp)
    q_got = ab.prep_paged(q, k, v, Kp, Vp, torch.from_numpy(table).cuda(), bs, nq, nkv, hd, rope,
                          pos_start=ps)
    torch.cuda.synchronize()
    assert torch.equal(q_got, q_ref)
    Kg = gather_rows(Kp, table, bs, ps + P)
    Vg = gather_rows(Vp, table, bs, ps + P)
    assert torch.equal(Kg[ps:], cache.K[ps:ps + P])
    assert torch.equal(Vg[ps:], cache.V[ps:ps + P])
    assert int(Kg[:ps].float().abs().sum()) == 0          # rows before pos_start untouched
    cache.free()


def test_prep_paged_lanes_then_decode_paged(ab, oracle):
    """Decode batch: lane b appends at pos[b] through table row b, then the
    paged decode over the same pools equals the oracle on the gathered rows."""
    nq, nkv, hd, bs = 32, 8, 128, 32
    lens = [1, 31, 32, 33, 500, 1201]
    nblk = [(L + bs - 1) // bs for L in lens]
    total = sum(nblk) + 4
    table = scattered_tables(len(lens), nblk, total, 9)
    g = torch.Generator(device="cuda").manual_seed(9)
    Kp = torch.randn(total * bs, nkv * hd, generator=g, device="cuda").half()
    Vp = torch.randn(total * bs, nkv * hd, generator=g, device="cuda").half()
    B = len(lens)
    q = torch.randn(B, nq * hd, generator=g, device="cuda")
    k = torch.randn(B, nkv * hd, generator=g, device="cuda")
    v = torch.randn(B, nkv * hd, generator=g, device="cuda")
    pos = torch.tensor([L - 1 for L in lens], dtype=torch.int32, device="cuda")
    tab = torch.from_numpy(table).cuda()
    rope = ab.RopeParams(dim=hd, freq_base=500000.0)
    qr = ab.prep_paged(q, k, v, Kp, Vp, tab, bs, nq, nkv, hd, rope, pos=pos)
    out = ab.decode_paged(qr, Kp, Vp, tab, bs, pos, nq, nkv, hd, max_kv_len=max(lens))
    torch.cuda.synchronize()
    assert ab.device_status() == 0
    Ks = [gather_rows(Kp, table[b], bs, L) for b, L in enumerate(lens)]
    Vs = [gather_rows(Vp, table[b], bs, L) for b, L in enumerate(lens)]
    for b in range(B):   # the appended row is V as given, K roped (as prep on a contiguous cache)
        assert torch.equal(Vs[b][-1], v[b].half())
    ref = oracle.decode_batch(qr.cpu().numpy(), [x.float().cpu().numpy() for x in Ks],
                              [x.float().cpu().numpy() for x in Vs], [L - 1 for L in lens], nq,
                              nkv, hd)
    assert_parity(out.cpu().numpy(), ref, what="prep_paged + decode_paged")


@pytest.mark.parametrize("hd,nq,nkv,bs,window,softcap", [(128, 32, 8, 128, 0, 0.0),
                                                         (128, 16, 4, 256, 300, 0.0),
                                                         (64, 8, 2, 128, 0, 0.0),
                                                         (256, 16, 8, 64, 0, 50.0),
                                                         (256, 16, 8, 128, 1024, 50.0)])
def test_prefill_paged_matches_contiguous(ab, oracle, hd, nq, nkv, bs, window, softcap):
    """Prefill of P tokens after a cached prefix, K/V in scattered pool blocks
    (the block after the sequence's end holds finite garbage). Bit-exact with
    the contiguous prefill; oracle on sampled rows."""
    P, ps = 700, 333
    L = ps + P
    nb = (L + bs - 1) // bs
    total = nb + 3
    table = scattered_tables(1, [nb], total, hd + bs)[0]
    g = torch.Generator(device="cuda").manual_seed(hd + bs + window)
    Kp = torch.randn(total * bs, nkv * hd, generator=g, device="cuda").half()
    Vp = torch.randn(total * bs, nkv * hd, generator=g, device="cuda").half()
    q = torch.randn(P, nq * hd, generator=g, device="cuda").half()
    scale = 1.0 / 16 if hd == 256 else None
    got = ab.prefill_paged(q, Kp, Vp, torch.from_numpy(table).cuda(), bs, nq, nkv, hd, ps,
                           scale=scale, window=window, softcap=softcap, out_dtype=torch.float32)
    K = gather_rows(Kp, table, bs, L).contiguous()
    V = gather_rows(Vp, table, bs, L).contiguous()
    ref_c = ab.prefill(q, K, V, nq, nkv, hd, ps, scale=scale, window=window, softcap=softcap,
                       out_dtype=torch.float32)
    torch.cuda.synchronize()
    assert ab.device_status() == 0
    assert torch.equal(got, ref_c)
    rows = [0, 1, 127, 128, 400, P - 1]
    ref = oracle.prefill(q.float().cpu().numpy(), K.float().cpu().numpy(),
                         V.float().cpu().numpy(), ps, nq, nkv, hd, rows=rows,
                         scale=scale, window=window, softcap=softcap)
    assert_parity(got.cpu().numpy()[rows], ref[rows], what=f"prefill_paged hd{hd}")


def test_prefill_paged_rejects_small_blocks(ab):
    from aspida_b200.attention import GPUError
    nq, nkv, hd, bs = 8, 2, 128, 64          # 64 < the 128-key tile of hd 128
    Kp = torch.zeros(4 * bs, nkv * hd, dtype=torch.half, device="cuda")
    q = torch.zeros(10, nq * hd, dtype=torch.half, device="cuda")
    tab = torch.arange(4, dtype=torch.int32, device="cuda")
    with pytest.raises(GPUError) as e:
        ab.prefill_paged(q, Kp, Kp, tab, bs, nq, nkv, hd, 0)
    assert e.value.code == -4
