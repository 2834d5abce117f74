"""GPU parity of the Q8_0 KV path: the quantiser (bit-exact against the
oracle restatement of k_to_q8, gpu/fattn_kvhalf.cu:143-152) and decode over
Q8_0 caches (against the oracle on the dequantised caches, and against the
reference kernel k_gqa_kv<..., 2>'s own output for the decode-shaped golden
case)."""
import math
import os

import numpy as np
import pytest
import torch

from tests.golden import cases
from tests.util import assert_parity

pytestmark = pytest.mark.gpu
GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


@pytest.fixture(scope="module")
def ab():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    import aspida_b200
    return aspida_b200


def make_q8_batch(ab, lens, nq, nkv, hd, seed, amp=1.0):
    g = torch.Generator(device="cuda").manual_seed(seed)
    kvd = nkv * hd
    K8, V8, Ks, Vs, Kf, Vf = [], [], [], [], [], []
    for L in lens:
        k = torch.randn(L, kvd, generator=g, device="cuda") * amp
        v = torch.randn(L, kvd, generator=g, device="cuda") * amp
        kq, ks = ab.quantize_q8(k)
        vq, vs = ab.quantize_q8(v)
        K8.append(kq); Ks.append(ks); V8.append(vq); Vs.append(vs)
        Kf.append(k); Vf.append(v)
    q = torch.randn(len(lens), nq * hd, generator=g, device="cuda")
    return q, K8, V8, Ks, Vs, Kf, Vf


def run_q8(ab, q, K8, V8, Ks, Vs, pos, nq, nkv, hd, **kw):
    dev = q.device
    tabs = [ab.ptr_table(x, dev) for x in (K8, V8, Ks, Vs)]
    p = torch.tensor(pos, dtype=torch.int32, device=dev)
    ml = kw.pop("max_len", None)
    mlt = torch.tensor(ml, dtype=torch.int32, device=dev) if ml is not None else None
    mkv = kw.pop("max_kv_len", max(pos) + 1)
    out = ab.decode_q8(q, *tabs, p, nq, nkv, hd, max_len=mlt, max_kv_len=mkv, **kw)
    torch.cuda.synchronize()
    assert ab.device_status() == 0
    return out.cpu().numpy()


def deq(oracle, q8, sc):
    return oracle.dequantize_q8(q8.cpu().numpy(), sc.cpu().numpy())


def test_quantiser_bit_exact(ab, oracle):
    c = cases.Q8_QUANT_CASES[0]
    x = cases.q8_quant_inputs(c)
    q, s = ab.quantize_q8(torch.from_numpy(x).cuda())
    qo, so = oracle.quantize_q8(x)
    np.testing.assert_array_equal(q.cpu().numpy(), qo)
    np.testing.assert_array_equal(s.cpu().numpy().view(np.uint16), so.view(np.uint16))
    r = np.random.RandomState(5).standard_normal(1 << 20).astype(np.float32) * 7
    q, s = ab.quantize_q8(torch.from_numpy(r).cuda())
    qo, so = oracle.quantize_q8(r)
    np.testing.assert_array_equal(q.cpu().numpy(), qo)
    np.testing.assert_array_equal(s.cpu().numpy().view(np.uint16), so.view(np.uint16))


def test_quantiser_appends_rows_in_place(ab, oracle):
    """Appending = quantising the new rows straight into the cache views."""
    kvd, rows = 8 * 128, 64
    cache = torch.zeros(rows, kvd, dtype=torch.int8, device="cuda")
    scales = torch.zeros(rows, kvd // 32, dtype=torch.float16, device="cuda")
    new = torch.randn(3, kvd, device="cuda")
    ab.quantize_q8(new, cache[10:13], scales[10:13])
    qo, so = oracle.quantize_q8(new.cpu().numpy())
    np.testing.assert_array_equal(cache[10:13].cpu().numpy(), qo)
    np.testing.assert_array_equal(scales[10:13].cpu().numpy().view(np.uint16), so.view(np.uint16))
    assert int(cache[:10].abs().sum()) == 0 and int(cache[13:].abs().sum()) == 0


@pytest.mark.parametrize("hd,nq,nkv", [(128, 32, 8), (128, 64, 8), (64, 32, 8), (256, 16, 8),
                                       (256, 16, 2), (128, 8, 2), (64, 16, 4), (256, 8, 1)])
def test_decode_q8_shapes(ab, oracle, hd, nq, nkv):
    lens = [1, 15, 16, 17, 100, 333, 1000, 2049]
    q, K8, V8, Ks, Vs, _, _ = make_q8_batch(ab, lens, nq, nkv, hd, seed=hd + nq + nkv)
    pos = [L - 1 for L in lens]
    got = run_q8(ab, q, K8, V8, Ks, Vs, pos, nq, nkv, hd, chunk=256)
    ref = oracle.decode_batch(q.cpu().numpy(), [deq(oracle, a, b) for a, b in zip(K8, Ks)],
                              [deq(oracle, a, b) for a, b in zip(V8, Vs)], pos, nq, nkv, hd)
    assert_parity(got, ref, what=f"q8 hd{hd} {nq}/{nkv}")


def test_decode_q8_window_softcap_gate_maxlen(ab, oracle):
    nq, nkv, hd = 32, 8, 128
    lens = [700, 1500, 90]
    q, K8, V8, Ks, Vs, _, _ = make_q8_batch(ab, lens, nq, nkv, hd, seed=77, amp=3.0)
    gate = torch.randn(len(lens), nq * hd, device="cuda")
    pos = [L - 1 for L in lens]
    Kd = [deq(oracle, a, b) for a, b in zip(K8, Ks)]
    Vd = [deq(oracle, a, b) for a, b in zip(V8, Vs)]
    got = run_q8(ab, q, K8, V8, Ks, Vs, pos, nq, nkv, hd, window=257, softcap=30.0, gate=gate,
                 scale=1.0)
    ref = oracle.decode_batch(q.cpu().numpy(), Kd, Vd, pos, nq, nkv, hd, window=257,
                              softcap=30.0, gate=gate.cpu().numpy(), scale=1.0)
    assert_parity(got, ref, what="q8 window/softcap/gate")
    # keys clamped below max_len
    ml = [500, 1500, 40]
    got = run_q8(ab, q, K8, V8, Ks, Vs, pos, nq, nkv, hd, max_len=ml)
    ref = oracle.decode_batch(q.cpu().numpy(), [k[:m] for k, m in zip(Kd, ml)],
                              [v[:m] for v, m in zip(Vd, ml)], [m - 1 for m in ml], nq, nkv, hd)
    assert_parity(got, ref, what="q8 max_len")


def test_decode_q8_matches_reference_kernel_output(ab):
    """Decode-shaped golden case (P = 1): the reference's own k_gqa_kv over
    its own k_to_q8 cache; our quantiser + decode_q8 must land on it."""
    c = [c for c in cases.Q8_GQA_CASES if c["P"] == 1][0]
    p = os.path.join(GOLDEN, c["name"] + ".npz")
    if not os.path.exists(p):
        pytest.skip("golden fixture missing")
    ref = np.load(p)["out"].reshape(1, -1)
    q, g, K, V = cases.q8_gqa_inputs(c)
    kq, ks = ab.quantize_q8(torch.from_numpy(K).cuda())
    vq, vs = ab.quantize_q8(torch.from_numpy(V).cuda())
    got = run_q8(ab, torch.from_numpy(q).cuda(), [kq], [vq], [ks], [vs], [c["ps"]], c["nq"],
                 c["nkv"], c["hd"], gate=torch.from_numpy(g).cuda(),
                 scale=1.0 / math.sqrt(c["hd"]))
    assert_parity(got, ref, what="q8 vs reference kernel")


def test_decode_q8_cfg2_full_size(ab, oracle):
    """Config-2 shape (B=32, 32/8, hd128, len ~ U[512, 8192]) on Q8_0 caches."""
    rng = np.random.RandomState(2)
    lens = rng.randint(512, 8193, size=32).tolist()
    q, K8, V8, Ks, Vs, _, _ = make_q8_batch(ab, lens, 32, 8, 128, seed=2)
    pos = [L - 1 for L in lens]
    got = run_q8(ab, q, K8, V8, Ks, Vs, pos, 32, 8, 128)
    ref = oracle.decode_batch(q.cpu().numpy(), [deq(oracle, a, b) for a, b in zip(K8, Ks)],
                              [deq(oracle, a, b) for a, b in zip(V8, Vs)], pos, 32, 8, 128)
    assert_parity(got, ref, what="q8 cfg2")


def test_decode_q8_unsupported_and_errors(ab):
    from aspida_b200.attention import GPUError
    nq, nkv, hd = 4, 1, 128      # group slice of 128 bytes: scales not 16-byte units
    q, K8, V8, Ks, Vs, _, _ = make_q8_batch(ab, [40], nq, nkv, hd, seed=1)
    with pytest.raises(GPUError) as e:
        run_q8(ab, q, K8, V8, Ks, Vs, [39], nq, nkv, hd)
    assert e.value.code == -4
    with pytest.raises(ValueError):
        ab.quantize_q8(torch.zeros(33, device="cuda"))


@pytest.mark.parametrize("c", cases.Q8_GQA_CASES, ids=lambda c: c["name"])
def test_prefill_q8_gated_matches_reference_kernel(ab, c):
    """aspida_attn_prefill_q8_gated on the golden cases: the reference's own
    k_to_q8 + k_gqa_kv<2, hd/32, 2> outputs (gated causal chunks over a Q8_0
    cache); our quantiser is bit-exact, so the caches are the same."""
    p = os.path.join(GOLDEN, c["name"] + ".npz")
    if not os.path.exists(p):
        pytest.skip("golden fixture missing")
    ref = np.load(p)["out"].reshape(c["P"], -1)
    q, g, K, V = cases.q8_gqa_inputs(c)
    kq, ks = ab.quantize_q8(torch.from_numpy(K).cuda())
    vq, vs = ab.quantize_q8(torch.from_numpy(V).cuda())
    got = ab.prefill_q8_gated(torch.from_numpy(q).cuda(), kq, vq, ks, vs, c["nq"], c["nkv"],
                              c["hd"], c["ps"], gate=torch.from_numpy(g).cuda())
    torch.cuda.synchronize()
    assert ab.device_status() == 0
    assert_parity(got.cpu().numpy(), ref, what=f"q8 prefill vs reference {c['name']}")


def test_prefill_q8_gated_hura_vs_oracle(ab, oracle):
    """A 300-token chunk after 2000 keys at the hura dims (16/2 heads, hd 256)
    against the oracle on the dequantised caches (sampled rows)."""
    nq, nkv, hd, P, ps = 16, 2, 256, 300, 2000
    g = torch.Generator(device="cuda").manual_seed(12)
    q = torch.randn(P, nq * hd, generator=g, device="cuda")
    gate = torch.randn(P, nq * hd, generator=g, device="cuda")
    K = torch.randn(ps + P, nkv * hd, generator=g, device="cuda")
    V = torch.randn(ps + P, nkv * hd, generator=g, device="cuda")
    kq, ks = ab.quantize_q8(K)
    vq, vs = ab.quantize_q8(V)
    got = ab.prefill_q8_gated(q, kq, vq, ks, vs, nq, nkv, hd, ps, gate=gate)
    torch.cuda.synchronize()
    rows = [0, 1, 127, 128, 200, 298, 299]
    ref = oracle.prefill(q.cpu().numpy(), deq(oracle, kq, ks), deq(oracle, vq, vs), ps, nq, nkv,
                         hd, gate=gate.cpu().numpy(), rows=rows)
    assert_parity(got.cpu().numpy()[rows], ref[rows], what="q8 prefill hura")
