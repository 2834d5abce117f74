"""GPU parity of the fp8 (e4m3) KV path: the block quantiser (bit-exact
against the numpy restatement in oracle.quantize_fp8, which is pinned to the
OCP E4M3 encoding by tests/test_oracle.py) and decode over fp8 caches (against
the oracle on the dequantised caches). The caches use the Q8_0 storage
geometry (8-bit values [rows][nkv*hd], fp16 scales per 32 values), so the
shapes mirror tests/test_q8_gpu.py."""
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


def make_fp8_batch(ab, lens, nq, nkv, hd, seed, amp=1.0):
    g = torch.Generator(device="cuda").manual_seed(seed)
    kvd = nkv * hd
    K8, V8, Ks, Vs = [], [], [], []
    for L in lens:
        k = torch.randn(L, kvd, generator=g, device="cuda") * amp
        v = torch.randn(L, kvd, generator=g, device="cuda") * amp
        kq, ks = ab.quantize_fp8(k)
        vq, vs = ab.quantize_fp8(v)
        K8.append(kq); Ks.append(ks); V8.append(vq); Vs.append(vs)
    q = torch.randn(len(lens), nq * hd, generator=g, device="cuda")
    return q, K8, V8, Ks, Vs


def run_fp8(ab, q, K8, V8, Ks, Vs, pos, nq, nkv, hd, **kw):
    dev = q.device
    tabs = [ab.ptr_table(x, dev) for x in (K8, V8, Ks, Vs)]
    p = torch.tensor(pos, dtype=torch.int32, device=dev)
    ml = kw.pop("max_len", None)
    mlt = torch.tensor(ml, dtype=torch.int32, device=dev) if ml is not None else None
    mkv = kw.pop("max_kv_len", max(pos) + 1)
    out = ab.decode_fp8(q, *tabs, p, nq, nkv, hd, max_len=mlt, max_kv_len=mkv, **kw)
    torch.cuda.synchronize()
    assert ab.device_status() == 0
    return out.cpu().numpy()


def deq(oracle, q8, sc):
    return oracle.dequantize_fp8(q8.cpu().numpy(), sc.cpu().numpy())


def test_fp8_quantiser_bit_exact(ab, oracle):
    rng = np.random.RandomState(71)
    x = (rng.standard_normal((4096, 32)) * rng.uniform(1e-3, 300, (4096, 1))).astype(np.float32)
    x[0] = 0.0                          # zero block
    x[1] = 0.0
    x[1, 3] = -5.0                      # one value
    x[2] = np.arange(32, dtype=np.float32) * 14.0   # exact multiples after scaling
    x[3] *= 1e-6                        # scale in the fp16 subnormal range
    x[4] = 1e-30                        # scale rounds to zero
    x = x.reshape(-1)
    q, s = ab.quantize_fp8(torch.from_numpy(x).cuda())
    qo, so = oracle.quantize_fp8(x)
    np.testing.assert_array_equal(s.cpu().numpy().view(np.uint16), so.view(np.uint16))
    np.testing.assert_array_equal(q.cpu().numpy(), qo)
    r = np.random.RandomState(5).standard_normal(1 << 20).astype(np.float32) * 7
    q, s = ab.quantize_fp8(torch.from_numpy(r).cuda())
    qo, so = oracle.quantize_fp8(r)
    np.testing.assert_array_equal(q.cpu().numpy(), qo)
    np.testing.assert_array_equal(s.cpu().numpy().view(np.uint16), so.view(np.uint16))


@pytest.mark.parametrize("hd,nq,nkv", [(128, 32, 8), (128, 64, 8), (64, 32, 8), (256, 16, 8),
                                       (256, 16, 2), (128, 8, 2), (64, 16, 4), (256, 8, 1)])
def test_decode_fp8_shapes(ab, oracle, hd, nq, nkv):
    lens = [1, 15, 16, 17, 100, 333, 1000, 2049]
    q, K8, V8, Ks, Vs = make_fp8_batch(ab, lens, nq, nkv, hd, seed=hd + nq + nkv + 1)
    pos = [L - 1 for L in lens]
    got = run_fp8(ab, q, K8, V8, Ks, Vs, pos, nq, nkv, hd, chunk=256)
    ref = oracle.decode_batch(q.cpu().numpy(), [deq(oracle, a, b) for a, b in zip(K8, Ks)],
                              [deq(oracle, a, b) for a, b in zip(V8, Vs)], pos, nq, nkv, hd)
    assert_parity(got, ref, what=f"fp8 hd{hd} {nq}/{nkv}")


def test_decode_fp8_window_softcap_gate_maxlen(ab, oracle):
    nq, nkv, hd = 32, 8, 128
    lens = [700, 1500, 90]
    q, K8, V8, Ks, Vs = make_fp8_batch(ab, lens, nq, nkv, hd, seed=78, amp=3.0)
    gate = torch.randn(len(lens), nq * hd, device="cuda")
    pos = [L - 1 for L in lens]
    Kd = [deq(oracle, a, b) for a, b in zip(K8, Ks)]
    Vd = [deq(oracle, a, b) for a, b in zip(V8, Vs)]
    got = run_fp8(ab, q, K8, V8, Ks, Vs, pos, nq, nkv, hd, window=257, softcap=30.0, gate=gate,
                  scale=1.0)
    ref = oracle.decode_batch(q.cpu().numpy(), Kd, Vd, pos, nq, nkv, hd, window=257,
                              softcap=30.0, gate=gate.cpu().numpy(), scale=1.0)
    assert_parity(got, ref, what="fp8 window/softcap/gate")
    ml = [500, 1500, 40]
    got = run_fp8(ab, q, K8, V8, Ks, Vs, pos, nq, nkv, hd, max_len=ml)
    ref = oracle.decode_batch(q.cpu().numpy(), [k[:m] for k, m in zip(Kd, ml)],
                              [v[:m] for v, m in zip(Vd, ml)], [m - 1 for m in ml], nq, nkv, hd)
    assert_parity(got, ref, what="fp8 max_len")


def test_decode_fp8_cfg2_full_size(ab, oracle):
    """The config-2 batch (B=32, 32/8 heads, hd 128, len ~ U[512, 8192]) on
    fp8 caches; half the bytes of the fp16 cache."""
    rng = np.random.RandomState(2)
    lens = rng.randint(512, 8193, size=32).tolist()
    q, K8, V8, Ks, Vs = make_fp8_batch(ab, lens, 32, 8, 128, seed=22)
    pos = [L - 1 for L in lens]
    got = run_fp8(ab, q, K8, V8, Ks, Vs, pos, 32, 8, 128)
    ref = oracle.decode_batch(q.cpu().numpy(), [deq(oracle, a, b) for a, b in zip(K8, Ks)],
                              [deq(oracle, a, b) for a, b in zip(V8, Vs)], pos, 32, 8, 128)
    assert_parity(got, ref, what="fp8 cfg2")
