"""CPU tests of the oracle (oracle/attn_oracle.cpp) — its pins.

1. Golden fixtures made by the reference's own fp32 kernels (k_attn, k_rope,
   k_fattn_attend_chunk) through oracle/ref_harness.cu (tests/golden/).
2. The reference's known-answer tests, restated:
   - gpu/experiments/phase1/ops.cu:131-153 closed-form GQA decode (abs 1e-4);
   - tests/test_mrope_sections.adb scenarios 1-5;
   - tests/test_rope_scale.adb linear-scale checks;
   - tests/test_fullattn.adb causality and incremental == batched (1e-5).
"""
import os

import numpy as np
import pytest

from tests.golden import cases

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def _fixture(name):
    p = os.path.join(GOLDEN, name + ".npz")
    if not os.path.exists(p):
        pytest.skip(f"golden fixture {name} not generated yet")
    return np.load(p)["out"]


# ---------------------------------------------------------------- golden pins
@pytest.mark.parametrize("c", cases.ATTN_CASES, ids=lambda c: c["name"])
def test_decode_matches_reference_kernel(oracle, c):
    Q, K, V, scale = cases.attn_inputs(c)
    ref = _fixture(c["name"])
    got = oracle.decode_batch(Q[None], [K], [V], [c["seq"] - 1], c["nh"], c["nkv"], c["hd"],
                              scale=scale)[0]
    np.testing.assert_allclose(got, ref, rtol=2e-5, atol=2e-6)


@pytest.mark.parametrize("c", cases.ROPE_CASES, ids=lambda c: c["name"])
def test_rope_matches_reference_kernel(oracle, c):
    x, ff = cases.rope_inputs(c)
    ref = _fixture(c["name"])
    use_ff = None if c["ff"] == "ones" else ff
    got = oracle.rope_apply(x, c["base"], c["pos"], ff=use_ff)
    # theta = pos / base^(2i/d) in f32: a 1-ulp powf difference between CUDA and
    # libm moves the angle by ~pos * 6e-8 rad, so the bound grows with pos.
    np.testing.assert_allclose(got, ref, rtol=0, atol=2e-5 + 1.2e-7 * c["pos"] * np.abs(x).max())


@pytest.mark.parametrize("c", cases.CHUNK_CASES, ids=lambda c: c["name"])
def test_gated_chunk_matches_reference_kernel(oracle, c):
    q, g, K, V = cases.chunk_inputs(c)
    ref = _fixture(c["name"]).reshape(c["P"], -1)
    got = oracle.prefill(q, K, V, c["ps"], c["nq"], c["nkv"], c["hd"], gate=g)
    np.testing.assert_allclose(got, ref, rtol=2e-5, atol=2e-6)


def _npz(name):
    p = os.path.join(GOLDEN, name + ".npz")
    if not os.path.exists(p):
        pytest.skip(f"golden fixture {name} not generated yet")
    return np.load(p)


@pytest.mark.parametrize("c", cases.Q8_QUANT_CASES, ids=lambda c: c["name"])
def test_q8_quantiser_matches_reference_kernel(oracle, c):
    """Bit-exact against k_to_q8 (gpu/fattn_kvhalf.cu:143) incl. zero, tie and
    extreme blocks."""
    x = cases.q8_quant_inputs(c)
    ref = _npz(c["name"])
    q, s = oracle.quantize_q8(x)
    np.testing.assert_array_equal(q.reshape(-1), ref["q"])
    np.testing.assert_array_equal(s.reshape(-1).view(np.uint16), ref["scales"].view(np.uint16))


@pytest.mark.parametrize("c", cases.Q8_GQA_CASES, ids=lambda c: c["name"])
def test_q8_gqa_matches_reference_kernel(oracle, c):
    """The oracle's gated causal attention over the dequantised Q8_0 cache
    against k_gqa_kv<2, hd/32, 2> (gpu/fattn_kvhalf.cu:59) on the same cache."""
    q, g, K, V = cases.q8_gqa_inputs(c)
    ref = _npz(c["name"])["out"].reshape(c["P"], -1)
    Kd = oracle.dequantize_q8(*oracle.quantize_q8(K))
    Vd = oracle.dequantize_q8(*oracle.quantize_q8(V))
    got = oracle.prefill(q, Kd, Vd, c["ps"], c["nq"], c["nkv"], c["hd"], gate=g)
    np.testing.assert_allclose(got, ref, rtol=2e-5, atol=2e-6)


# ------------------------------------------------------- known-answer restated
def test_closed_form_gqa_decode_known_answer(oracle):
    """ops.cu:131-153: nh8/nkv2/hd128/seq40 closed-form inputs, abs tol 1e-4,
    against an independent float64 evaluation of the same formula."""
    c = cases.ATTN_CASES[0]
    Q, K, V, scale = cases.attn_inputs(c)
    got = oracle.decode_batch(Q[None], [K], [V], [c["seq"] - 1], 8, 2, 128, scale=scale)[0]
    exp = np.empty(8 * 128)
    for h in range(8):
        kv = h // 4
        q = Q[h * 128:(h + 1) * 128].astype(np.float64)
        k = K[:, kv * 128:(kv + 1) * 128].astype(np.float64)
        v = V[:, kv * 128:(kv + 1) * 128].astype(np.float64)
        s = k @ q * float(scale)
        p = np.exp(s - s.max())
        exp[h * 128:(h + 1) * 128] = (p / p.sum()) @ v
    assert np.max(np.abs(got - exp)) < 1e-4


def _fill_x(d):
    return (0.13 * np.arange(1, d + 1, dtype=np.float32) - 0.7).astype(np.float32)


def test_mrope_sections_scenarios(oracle):
    """tests/test_mrope_sections.adb scenarios 1-5."""
    ap = oracle.rope_apply_sections
    # 1: Sections [11,11,10,0], Dim 64: Apply(P,X,p) == Apply_Sections(P,X,Uniform[p])
    x = _fill_x(64)
    for p in (7, 0, -3):
        a = ap(x, 1e6, [11, 11, 10, 0], [p] * 4)
        b = oracle.rope_apply(x, 1e6, p)
        np.testing.assert_allclose(a, b, atol=1e-5, rtol=0)
    # 2: single section [16,0,0,0] == legacy Apply
    x = _fill_x(32)
    np.testing.assert_allclose(ap(x, 1e6, [16, 0, 0, 0], [5, 0, 0, 0]), oracle.rope_apply(x, 1e6, 5),
                               atol=1e-5, rtol=0)
    np.testing.assert_allclose(ap(x, 1e6, [16, 0, 0, 0], [0] * 4), oracle.rope_apply(x, 1e6, 0),
                               atol=1e-5, rtol=0)
    # 3: section in the middle [0,16,0,0] at Pos 11 rotates both halves
    r = ap(x, 1e6, [0, 16, 0, 0], [0, 11, 0, 0])
    assert not np.array_equal(r[:16], x[:16]) and not np.array_equal(r[16:], x[16:])
    # 4: two sections [8,8,0,0]: pairs 0..7 follow Sec(0), 8..15 follow Sec(1)
    r_mix = ap(x, 1e6, [8, 8, 0, 0], [5, 9, 0, 0])
    r_uni = ap(x, 1e6, [8, 8, 0, 0], [5, 5, 0, 0])
    r_s0 = ap(x, 1e6, [8, 8, 0, 0], [5, 0, 0, 0])
    assert np.array_equal(r_mix[:8], r_uni[:8]) and np.array_equal(r_mix[16:24], r_uni[16:24])
    assert not np.array_equal(r_mix[8:16], r_uni[8:16]) or not np.array_equal(r_mix[24:], r_uni[24:])
    assert not np.array_equal(r_mix[8:16], r_s0[8:16]) or not np.array_equal(r_mix[24:], r_s0[24:])
    # 5: trailing empty section ignores its position; section 0 matches Apply
    x = _fill_x(48)
    r_bad = ap(x, 1e6, [8, 8, 8, 0], [3, 5, 7, 999])
    r_ok = ap(x, 1e6, [8, 8, 8, 0], [3, 5, 7, 0])
    np.testing.assert_allclose(r_bad, r_ok, atol=1e-5, rtol=0)
    assert np.array_equal(r_ok[:8], oracle.rope_apply(x, 1e6, 3)[:8])


def test_rope_linear_scale(oracle):
    """tests/test_rope_scale.adb: factor 1 no-op; factor 2 scaled@4 == unscaled@2."""
    x = (0.1 * np.arange(1, 9, dtype=np.float32) - 0.3).astype(np.float32)
    sec = [11, 11, 10, 0]
    base = oracle.rope_apply_sections(x, 1e4, sec, [4] * 4)
    noop = oracle.rope_apply_sections(x, 1e4, sec, [4] * 4, freq_scale=1.0)
    np.testing.assert_allclose(noop, base, atol=1e-5, rtol=0)
    s4 = oracle.rope_apply_sections(x, 1e4, sec, [4] * 4, freq_scale=0.5)
    u2 = oracle.rope_apply_sections(x, 1e4, sec, [2] * 4)
    np.testing.assert_allclose(s4, u2, atol=1e-5, rtol=0)
    s8 = oracle.rope_apply_sections(x, 1e4, sec, [8] * 4, freq_scale=0.5)
    u4 = oracle.rope_apply_sections(x, 1e4, sec, [4] * 4)
    np.testing.assert_allclose(s8, u4, atol=1e-5, rtol=0)
    assert np.max(np.abs(s4 - base)) > 1e-5


# tests/test_fullattn.adb: dim 4, hd 4, 2 q heads / 1 kv head, rope dim 2.
def _mk2(rows, cols, seed):
    r = np.arange(1, rows + 1)[:, None]
    c = np.arange(1, cols + 1)[None, :]
    return (0.1 * (((r * 7 + c * 3 + seed) % 11) - 5)).astype(np.float32)


def _mk1(n, seed):
    i = np.arange(1, n + 1)
    return (0.5 + 0.1 * ((i * 5 + seed) % 7)).astype(np.float32)


def _fullattn_layer_outputs(oracle, X):
    """LLM_FullAttn.Forward (llm_fullattn.adb:88-231) on rows X [T, 4]."""
    dim, hd, nq, nkv, rd = 4, 4, 2, 1, 2
    Wq, Wk, Wv = _mk2(nq * 2 * hd, dim, 1), _mk2(nkv * hd, dim, 2), _mk2(nkv * hd, dim, 3)
    qn, kn, Wo = _mk1(hd, 4), _mk1(hd, 5), _mk2(dim, nq * hd, 6)
    T = X.shape[0]
    q_all = np.zeros((T, nq * hd), np.float32)
    g_all = np.zeros((T, nq * hd), np.float32)
    K = np.zeros((T, nkv * hd), np.float32)
    V = np.zeros((T, nkv * hd), np.float32)
    for t in range(T):
        qg, kt, vt = Wq @ X[t], Wk @ X[t], Wv @ X[t]
        for h in range(nq):
            g_all[t, h * hd:(h + 1) * hd] = qg[h * 2 * hd + hd:(h + 1) * 2 * hd]
            q_all[t, h * hd:(h + 1) * hd] = oracle.norm_rope(qg[h * 2 * hd:h * 2 * hd + hd], qn, hd,
                                                             rd, t, 1e4)
        K[t] = oracle.norm_rope(kt, kn, hd, rd, t, 1e4)
        V[t] = vt
    attn = oracle.prefill(q_all, K, V, 0, nq, nkv, hd, gate=g_all)
    return attn @ Wo.T, (q_all, g_all, K, V)


def test_fullattn_causal_and_incremental(oracle):
    X3 = np.array([[0.3 * t - 0.2 * i for i in range(1, 5)] for t in range(1, 4)], np.float32)
    O3, (q_all, g_all, K, V) = _fullattn_layer_outputs(oracle, X3)
    O2, _ = _fullattn_layer_outputs(oracle, X3[:2])
    assert O3.shape == (3, 4)
    assert np.all(np.abs(O3[:2] - O2) < 1e-5)                 # causal
    for t in range(3):                                         # incremental == batched
        a = oracle.decode_batch(q_all[t:t + 1], [K[:t + 1]], [V[:t + 1]], [t], 2, 1, 4,
                                gate=g_all[t:t + 1])
        step = a @ _mk2(4, 8, 6).T
        assert np.all(np.abs(step[0] - O3[t]) < 1e-5)


# ---------------------------------------------------------------- properties
def test_split_merge_equals_whole(oracle):
    """Splitting the keys into slices and merging (fattn_sk.cu:84-97) equals
    attending the whole range."""
    r = np.random.RandomState(5)
    nq, nkv, hd, L = 8, 2, 64, 300
    q = r.standard_normal((1, nq * hd)).astype(np.float32)
    K = r.standard_normal((L, nkv * hd)).astype(np.float32)
    V = r.standard_normal((L, nkv * hd)).astype(np.float32)
    whole = oracle.decode_batch(q, [K], [V], [L - 1], nq, nkv, hd)
    cuts = [0, 97, 98, 250, L]
    ms, ls, os_ = [], [], []
    scale = 1 / np.sqrt(hd)
    for a, b in zip(cuts[:-1], cuts[1:]):
        s = np.stack([K[a:b, (h // 4) * hd:(h // 4 + 1) * hd] @ q[0, h * hd:(h + 1) * hd]
                      for h in range(nq)]) * scale          # [nq, n]
        m = s.max(axis=1)
        p = np.exp(s - m[:, None])
        o = np.stack([p[h] @ V[a:b, (h // 4) * hd:(h // 4 + 1) * hd] for h in range(nq)])
        ms.append(m); ls.append(p.sum(axis=1)); os_.append(o)
    merged = oracle.merge(np.stack(ms), np.stack(ls), np.stack(os_))
    np.testing.assert_allclose(merged.reshape(-1), whole[0], atol=2e-6, rtol=1e-5)


def test_window_and_softcap_definitions(oracle):
    r = np.random.RandomState(6)
    nq, nkv, hd, L, W, cap = 4, 2, 64, 50, 16, 5.0
    q = r.standard_normal((1, nq * hd)).astype(np.float32) * 3
    K = r.standard_normal((L, nkv * hd)).astype(np.float32)
    V = r.standard_normal((L, nkv * hd)).astype(np.float32)
    got = oracle.decode_batch(q, [K], [V], [L - 1], nq, nkv, hd, window=W, softcap=cap, scale=1.0)
    for h in range(nq):
        kv = h // 2
        s = K[L - W:, kv * hd:(kv + 1) * hd].astype(np.float64) @ q[0, h * hd:(h + 1) * hd]
        s = cap * np.tanh(s / cap)
        p = np.exp(s - s.max()); p /= p.sum()
        np.testing.assert_allclose(got[0, h * hd:(h + 1) * hd], p @ V[L - W:, kv * hd:(kv + 1) * hd],
                                   atol=1e-5, rtol=1e-4)


def test_e4m3_codec_known_answers(oracle):
    """The numpy e4m3 codec (the fp8 KV oracle) against the OCP FP8 E4M3
    encoding: exact values, the largest finite value, saturation, the
    smallest normal and subnormal, ties to the even code, signed zero (a
    negative value that rounds to zero keeps its sign, as cvt does)."""
    cases = {1.0: 0x38, 0.5: 0x30, -2.0: 0xC0, 448.0: 0x7E, 1000.0: 0x7E, -1e9: 0xFE,
             2.0 ** -6: 0x08, 2.0 ** -9: 0x01, 0.875 * 2.0 ** -6: 0x07, 1.0625: 0x38,
             1.1875: 0x3A, 2.0 ** -10: 0x00, 3 * 2.0 ** -10: 0x02, 0.0: 0x00, 240.0: 0x77,
             -2.0 ** -11: 0x80}
    got = oracle.e4m3_encode(np.array(list(cases), np.float32))
    assert list(got) == list(cases.values())
    codes = np.arange(256, dtype=np.uint8)
    codes = codes[(codes & 0x7F) != 0x7F]                       # drop the NaN codes
    back = oracle.e4m3_encode(oracle.e4m3_decode(codes))
    assert np.array_equal(back, codes)


def test_fp8_block_quantiser_round_trip(oracle):
    rng = np.random.RandomState(61)
    x = (rng.standard_normal((64, 32)) * rng.uniform(0.01, 100, (64, 1))).astype(np.float32)
    x[0] = 0.0
    q, s = oracle.quantize_fp8(x)
    y = oracle.dequantize_fp8(q, s)
    assert np.all(y[0] == 0)
    # e4m3 keeps 3 mantissa bits: relative error <= 2^-4 of the block max
    err = np.abs(y - x).max(axis=1) / np.maximum(np.abs(x).max(axis=1), 1e-30)
    assert float(err.max()) <= 2.0 ** -4 + 1e-3
