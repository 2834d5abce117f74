"""Golden-fixture cases: shapes, seeds and input generation.

Inputs are regenerated from `numpy.random.RandomState(seed)` (numpy's frozen
legacy stream), so a fixture stores only the case parameters and the
reference kernel's outputs. Used by make_golden.py (which ran the reference's
own kernels through oracle/ref_harness.cu) and by tests/test_oracle.py.
"""
import numpy as np

# Decode attention, reference kernel k_attn (gpu/experiments/phase1/ops.cu:39).
# "closed" is that file's own known-answer inputs (ops.cu:131-140).
ATTN_CASES = [
    dict(name="attn_closed_nh8_nkv2_hd128_seq40", nh=8, nkv=2, hd=128, seq=40, seed=None),
    dict(name="attn_cfg1_nh32_nkv8_hd64_seq1024", nh=32, nkv=8, hd=64, seq=1024, seed=11),
    dict(name="attn_nh32_nkv8_hd128_seq700", nh=32, nkv=8, hd=128, seq=700, seed=12),
    dict(name="attn_nh16_nkv8_hd256_seq333", nh=16, nkv=8, hd=256, seq=333, seed=13),
    dict(name="attn_nh64_nkv8_hd128_seq4096", nh=64, nkv=8, hd=128, seq=4096, seed=14),
]

# RoPE, reference kernel k_rope (gpu/experiments/phase1/ops.cu:18): NeoX
# split-half over the whole vector, theta /= ff[i].
ROPE_CASES = [
    dict(name="rope_d64_p7_b5e5", dim=64, pos=7, base=500000.0, ff="ones", seed=21),
    dict(name="rope_d128_p1023_b5e5", dim=128, pos=1023, base=500000.0, ff="ones", seed=22),
    dict(name="rope_d128_p4095_ff", dim=128, pos=4095, base=500000.0, ff="rand", seed=23),
    dict(name="rope_d256_p32767_b1e6", dim=256, pos=32767, base=1000000.0, ff="ones", seed=24),
    dict(name="rope_d64_p0", dim=64, pos=0, base=10000.0, ff="ones", seed=25),
]

# Gated causal chunk, reference kernel k_fattn_attend_chunk (gpu/fattn_bench.cu:72):
# P queries at pos_start.., keys 0..pos_start+t, scale 1/sqrt(hd), x sigmoid(gate).
CHUNK_CASES = [
    dict(name="chunk_nq8_nkv2_hd64_P48_ps37", nq=8, nkv=2, hd=64, P=48, ps=37, seed=31),
    dict(name="chunk_nq4_nkv1_hd128_P20_ps0", nq=4, nkv=1, hd=128, P=20, ps=0, seed=32),
    dict(name="chunk_nq32_nkv8_hd128_P16_ps500", nq=32, nkv=8, hd=128, P=16, ps=500, seed=33),
    dict(name="chunk_nq16_nkv8_hd256_P8_ps100", nq=16, nkv=8, hd=256, P=8, ps=100, seed=34),
]


def attn_inputs(c):
    nh, nkv, hd, seq = c["nh"], c["nkv"], c["hd"], c["seq"]
    if c["seed"] is None:  # ops.cu closed form
        Q = np.sin(0.01 * np.arange(nh * hd, dtype=np.float32)).astype(np.float32)
        i = np.arange(seq * nkv * hd, dtype=np.float32)
        K = np.cos(np.float32(0.013) * i).astype(np.float32)
        V = np.sin(np.float32(0.007) * i).astype(np.float32)
    else:
        r = np.random.RandomState(c["seed"])
        Q = r.standard_normal(nh * hd).astype(np.float32)
        K = r.standard_normal(seq * nkv * hd).astype(np.float32)
        V = r.standard_normal(seq * nkv * hd).astype(np.float32)
    scale = np.float32(1.0) / np.sqrt(np.float32(hd))
    return Q, K.reshape(seq, nkv * hd), V.reshape(seq, nkv * hd), np.float32(scale)


def rope_inputs(c):
    r = np.random.RandomState(c["seed"])
    x = r.standard_normal(c["dim"]).astype(np.float32)
    if c["ff"] == "ones":
        ff = np.ones(c["dim"] // 2, np.float32)
    else:
        ff = r.uniform(1.0, 4.0, c["dim"] // 2).astype(np.float32)
    return x, ff


def chunk_inputs(c):
    r = np.random.RandomState(c["seed"])
    nq, nkv, hd, P, ps = c["nq"], c["nkv"], c["hd"], c["P"], c["ps"]
    q = r.standard_normal((P, nq * hd)).astype(np.float32)
    g = r.standard_normal((P, nq * hd)).astype(np.float32)
    K = r.standard_normal((ps + P, nkv * hd)).astype(np.float32)
    V = r.standard_normal((ps + P, nkv * hd)).astype(np.float32)
    return q, g, K, V


# Q8_0 quantiser, reference kernel k_to_q8 (gpu/fattn_kvhalf.cu:143). Besides
# random blocks the input holds an all-zero block, a one-value block, a block
# of exact ties (max 127 so d = 1, values k + 0.5), negative extremes and a
# large-magnitude block.
Q8_QUANT_CASES = [
    dict(name="q8quant_n4096", nblk=4096, seed=41),
]

# Gated causal GQA over a Q8_0 cache, reference kernel k_gqa_kv<2, hd/32, 2>
# (gpu/fattn_kvhalf.cu:59), which quantises K/V with k_to_q8 first. P = 1 is
# the decode shape (one query at position ps).
Q8_GQA_CASES = [
    dict(name="q8gqa_nq16_nkv2_hd256_P8_ps300", nq=16, nkv=2, hd=256, P=8, ps=300, seed=51),
    dict(name="q8gqa_nq32_nkv8_hd128_P4_ps1000", nq=32, nkv=8, hd=128, P=4, ps=1000, seed=52),
    dict(name="q8gqa_nq8_nkv2_hd128_P1_ps777", nq=8, nkv=2, hd=128, P=1, ps=777, seed=53),
]


def q8_quant_inputs(c):
    r = np.random.RandomState(c["seed"])
    x = (r.standard_normal((c["nblk"], 32)) * 2.0).astype(np.float32)
    x[0] = 0.0
    x[1] = 0.0
    x[1, 7] = -3.25
    x[2] = np.arange(32, dtype=np.float32) - 15.5   # ties once scaled
    x[2, 0] = 127.0
    x[3] = -np.abs(x[3])
    x[4] *= 1000.0
    x[5] = 1e-6 * r.standard_normal(32).astype(np.float32)
    return x.reshape(-1)


def q8_gqa_inputs(c):
    return chunk_inputs(c)
