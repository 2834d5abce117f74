"""GPU parity at the stated sizes of the benchmark configurations that the
other GPU tests reach only in part: config 1 (the CPU recipe run through the
GPU path: RoPE'd f32 Q/K, 32/8 heads, hd 64, 1024 keys), config 4 (Gemma-3
shapes: 8192-token prefill with global and window-1024 layers, softcap 50,
hd 256; decode B=8 at context 32768) and config 5a (one 131072-key sequence,
64/8 heads, hd 128, split into KV chunks and merged). Everything goes
through the C ABI; references come from the CPU oracle (on row / sequence
subsets where the full oracle would take minutes) and, for config 1, from
the reference kernel's own output in tests/golden.
"""
import math
import os

import numpy as np
import pytest
import torch

from tests.util import assert_parity

pytestmark = pytest.mark.gpu

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


@pytest.fixture(scope="module")
def ab():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    import aspida_b200
    return aspida_b200


def _f16(x):
    return np.asarray(x, np.float32).astype(np.float16).astype(np.float32)


# ---------------------------------------------------------------------------
# Config 1: batch 1, 32/8 heads, hd 64, KV length 1024, scale 1/8, f32 Q/K/V
# ~ N(0,1) from a seed, NeoX RoPE theta 500000 on Q/K at their positions
# (LLM_Llama: RoPE llm_llama.adb:829-844, attention 876-898).
# ---------------------------------------------------------------------------
def _cfg1_inputs():
    from tests.golden import cases
    c = next(c for c in cases.ATTN_CASES if c["name"].startswith("attn_cfg1"))
    Q, K, V, scale = cases.attn_inputs(c)
    return c, Q, K, V, float(scale)


def test_cfg1_recipe_prep_then_decode(ab, oracle):
    """Keys at positions 0..1023 and the query at 1023 are rotated by
    aspida_attn_prep (NeoX, theta 5e5, all 64 dims) while K/V are appended to
    the fp16 cache; aspida_attn_decode then attends all 1024 keys."""
    c, Q, K, V, scale = _cfg1_inputs()
    nq, nkv, hd, L = c["nh"], c["nkv"], c["hd"], c["seq"]
    dev = torch.device("cuda")
    qrows = np.zeros((L, nq * hd), np.float32)
    qrows[L - 1] = Q
    Kc = torch.zeros(L, nkv * hd, dtype=torch.float16, device=dev)
    Vc = torch.zeros(L, nkv * hd, dtype=torch.float16, device=dev)
    rope = ab.RopeParams(dim=hd, freq_base=500000.0)
    q_rot = ab.prep(torch.from_numpy(qrows).to(dev), torch.from_numpy(K).to(dev),
                    torch.from_numpy(V).to(dev), Kc, Vc, 0, nq, nkv, hd, rope)
    out = ab.decode(q_rot[L - 1:L].contiguous(), ab.ptr_table([Kc], dev),
                    ab.ptr_table([Vc], dev), torch.tensor([L - 1], dtype=torch.int32, device=dev),
                    nq, nkv, hd, scale=scale, max_kv_len=L)
    torch.cuda.synchronize()
    assert ab.device_status() == 0
    # oracle: the same recipe on the CPU (rotate, round the cache to fp16)
    q_ref = oracle.rope_rows(Q[None], nq, hd, [L - 1], 500000.0)
    K_ref = _f16(oracle.rope_rows(K, nkv, hd, range(L), 500000.0))
    ref = oracle.decode_batch(q_ref, [K_ref], [_f16(V)], [L - 1], nq, nkv, hd, scale=scale)
    assert_parity(out.cpu().numpy(), ref, what="cfg1 recipe")
    # the cache rows the prep wrote are the oracle's rotated keys, rounded
    np.testing.assert_allclose(Kc.float().cpu().numpy(), K_ref, rtol=0, atol=2e-3)


def test_cfg1_unroped_against_reference_kernel(ab):
    """The same inputs without RoPE against the reference kernel's own f32
    output (tests/golden/attn_cfg1_*.npz, k_attn run on a B200): only the
    fp16 rounding of the cache separates the two."""
    c, Q, K, V, scale = _cfg1_inputs()
    nq, nkv, hd, L = c["nh"], c["nkv"], c["hd"], c["seq"]
    dev = torch.device("cuda")
    Kc = torch.from_numpy(K).to(dev).half()
    Vc = torch.from_numpy(V).to(dev).half()
    out = ab.decode(torch.from_numpy(Q[None]).to(dev), ab.ptr_table([Kc], dev),
                    ab.ptr_table([Vc], dev), torch.tensor([L - 1], dtype=torch.int32, device=dev),
                    nq, nkv, hd, scale=scale, max_kv_len=L)
    torch.cuda.synchronize()
    gold = np.load(os.path.join(GOLDEN, c["name"] + ".npz"))["out"]
    assert_parity(out.cpu().numpy()[0], gold, what="cfg1 vs reference kernel")


# ---------------------------------------------------------------------------
# Config 4: Gemma-3-12B shapes, 16/8 heads, hd 256, softcap 50, layers of
# window 1024 (local) and global; prefill 8192 tokens; decode B=8 at 32768
# (LLM_Gemma attention, llm_gemma.adb:534-572: Lo = max(0, p - win + 1)).
# ---------------------------------------------------------------------------
CFG4 = dict(nq=16, nkv=8, hd=256)


@pytest.fixture(scope="module")
def cfg4_prefill_inputs(ab):
    P = 8192
    nq, nkv, hd = CFG4["nq"], CFG4["nkv"], CFG4["hd"]
    g = torch.Generator(device="cuda").manual_seed(404)
    q = torch.randn(P, nq * hd, generator=g, device="cuda").half()
    K = torch.randn(P, nkv * hd, generator=g, device="cuda").half()
    V = torch.randn(P, nkv * hd, generator=g, device="cuda").half()
    host = (q.float().cpu().numpy(), K.float().cpu().numpy(), V.float().cpu().numpy())
    return q, K, V, host


@pytest.mark.parametrize("window,scale,out_dtype", [
    (0, 1.0 / 16, torch.float32), (1024, 1.0 / 16, torch.float32),
    (0, 1.0, torch.float32), (1024, 1.0, torch.float16)])
def test_cfg4_prefill_full_size_rows(ab, oracle, cfg4_prefill_inputs, window, scale, out_dtype):
    """8192-token causal prefill at hd 256 with softcap 50, global and
    window-1024, at scale 1/16 and 1.0; checked on the last 256 rows and
    every 64th row."""
    q, K, V, (qh, Kh, Vh) = cfg4_prefill_inputs
    nq, nkv, hd = CFG4["nq"], CFG4["nkv"], CFG4["hd"]
    P = q.shape[0]
    out = ab.prefill(q, K, V, nq, nkv, hd, 0, scale=scale, window=window, softcap=50.0,
                     out_dtype=out_dtype)
    torch.cuda.synchronize()
    assert ab.device_status() == 0
    rows = sorted(set(range(P - 256, P)) | set(range(0, P, 64)))
    ref = oracle.prefill(qh, Kh, Vh, 0, nq, nkv, hd, rows=rows, scale=scale, window=window,
                         softcap=50.0)
    tol = 2e-3 if out_dtype == torch.float32 else 4e-3   # fp16 output rounding adds <= 2^-11 |o|
    assert_parity(out.float().cpu().numpy()[rows], ref[rows], max_abs=tol,
                  what=f"cfg4 prefill window {window} scale {scale}")


@pytest.mark.parametrize("window,scale", [(0, 1.0 / 16), (1024, 1.0 / 16), (0, 1.0)])
def test_cfg4_decode_b8_ctx32768_sampled(ab, oracle, window, scale):
    """Decode B=8 at context 32768 (2.1 GB of fp16 KV), softcap 50; two
    sampled sequences against the oracle."""
    nq, nkv, hd, B, L = CFG4["nq"], CFG4["nkv"], CFG4["hd"], 8, 32768
    dev = torch.device("cuda")
    g = torch.Generator(device="cuda").manual_seed(4040)
    Ks = [torch.randn(L, nkv * hd, generator=g, device=dev).half() for _ in range(B)]
    Vs = [torch.randn(L, nkv * hd, generator=g, device=dev).half() for _ in range(B)]
    q = torch.randn(B, nq * hd, generator=g, device=dev)
    pos = torch.full((B,), L - 1, dtype=torch.int32, device=dev)
    out = ab.decode(q, ab.ptr_table(Ks, dev), ab.ptr_table(Vs, dev), pos, nq, nkv, hd,
                    scale=scale, window=window, softcap=50.0, max_kv_len=L)
    torch.cuda.synchronize()
    assert ab.device_status() == 0
    got = out.cpu().numpy()
    pick = [1, 6]
    ref = oracle.decode_batch(q.cpu().numpy()[pick], [Ks[b].float().cpu().numpy() for b in pick],
                              [Vs[b].float().cpu().numpy() for b in pick], [L - 1] * len(pick),
                              nq, nkv, hd, scale=scale, window=window, softcap=50.0)
    assert_parity(got[pick], ref, what=f"cfg4 decode window {window} scale {scale}")


# ---------------------------------------------------------------------------
# Config 5a: Llama-3-70B shapes, one sequence at KV length 131072, 64/8
# heads, hd 128, the cache split into chunks whose (m, l, o) partials are
# merged (the split-K combine of gpu/fattn_sk.cu:84-97).
# ---------------------------------------------------------------------------
@pytest.fixture(scope="module")
def cfg5a(ab, oracle):
    nq, nkv, hd, L = 64, 8, 128, 131072
    dev = torch.device("cuda")
    g = torch.Generator(device="cuda").manual_seed(505)
    K = torch.randn(L, nkv * hd, generator=g, device=dev).half()
    V = torch.randn(L, nkv * hd, generator=g, device=dev).half()
    q = torch.randn(1, nq * hd, generator=g, device=dev)
    ref = oracle.decode_batch(q.cpu().numpy(), [K.float().cpu().numpy()],
                              [V.float().cpu().numpy()], [L - 1], nq, nkv, hd)
    return q, K, V, ref, (nq, nkv, hd, L)


def test_cfg5a_seq_parallel_world1(ab, cfg5a):
    """SeqParallelDecode with one rank holding all 131072 keys."""
    from aspida_b200 import shard
    q, K, V, ref, (nq, nkv, hd, L) = cfg5a
    op = shard.SeqParallelDecode([K], [V], L, nq, nkv, hd)
    try:
        for step in range(2):
            out = op(q).clone()
            torch.cuda.synchronize()
            assert ab.device_status() == 0
            assert_parity(out.cpu().numpy(), ref, what=f"cfg5a world 1 step {step}")
    finally:
        op.close()


@pytest.mark.parametrize("parts", [8, 3])
def test_cfg5a_chunk_partials_and_merge(ab, cfg5a, parts):
    """The 131072 keys split into `parts` chunks as kv_chunks deals them to
    ranks: one decode_partial per chunk (each chunk its own cache, as on its
    GPU), then aspida_attn_merge."""
    from aspida_b200 import shard
    q, K, V, ref, (nq, nkv, hd, L) = cfg5a
    dev = q.device
    ms, ls, os_ = [], [], []
    for lo, hi in shard.kv_chunks(L, parts):
        Kt = ab.ptr_table([K[lo:]], dev)
        Vt = ab.ptr_table([V[lo:]], dev)
        m, l, o = ab.decode_partial(q, Kt, Vt, torch.tensor([0], dtype=torch.int32, device=dev),
                                    torch.tensor([hi - lo], dtype=torch.int32, device=dev),
                                    nq, nkv, hd, max_kv_len=max(1, hi - lo))
        ms.append(m)
        ls.append(l)
        os_.append(o)
    out = ab.merge(torch.stack(ms).reshape(parts, -1), torch.stack(ls).reshape(parts, -1),
                   torch.stack(os_).reshape(parts, nq, hd))
    torch.cuda.synchronize()
    assert ab.device_status() == 0
    assert_parity(out.reshape(1, -1).cpu().numpy(), ref, what=f"cfg5a {parts} chunks")
