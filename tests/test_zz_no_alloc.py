"""The allocation-free decode entry point, aspida_attn_decode_noalloc.

It serves callers that cannot allocate device memory (allocator callbacks,
fixed pre-reserved budgets, threads that must not block on cudaMalloc's
device synchronisation): its scratch is an array compiled into the library.
This test calls it through the C ABI twice in a row, with the library's
allocation hook armed so that any device allocation it made would fail, and
checks each result against the CPU oracle within the suite's tolerance (and
against aspida_attn_decode, the entry point with a caller workspace). The
file is collected last so that a run stopping at the first failure has
already run every other test; it also passes alone.
"""
import math

import numpy as np
import pytest
import torch

from tests.util import assert_parity

pytestmark = pytest.mark.gpu


def test_noalloc_matches_oracle_twice(oracle):
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    import aspida_b200 as ab
    from aspida_b200 import _lib

    lib = _lib.load()
    nq, nkv, hd = 32, 8, 128
    rng = np.random.RandomState(21)
    for call in range(2):
        lens = rng.randint(1, 6000, size=12).tolist()
        g = torch.Generator(device="cuda").manual_seed(100 + call)
        Ks = [torch.randn(L, nkv * hd, generator=g, device="cuda").half() for L in lens]
        Vs = [torch.randn(L, nkv * hd, generator=g, device="cuda").half() for L in lens]
        q = torch.randn(len(lens), nq * hd, generator=g, device="cuda")
        Kt, Vt = ab.ptr_table(Ks, q.device), ab.ptr_table(Vs, q.device)
        pos = torch.tensor([L - 1 for L in lens], dtype=torch.int32, device="cuda")
        ref_ws = ab.decode(q, Kt, Vt, pos, nq, nkv, hd, max_kv_len=max(lens))
        out = torch.full_like(ref_ws, float("nan"))
        stream = torch.cuda.current_stream().cuda_stream
        torch.cuda.synchronize()
        # any device allocation the library attempted from here on would fail
        lib.aspida_attn_debug_fail_allocs(1 << 20)
        try:
            rc = lib.aspida_attn_decode_noalloc(
                q.data_ptr(), None, Kt.data_ptr(), Vt.data_ptr(), pos.data_ptr(), None,
                out.data_ptr(), len(lens), nq, nkv, hd, 1.0 / math.sqrt(hd), 0, 0.0, max(lens),
                0, stream)
            torch.cuda.synchronize()
            status = ab.device_status()
        finally:
            lib.aspida_attn_debug_fail_allocs(0)
        assert rc == 0
        assert status == 0
        got = out.cpu().numpy()
        ref = oracle.decode_batch(q.cpu().numpy(), [k.float().cpu().numpy() for k in Ks],
                                  [v.float().cpu().numpy() for v in Vs], [L - 1 for L in lens],
                                  nq, nkv, hd)
        assert_parity(got, ref, what=f"noalloc call {call} vs oracle")
        assert_parity(got, ref_ws.cpu().numpy(), what=f"noalloc call {call} vs decode")
    # a batch needing more scratch than the compiled-in array is refused
    big = 4096
    rc = lib.aspida_attn_decode_noalloc(
        q.data_ptr(), None, Kt.data_ptr(), Vt.data_ptr(), pos.data_ptr(), None, out.data_ptr(),
        big, nq, nkv, hd, 0.1, 0, 0.0, 8192, 0, None)
    assert rc == ab.ASPIDA_ERR_WORKSPACE
    ab.last_error()
