"""The allocation-free decode entry point, aspida_attn_decode_noalloc.

It serves callers that cannot allocate device memory (allocator callbacks,
fixed pre-reserved budgets, threads that must not block on cudaMalloc's
device synchronisation): its scratch is an array compiled into the library.
This test calls it through the C ABI twice in a row and checks each result
against aspida_attn_decode (the entry point with a caller workspace) within
the suite's tolerance. The file is collected last so that a run stopping at
the first failure has already run every other test; it also passes alone.
"""
import ctypes as C
import math

import numpy as np
import pytest
import torch

from tests.util import assert_parity

pytestmark = pytest.mark.gpu


def test_noalloc_matches_decode_twice():
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
        ref = ab.decode(q, Kt, Vt, pos, nq, nkv, hd, max_kv_len=max(lens))
        out = torch.full_like(ref, float("nan"))
        stream = torch.cuda.current_stream().cuda_stream
        rc = lib.aspida_attn_decode_noalloc(
            q.data_ptr(), None, Kt.data_ptr(), Vt.data_ptr(), pos.data_ptr(), None,
            out.data_ptr(), len(lens), nq, nkv, hd, 1.0 / math.sqrt(hd), 0, 0.0, max(lens), 0,
            stream)
        assert rc == 0
        torch.cuda.synchronize()
        assert_parity(out.cpu().numpy(), ref.cpu().numpy(), what=f"noalloc call {call}")
    # a batch needing more scratch than the compiled-in array is refused
    big = 4096
    rc = lib.aspida_attn_decode_noalloc(
        q.data_ptr(), None, Kt.data_ptr(), Vt.data_ptr(), pos.data_ptr(), None, out.data_ptr(),
        big, nq, nkv, hd, 0.1, 0, 0.0, 8192, 0, None)
    assert rc == ab.ASPIDA_ERR_WORKSPACE
    ab.last_error()
