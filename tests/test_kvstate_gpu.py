"""KV-state lifecycle on the GPU: handle reuse, snapshot/restore round trips
(gpu/gpu_matvec.cu:1316-1425 semantics), failure paths via the host hook."""
import pytest
import torch

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def ab():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    import aspida_b200
    return aspida_b200


def test_new_free_reuse(ab):
    ab.last_error()                       # a status latched by an earlier test
    h1 = ab.fattn_new(128, 1024, 32)
    h2 = ab.fattn_new(64, 1024, 32)
    assert h1 >= 0 and h2 >= 0 and h1 != h2
    ab.fattn_free(h1)
    h3 = ab.fattn_new(32, 512, 8)
    assert h3 == h1                       # freed slot reused
    K, V = ab.fattn_kv(h3)
    assert K.shape == (32, 512) and K.dtype == torch.float16
    ab.fattn_free(h2)
    ab.fattn_free(h3)
    ab.fattn_free(12345)                  # unknown handle ignored
    assert ab.fattn_new(0, 1024, 32) == -1
    assert ab.last_error() == ab.ASPIDA_ERR_ARG


def test_snapshot_restore(ab):
    c = ab.KVCache(256, 8, 128, 32)
    c.K.copy_(torch.randn_like(c.K, dtype=torch.float32).half())
    c.V.copy_(torch.randn_like(c.V, dtype=torch.float32).half())
    k0, v0 = c.K[:100].clone(), c.V[:100].clone()
    slot = ab.fattn_snapshot(c.handle, 100, -1)
    assert slot >= 0
    d = ab.KVCache(300, 8, 128, 32)
    assert ab.fattn_restore(d.handle, slot) == 0
    assert torch.equal(d.K[:100], k0) and torch.equal(d.V[:100], v0)
    # overwrite the same slot in place
    c.K[:100].zero_()
    assert ab.fattn_snapshot(c.handle, 100, slot) == slot
    assert ab.fattn_restore(d.handle, slot) == 0
    assert float(d.K[:100].abs().max()) == 0.0
    # geometry mismatch and bad slots fail cleanly
    e = ab.KVCache(50, 8, 128, 32)
    assert ab.fattn_restore(e.handle, slot) == -1       # rows > max_len
    assert ab.fattn_restore(d.handle, 999) == -1
    assert ab.fattn_snapshot(c.handle, 0, -1) == -1
    assert ab.fattn_snapshot(c.handle, 257, -1) == -1
    ab.prefix_reset()
    assert ab.fattn_restore(d.handle, slot) == -1       # snapshots gone
    ab.last_error()
    for x in (c, d, e):
        x.free()


def test_allocation_failure_hook(ab):
    ab.last_error()
    ab.debug_fail_allocs(1)
    assert ab.fattn_new(16, 64, 4) == -1
    assert ab.last_error() == ab.ASPIDA_ERR_NOMEM
    ab.debug_fail_allocs(2)
    with pytest.raises(ab.GPUError):
        ab.KVCache(16, 1, 64, 4)
    ab.debug_fail_allocs(0)
    h = ab.fattn_new(16, 64, 4)
    assert h >= 0
    ab.fattn_free(h)
