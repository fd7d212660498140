"""fe_evict_noalloc: evict() for callers that cannot allocate device memory.

Some hosts run eviction where no device allocation is allowed (a memory pool
that owns the whole GPU, a serving loop that forbids cudaMalloc, a C/FFI host
without an allocator).  fe_evict_noalloc keeps the only scratch the path
needs -- the per-row softmax statistics -- in a fixed array inside the
library.  This test calls it through the C ABI twice in a row, with different
inputs, and checks each result against fe_evict (which takes a
caller-allocated workspace) on the same inputs.  The file name sorts last so
that a stop-at-first-failure run has already run every other test.
"""
import pytest
import torch

from flash_evict import _lib

pytestmark = pytest.mark.gpu


def _call(fn_name, q, k, v, budget, recent, pool, decay, window, weighted, with_workspace):
    lib = _lib.load()
    b, h, n, d = q.shape
    hk = k.shape[1]
    out = torch.empty_like(q)
    imp = torch.empty(b, hk, n, device=q.device)
    idx = torch.empty(b, hk, budget, dtype=torch.int64, device=q.device)
    mask = torch.empty(b, hk, n, dtype=torch.bool, device=q.device)
    dtype = _lib.DTYPE_BF16 if q.dtype == torch.bfloat16 else _lib.DTYPE_F16
    args = [q.data_ptr(), _lib.strides(q), k.data_ptr(), _lib.strides(k), v.data_ptr(), _lib.strides(v),
            out.data_ptr(), imp.data_ptr(), idx.data_ptr(), mask.data_ptr()]
    if with_workspace:
        stats = torch.empty(b, h, n, 2, device=q.device)
        args.append(stats.data_ptr())
    args += [b, h, hk, n, d, dtype, 1, d ** -0.5, decay, window, 1 if weighted else 0, budget, recent, pool,
             torch.cuda.current_stream().cuda_stream]
    _lib.check(getattr(lib, fn_name)(*args))
    torch.cuda.synchronize()
    return out, imp, idx, mask


def _inputs(seed, b, h, hk, n, d, dtype):
    g = torch.Generator().manual_seed(seed)
    q = torch.randn(b, n, h, d, generator=g).to(dtype).cuda().transpose(1, 2)
    k = torch.randn(b, hk, n, d, generator=g).to(dtype).cuda()
    v = torch.randn(b, hk, n, d, generator=g).to(dtype).cuda()
    return q, k, v


def test_no_alloc_matches_workspace_entry_point_twice():
    cases = [
        (_inputs(11, 1, 8, 2, 3000, 128, torch.bfloat16), 300, 32, 5, 0.05, 0, True, 0.012),
        (_inputs(12, 2, 4, 4, 1500, 64, torch.float16), 150, 0, 1, 0.0, 128, False, 0.002),
    ]
    for (q, k, v), budget, recent, pool, decay, window, weighted, atol in cases:
        ref = _call("fe_evict", q, k, v, budget, recent, pool, decay, window, weighted, True)
        got = _call("fe_evict_noalloc", q, k, v, budget, recent, pool, decay, window, weighted, False)
        # Same three kernels on the same inputs, so the same bits: any
        # difference would point at the shared scratch (aliasing, offsets).
        assert torch.equal(got[0], ref[0])
        assert torch.equal(got[1].view(torch.int32), ref[1].view(torch.int32))
        assert torch.equal(got[2], ref[2])
        assert torch.equal(got[3], ref[3])
    assert _lib.device_status(torch.cuda.current_device()) == 0


def test_no_alloc_reports_an_earlier_timeout_then_runs():
    # A kernel that gave up on a wait after an earlier call returned is
    # reported by the next call, here the allocation-free one (which launches
    # nothing then); the call after it runs and matches fe_evict bit for bit.
    lib = _lib.load()
    dev = torch.cuda.current_device()
    _lib.device_status(dev, clear=True)
    (q, k, v) = _inputs(13, 1, 4, 2, 900, 64, torch.float16)
    ref = _call("fe_evict", q, k, v, 90, 8, 3, 0.0, 0, True, True)
    _lib.check(lib.fe_watchdog_selftest(2_000_000, torch.cuda.current_stream().cuda_stream))
    torch.cuda.synchronize()
    with pytest.raises(RuntimeError, match="device watchdog timeout"):
        _call("fe_evict_noalloc", q, k, v, 90, 8, 3, 0.0, 0, True, False)
    got = _call("fe_evict_noalloc", q, k, v, 90, 8, 3, 0.0, 0, True, False)
    for a, b_ in zip(got, ref):
        assert torch.equal(a.view(torch.int32) if a.dtype == torch.float32 else a,
                           b_.view(torch.int32) if b_.dtype == torch.float32 else b_)
    assert _lib.device_status(dev, clear=True) == _lib.STATUS_TIMEOUT


def test_no_alloc_rejects_oversized_requests():
    lib = _lib.load()
    q = torch.zeros(1, 1, 8, 64, device="cuda", dtype=torch.float16)
    st = _lib.strides(q)
    rc = lib.fe_evict_noalloc(q.data_ptr(), st, q.data_ptr(), st, q.data_ptr(), st, q.data_ptr(), q.data_ptr(),
                              q.data_ptr(), q.data_ptr(), 64, 64, 64, 2048, 64, _lib.DTYPE_F16, 1, 0.125, 0.0, 0, 1,
                              8, 0, 1, torch.cuda.current_stream().cuda_stream)
    assert rc == _lib.STATUS_UNSUPPORTED
    assert b"capacity" in lib.fe_last_error()
