"""GPU: determinism, layouts, the C ABI called directly, the watchdog path
(timeouts raised at the caller's next call, NaN poisoning), the exp2
polynomial and CUDA-graph capture.  Parity at the BASELINE configurations is
in test_gpu_parity_configs.py."""
import ctypes

import numpy as np
import pytest
import torch

from flash_evict import _lib, evict, prefill
from oracle import restate as O

pytestmark = pytest.mark.gpu


def test_deterministic_and_score_flag_bitwise():
    torch.manual_seed(0)
    q = torch.randn(2, 8, 3000, 128, device="cuda", dtype=torch.bfloat16)
    k = torch.randn(2, 2, 3000, 128, device="cuda", dtype=torch.bfloat16)
    v = torch.randn(2, 2, 3000, 128, device="cuda", dtype=torch.bfloat16)
    o1, i1 = prefill(q, k, v, recency_decay=0.01)
    o2, i2 = prefill(q, k, v, recency_decay=0.01)
    o3, none = prefill(q, k, v, score=False)
    assert none is None
    assert torch.equal(o1, o2) and torch.equal(o1, o3)
    assert torch.equal(i1.view(torch.int32), i2.view(torch.int32))


@pytest.mark.parametrize("d", [8, 17, 40, 96, 120])
def test_odd_channel_counts_and_layouts(d):
    torch.manual_seed(d)
    base = torch.randn(1, 300, 6, d + 3, device="cuda", dtype=torch.float16)
    q = base[..., :d].transpose(1, 2)          # row pitch not a multiple of 8 for odd d
    k = torch.randn(1, 3, 300, d, device="cuda", dtype=torch.float16)
    v = torch.randn(1, 300, 3, d, device="cuda", dtype=torch.float16).transpose(1, 2)
    out, imp = prefill(q, k, v)
    ref_out, ref_imp = O.materialized(q, k, v)
    torch.testing.assert_close(out.float().cpu(), torch.from_numpy(ref_out), atol=0.002, rtol=0.006)
    torch.testing.assert_close(imp.cpu(), torch.from_numpy(ref_imp), atol=3e-3, rtol=3e-4)
    assert out.is_contiguous()


def test_negative_and_zero_scale():
    torch.manual_seed(5)
    q = torch.randn(1, 2, 200, 64, device="cuda", dtype=torch.float16)
    k = torch.randn(1, 1, 200, 64, device="cuda", dtype=torch.float16)
    v = torch.randn(1, 1, 200, 64, device="cuda", dtype=torch.float16)
    for scale in (-0.2, 0.0):
        out, imp = prefill(q, k, v, scale=scale)
        ro, ri = O.materialized(q, k, v, scale=scale)
        torch.testing.assert_close(out.float().cpu(), torch.from_numpy(ro), atol=0.002, rtol=0.006)
        torch.testing.assert_close(imp.cpu(), torch.from_numpy(ri), atol=3e-3, rtol=3e-4)


def test_c_abi_evict_matches_python():
    torch.manual_seed(9)
    b, h, hk, n, d = 1, 4, 2, 1000, 64
    q = torch.randn(b, h, n, d, device="cuda", dtype=torch.bfloat16)
    k = torch.randn(b, hk, n, d, device="cuda", dtype=torch.bfloat16)
    v = torch.randn(b, hk, n, d, device="cuda", dtype=torch.bfloat16)
    out_py, imp_py, idx_py, mask_py = evict(q, k, v, 100, reserved_recent=16, pool_kernel=5,
                                            recency_decay=0.05, observation_window=300)
    lib = _lib.load()
    out = torch.empty_like(q)
    imp = torch.empty(b, hk, n, device="cuda")
    idx = torch.empty(b, hk, 100, dtype=torch.int64, device="cuda")
    mask = torch.empty(b, hk, n, dtype=torch.bool, device="cuda")
    stats = torch.empty(b, h, n, 2, device="cuda")
    rc = lib.fe_evict(q.data_ptr(), _lib.strides(q), k.data_ptr(), _lib.strides(k), v.data_ptr(), _lib.strides(v),
                      out.data_ptr(), imp.data_ptr(), idx.data_ptr(), mask.data_ptr(), stats.data_ptr(),
                      b, h, hk, n, d, _lib.DTYPE_BF16, 1, d ** -0.5, 0.05, 300, 1, 100, 16, 5,
                      torch.cuda.current_stream().cuda_stream)
    _lib.check(rc)
    torch.cuda.synchronize()
    assert torch.equal(out, out_py) and torch.equal(imp, imp_py)
    assert torch.equal(idx, idx_py) and torch.equal(mask, mask_py)


def test_watchdog_timeout_is_reported_not_hung():
    lib = _lib.load()
    dev = torch.cuda.current_device()
    assert _lib.device_status(dev, clear=True) == 0
    _lib.check(lib.fe_watchdog_selftest(2_000_000, torch.cuda.current_stream().cuda_stream))  # 2 ms
    assert _lib.device_status(dev, clear=True) == _lib.STATUS_TIMEOUT
    assert _lib.device_status(dev, clear=True) == 0
    # the context stays usable
    x = torch.randn(1, 1, 64, 64, device="cuda", dtype=torch.float16)
    out, _ = prefill(x, x, x)
    assert torch.isfinite(out.float()).all()


def _watchdog_trip(dev):
    """Launch the self-test kernel whose wait nothing satisfies (2 ms limit)
    and wait for it, so its status is in the host word when the next call
    enters the library."""
    lib = _lib.load()
    _lib.check(lib.fe_watchdog_selftest(2_000_000, torch.cuda.current_stream().cuda_stream))
    torch.cuda.synchronize(dev)


def test_watchdog_timeout_raises_at_next_call_then_clears():
    # An asynchronous kernel failure reaches the Python caller: the next call
    # on the device raises RuntimeError (and launches nothing), the call
    # after it runs normally and gives the same bits as before the failure.
    from flash_evict import check_status
    dev = torch.cuda.current_device()
    assert _lib.device_status(dev, clear=True) == 0
    g = torch.Generator().manual_seed(3)
    q = torch.randn(1, 4, 700, 64, generator=g).to(torch.float16).cuda()
    k = torch.randn(1, 2, 700, 64, generator=g).to(torch.float16).cuda()
    v = torch.randn(1, 2, 700, 64, generator=g).to(torch.float16).cuda()
    ref = evict(q, k, v, 64, reserved_recent=8)
    torch.cuda.synchronize()
    _watchdog_trip(dev)
    with pytest.raises(RuntimeError, match="device watchdog timeout"):
        evict(q, k, v, 64, reserved_recent=8)
    got = evict(q, k, v, 64, reserved_recent=8)
    torch.cuda.synchronize()
    for a, b_ in zip(got, ref):
        assert torch.equal(a, b_)
    # the synchronous check still sees the device record once, then clears it
    with pytest.raises(RuntimeError, match="device watchdog timeout"):
        check_status(dev)
    check_status(dev)


def test_check_status_reports_without_a_later_call():
    from flash_evict import check_status
    dev = torch.cuda.current_device()
    check_status()
    _watchdog_trip(dev)
    with pytest.raises(RuntimeError, match="device watchdog timeout"):
        check_status(torch.device("cuda", dev))
    check_status(dev)
    # the host word was cleared with the device word: the next call runs
    x = torch.randn(1, 1, 64, 64, device="cuda", dtype=torch.float16)
    prefill(x, x, x)
    check_status()


def test_replay_poisons_keys_reached_by_nan_row_statistics():
    # What an aborted attention launch leaves behind (NaN {m, l} for its
    # rows) makes the replay write NaN importance for every key those rows
    # attend to, instead of a plausible partial sum.
    from flash_evict.prefill import _attention, _replay
    g = torch.Generator().manual_seed(8)
    n = 600
    q = torch.randn(1, 4, n, 64, generator=g).to(torch.bfloat16).cuda()
    k = torch.randn(1, 2, n, 64, generator=g).to(torch.bfloat16).cuda()
    v = torch.randn(1, 2, n, 64, generator=g).to(torch.bfloat16).cuda()
    out = torch.empty_like(q)
    stats = torch.empty(1, 4, n, 2, device="cuda")
    _attention(q, k, v, out, stats, True, 64 ** -0.5)
    imp_ok = torch.empty(1, 2, n, device="cuda")
    _replay(q, k, v, stats, imp_ok, True, 64 ** -0.5, 0.0, 0, True)
    stats[0, 1, 300] = float("nan")       # query head 1 -> kv head 0, row 300
    imp = torch.empty(1, 2, n, device="cuda")
    _replay(q, k, v, stats, imp, True, 64 ** -0.5, 0.0, 0, True)
    torch.cuda.synchronize()
    assert torch.isnan(imp[0, 0, :301]).all()           # keys row 300 attends to (causal)
    assert torch.equal(imp[0, 0, 301:], imp_ok[0, 0, 301:])
    assert torch.equal(imp[0, 1], imp_ok[0, 1])          # the other kv head is untouched
    assert torch.isfinite(imp_ok).all()


def test_head_dim_above_256_is_rejected():
    # the reference's contract (prefill.py:95-96): head dimension <= 256
    x = torch.randn(1, 1, 64, 264, device="cuda", dtype=torch.float16)
    with pytest.raises(ValueError, match="256"):
        prefill(x, x, x)
    lib = _lib.load()
    y = torch.empty_like(x)
    st = torch.empty(1, 1, 64, 2, device="cuda")
    rc = lib.fe_attention_fwd(x.data_ptr(), _lib.strides(x), x.data_ptr(), _lib.strides(x), x.data_ptr(),
                              _lib.strides(x), y.data_ptr(), st.data_ptr(), 1, 1, 1, 64, 264, _lib.DTYPE_F16, 1,
                              ctypes.c_float(0.06), None, 0, torch.cuda.current_stream().cuda_stream)
    assert rc == _lib.STATUS_INVALID and b"256" in lib.fe_last_error()


def test_exp2_polynomial_error_bound():
    """The packed FMA-pipe exp2 used for part of the replay's exponentials:
    relative error within the fitted bound (2.7e-6) of float64 exp2 over the
    input range, at most 2^-125 (about 2.35e-38, far below the resolution of
    any sum it enters) below -125 and for -inf; the MUFU path within 2^-21."""
    xs = torch.cat([torch.linspace(-125.0, 8.0, 2_000_001), torch.tensor([-125.5, -126.0, -200.0, -1e30,
                                                                            float("-inf")])]).cuda()
    poly = torch.empty_like(xs)
    mufu = torch.empty_like(xs)
    _lib.check(_lib.load().fe_selftest_exp2(xs.data_ptr(), poly.data_ptr(), mufu.data_ptr(), xs.numel(),
                                            torch.cuda.current_stream().cuda_stream))
    torch.cuda.synchronize()
    x64 = xs.double()
    ref = torch.exp2(x64)
    main = xs >= -125.0
    rel_poly = ((poly.double() - ref).abs() / ref)[main]
    assert rel_poly.max().item() < 3e-6, rel_poly.max().item()
    assert torch.all((poly[~main] >= 0) & (poly[~main] <= 2.4e-38))
    normal = xs >= -126.0
    rel_mufu = ((mufu.double() - ref).abs() / ref)[normal]
    assert rel_mufu.max().item() < 2 ** -21


def test_evict_in_cuda_graph():
    # The whole path (three launches, host-side tensor-map encoding) captures
    # into a CUDA graph and replays with identical results.
    g = torch.Generator().manual_seed(21)
    q = torch.randn(1, 8, 2048, 128, generator=g).to(torch.bfloat16).cuda()
    k = torch.randn(1, 2, 2048, 128, generator=g).to(torch.bfloat16).cuda()
    v = torch.randn(1, 2, 2048, 128, generator=g).to(torch.bfloat16).cuda()
    ref = evict(q, k, v, 256, reserved_recent=16, pool_kernel=5, recency_decay=0.05)
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        evict(q, k, v, 256, reserved_recent=16, pool_kernel=5, recency_decay=0.05)  # warm-up on the side stream
    torch.cuda.current_stream().wait_stream(s)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        out = evict(q, k, v, 256, reserved_recent=16, pool_kernel=5, recency_decay=0.05)
    for _ in range(3):
        graph.replay()
    torch.cuda.synchronize()
    for a, b in zip(out, ref):
        assert torch.equal(a, b)
    # new inputs in the same buffers are picked up by the replay
    q.copy_(torch.randn(q.shape, generator=g).to(q.dtype))
    graph.replay()
    torch.cuda.synchronize()
    ref2 = evict(q, k, v, 256, reserved_recent=16, pool_kernel=5, recency_decay=0.05)
    for a, b in zip(out, ref2):
        assert torch.equal(a, b)
