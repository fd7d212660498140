"""GPU: determinism, layouts, the C ABI called directly, the watchdog path,
and parity at the BASELINE configurations (full sizes, sampled oracle rows
plus size-independent properties)."""
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


# --------------------------------------------------------- BASELINE configs --

def _gen(shape, seed, dtype, scale=1.0):
    g = torch.Generator().manual_seed(seed)
    return (torch.randn(shape, generator=g) * scale).to(dtype)


def _check_config(q, k, v, budget, sample_rows, out_tol, imp_rtol, imp_atol, **kw):
    causal = kw.pop("causal", True)
    pool = kw.pop("pool_kernel", 1)
    recent = kw.pop("reserved_recent", 0)
    out, imp, idx, mask = evict(q, k, v, budget, causal=causal, pool_kernel=pool, reserved_recent=recent, **kw)
    torch.cuda.synchronize()
    n = q.shape[2]
    ref_out, ref_imp = O.chunked(q.cpu(), k.cpu(), v.cpu(), causal=causal, out_rows=sample_rows,
                                 recency_decay=kw.get("recency_decay", 0.0),
                                 observation_window=kw.get("observation_window", 0),
                                 value_weighted=kw.get("value_weighted", True), weight_floor=1e-30)
    got = out[:, :, sample_rows].float().cpu().numpy()
    np.testing.assert_allclose(got, ref_out[:, :, sample_rows], atol=out_tol, rtol=0.006)
    np.testing.assert_allclose(imp.cpu().numpy(), ref_imp, atol=imp_atol, rtol=imp_rtol)
    ref_idx, ref_keep = O.select_tokens(ref_imp, budget, reserved_recent=recent, pool_kernel=pool)
    from common import selection_mismatch
    mism, ok = selection_mismatch(~mask.cpu().numpy(), ref_keep, imp.cpu().numpy(), ref_imp, imp_atol, imp_rtol)
    assert ok, mism
    assert (~mask).sum(-1).eq(budget).all()
    return mism


def test_config2_llama_8k():
    # B1 Hq32 Hkv8 N8192 D128 bf16 causal, q,k ~ N(0,1)/D^0.25, decay 0.1, reserved 64, budget 1024
    n, d = 8192, 128
    q = (_gen((1, 32, n, d), 0, torch.float32) / d ** 0.25).to(torch.bfloat16).cuda()
    k = (_gen((1, 8, n, d), 1, torch.float32) / d ** 0.25).to(torch.bfloat16).cuda()
    v = _gen((1, 8, n, d), 2, torch.bfloat16).cuda()
    rows = np.unique(np.r_[0, 1, 127, 128, 4095, n - 1, np.random.default_rng(0).integers(0, n, 24)])
    _check_config(q, k, v, 1024, rows, 0.012, 1e-4, 1e-6, recency_decay=0.1, reserved_recent=64)


def test_config3_qwen_32k():
    # B1 Hq28 Hkv4 N32768 D128 fp16 causal, 1% of k rows x8, window 128, pool 5, budget 2048
    n, d = 32768, 128
    q = _gen((1, 28, n, d), 0, torch.float16).cuda()
    k = _gen((1, 4, n, d), 1, torch.float32)
    sink = torch.randperm(n, generator=torch.Generator().manual_seed(3))[: n // 100]
    k[:, :, sink] *= 8
    k = k.to(torch.float16).cuda()
    v = _gen((1, 4, n, d), 2, torch.float16).cuda()
    rows = np.unique(np.r_[0, 255, 256, n - 129, n - 1, np.random.default_rng(1).integers(0, n, 12)])
    _check_config(q, k, v, 2048, rows, 0.002, 3e-4, 3e-3, observation_window=128, pool_kernel=5)


def test_config5_batched_mha_noncausal_h2o_sampled():
    # B8 Hq=Hkv=32 N4096 D128 fp16 noncausal, [B,N,H,D] strides, q x30, 5% zero v rows, H2O, budget 410
    b, h, n, d = 8, 32, 4096, 128
    q = (_gen((b, n, h, d), 0, torch.float32) * 30).to(torch.float16).cuda().transpose(1, 2)
    k = _gen((b, n, h, d), 1, torch.float16).cuda().transpose(1, 2)
    v = _gen((b, n, h, d), 2, torch.float32)
    zero = torch.randperm(n, generator=torch.Generator().manual_seed(4))[: n * 5 // 100]
    v[:, zero] = 0
    v = v.to(torch.float16).cuda().transpose(1, 2)
    out, imp, idx, mask = evict(q, k, v, 410, causal=False, value_weighted=False)
    torch.cuda.synchronize()
    # size-independent: H2O mass of each (b, h) sums to N (noncausal softmax rows sum to 1)
    torch.testing.assert_close(imp.double().sum(-1), torch.full((b, h), float(n), dtype=torch.float64,
                                                                device="cuda"), rtol=1e-5, atol=1e-3)
    # exact oracle on a few (b, h) units
    for bi, hi in ((0, 0), (3, 17), (7, 31)):
        sl = slice(hi, hi + 1)
        rows = np.r_[0, 1, 2047, n - 1]
        ro, ri = O.chunked(q[bi:bi + 1, sl].cpu(), k[bi:bi + 1, sl].cpu(), v[bi:bi + 1, sl].cpu(), causal=False,
                           value_weighted=False, out_rows=rows)
        np.testing.assert_allclose(out[bi, hi, rows].float().cpu().numpy(), ro[0, 0, rows], atol=0.004, rtol=0.006)
        np.testing.assert_allclose(imp[bi, hi].cpu().numpy(), ri[0, 0], atol=1e-3, rtol=1e-3)
    assert (~mask).sum(-1).eq(410).all()


def test_exp2_polynomial_error_bound():
    """The FMA-pipe exp2 used for part of the softmax: relative error within
    the fitted bound (2.7e-6) of float64 exp2 over the softmax's input range,
    exact zero below -125 and for -inf; the MUFU path within 2^-21."""
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
    assert torch.all(poly[~main] == 0)
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
