"""KV compaction on the GPU: gather_tokens against torch.gather (the README.md:31
expression) and the oracle, the fused selection+gather launch against
select_tokens followed by the gather, and evict_compact against evict.
All comparisons are bitwise."""
import ctypes

import numpy as np
import pytest
import torch

from flash_evict import _lib, evict, evict_compact, gather_tokens, select_and_gather, select_tokens
from oracle import restate as O

pytestmark = pytest.mark.gpu


def torch_gather(x, idx):
    return x.gather(2, idx[..., None].expand(-1, -1, -1, x.shape[-1]))


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16, torch.float32, torch.int8])
@pytest.mark.parametrize("d", [128, 64, 37, 1])
def test_gather_matches_torch_gather(dtype, d):
    g = torch.Generator().manual_seed(d)
    x = (torch.randn(2, 3, 300, d, generator=g) * 50).to(dtype).cuda()
    idx = torch.randint(0, 300, (2, 3, 77), generator=g).cuda()  # unsorted, repeats
    got = gather_tokens(x, idx)
    assert got.is_contiguous() and got.shape == (2, 3, 77, d)
    assert torch.equal(got, torch_gather(x, idx))


def test_gather_strided_views_and_oracle():
    g = torch.Generator().manual_seed(1)
    base = torch.randn(2, 1000, 4, 128, generator=g).to(torch.bfloat16).cuda()
    x = base.transpose(1, 2)  # [B, H, N, D] view of a [B, N, H, D] buffer, no copy
    idx = torch.sort(torch.randint(0, 1000, (2, 4, 100), generator=g), -1).values.cuda()
    got = gather_tokens(x, idx)
    assert torch.equal(got, torch_gather(x, idx))
    ref = O.gather_tokens(x.float().cpu().numpy(), idx.cpu().numpy())
    np.testing.assert_array_equal(got.float().cpu().numpy(), ref)
    # channel stride != 1 is copied once by the wrapper
    xt = torch.randn(1, 2, 64, 50, generator=g).cuda().transpose(2, 3)
    idx2 = torch.randint(0, 50, (1, 2, 9), generator=g).cuda()
    assert torch.equal(gather_tokens(xt, idx2), torch_gather(xt, idx2))


@pytest.mark.parametrize("budget", [0, 1, 31, 32, 33, 4096])
def test_gather_budget_edges(budget):
    x = torch.randn(1, 2, 5000, 128, device="cuda", dtype=torch.float16)
    idx = torch.randint(0, 5000, (1, 2, budget), device="cuda")
    assert torch.equal(gather_tokens(x, idx), torch_gather(x, idx))


def test_gather_out_of_range_index_zero_fills_and_reports():
    dev = torch.cuda.current_device()
    _lib.device_status(dev, clear=True)
    x = torch.randn(1, 1, 10, 64, device="cuda", dtype=torch.bfloat16)
    idx = torch.tensor([[[0, 10, 3, -1, 9]]], device="cuda")
    got = gather_tokens(x, idx)
    assert _lib.device_status(dev, clear=True) == _lib.STATUS_BAD_INDEX
    assert torch.equal(got[0, 0, [0, 2, 4]], x[0, 0, [0, 3, 9]])
    assert not got[0, 0, [1, 3]].any()


CASES = [  # (rows as (B, H), N, D, budget, recent, pool)
    ((1, 4), 32768, 128, 2048, 0, 5),
    ((1, 8), 8192, 128, 1024, 64, 1),
    ((2, 3), 137, 64, 48, 32, 5),
    ((1, 2), 1000, 128, 64, 64, 1),      # budget == recent: only the suffix is kept
    ((1, 1), 500, 128, 500, 0, 1),       # budget == N
    ((1, 2), 200000, 128, 1024, 16, 1),  # large cluster
    ((4, 2), 3000, 80, 300, 7, 3),       # 160-byte rows
    ((1, 2), 5000, 256, 500, 16, 5),     # 512-byte rows
]


@pytest.mark.parametrize("case", CASES)
def test_select_and_gather_equals_select_then_gather(case):
    (b, h), n, d, budget, recent, pool = case
    g = torch.Generator().manual_seed(n + d)
    scores = torch.rand(b, h, n, generator=g).cuda()
    scores[..., ::97] = scores[..., 5:6]  # ties
    kbuf = torch.randn(b, n, h, d, generator=g).to(torch.bfloat16).cuda()
    k = kbuf.transpose(1, 2)
    v = torch.randn(b, h, n, d, generator=g).to(torch.bfloat16).cuda()
    idx, keep, kk, vk = select_and_gather(scores, budget, k, v, reserved_recent=recent, pool_kernel=pool)
    ref_idx, ref_keep = select_tokens(scores, budget, reserved_recent=recent, pool_kernel=pool)
    assert torch.equal(idx, ref_idx) and torch.equal(keep, ref_keep)
    assert torch.equal(kk, torch_gather(k, idx)) and torch.equal(vk, torch_gather(v, idx))
    if n <= 40000:
        o_idx, _ = O.select_tokens(scores.cpu().numpy(), budget, reserved_recent=recent, pool_kernel=pool)
        np.testing.assert_array_equal(idx.cpu().numpy(), o_idx)


def test_evict_compact_equals_evict_then_gather():
    g = torch.Generator().manual_seed(11)
    q = torch.randn(1, 8, 3000, 128, generator=g).to(torch.float16).cuda()
    k = torch.randn(1, 2, 3000, 128, generator=g).to(torch.float16).cuda()
    v = torch.randn(1, 2, 3000, 128, generator=g).to(torch.float16).cuda()
    kw = dict(reserved_recent=16, pool_kernel=5, recency_decay=0.01)
    out, imp, idx, mask, kk, vk = evict_compact(q, k, v, 300, **kw)
    r = evict(q, k, v, 300, **kw)
    for a, b_ in zip((out, imp, idx, mask), r):
        assert torch.equal(a, b_)
    assert torch.equal(kk, torch_gather(k, idx)) and torch.equal(vk, torch_gather(v, idx))


def test_c_abi_evict_compact_direct():
    lib = _lib.load()
    g = torch.Generator().manual_seed(12)
    b, hq, hk, n, d, budget = 1, 4, 2, 700, 64, 100
    q = torch.randn(b, hq, n, d, generator=g).to(torch.bfloat16).cuda()
    k = torch.randn(b, hk, n, d, generator=g).to(torch.bfloat16).cuda()
    v = torch.randn(b, hk, n, d, generator=g).to(torch.bfloat16).cuda()
    out = torch.empty_like(q)
    imp = torch.empty(b, hk, n, device="cuda")
    idx = torch.empty(b, hk, budget, dtype=torch.int64, device="cuda")
    mask = torch.empty(b, hk, n, dtype=torch.bool, device="cuda")
    kk = torch.empty(b, hk, budget, d, dtype=k.dtype, device="cuda")
    vk = torch.empty_like(kk)
    stats = torch.empty(b, hq, n, 2, device="cuda")
    s = torch.cuda.current_stream().cuda_stream
    rc = lib.fe_evict_compact(q.data_ptr(), _lib.strides(q), k.data_ptr(), _lib.strides(k), v.data_ptr(),
                              _lib.strides(v), out.data_ptr(), imp.data_ptr(), idx.data_ptr(), mask.data_ptr(),
                              kk.data_ptr(), vk.data_ptr(), stats.data_ptr(), b, hq, hk, n, d, _lib.DTYPE_BF16, 1,
                              ctypes.c_float(d ** -0.5), 0.0, 0, 1, budget, 8, 1, s)
    _lib.check(rc)
    r = evict(q, k, v, budget, reserved_recent=8)
    assert torch.equal(idx, r[2]) and torch.equal(mask, r[3])
    assert torch.equal(kk, torch_gather(k, idx)) and torch.equal(vk, torch_gather(v, idx))
