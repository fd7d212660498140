"""Several selection policies in one launch (flash_evict.policies) against
one select_tokens / snap_select call per policy, as the reference's paired
controller runs them (flash_evict/quality_adapter.py:39-51, 95-111): indices
and masks exactly equal, compacted K/V bitwise equal to torch.gather."""
import numpy as np
import pytest
import torch

from flash_evict import evict, select_tokens
from flash_evict.baselines import snap_scores, snap_select
from flash_evict.policies import select_and_gather_multi, select_tokens_multi
from oracle import restate as O

pytestmark = pytest.mark.gpu


def torch_gather(x, idx):
    return x.gather(2, idx[..., None].expand(-1, -1, -1, x.shape[-1]))


def test_paired_controller_methods_in_one_launch():
    # the default methods of quality_adapter.py:18-29 that select (budgets 256
    # and 1024): fused importance with reserved 0/64, SnapKV, value norm,
    # uniform recent (a suffix of `budget` = select with recent=budget)
    g = torch.Generator().manual_seed(21)
    n = 3000
    q = torch.randn(1, 28, n, 128, generator=g).to(torch.bfloat16).cuda()
    k = torch.randn(1, 4, n, 128, generator=g).to(torch.bfloat16).cuda()
    v = torch.randn(1, 4, n, 128, generator=g).to(torch.bfloat16).cuda()
    imp = evict(q, k, v, 256, recency_decay=0.1, observation_window=128)[1]
    snap = snap_scores(q, k, 32)
    vnorm = v.float().abs().sum(-1)
    pols = [(imp, 256, 0, 1), (imp, 256, 64, 1), (imp, 1024, 64, 1), (snap, 256, 32, 5), (snap, 1024, 32, 5),
            (vnorm, 256, 0, 1), (imp, 256, 256, 1)]
    res = select_and_gather_multi([p[0] for p in pols], [p[1] for p in pols], k, v, recents=[p[2] for p in pols],
                                  pool_kernels=[p[3] for p in pols])
    for (s, bud, rec, pool), (idx, keep, kk, vk) in zip(pols, res):
        ridx, rkeep = select_tokens(s, bud, reserved_recent=rec, pool_kernel=pool)
        assert torch.equal(idx, ridx) and torch.equal(keep, rkeep)
        assert torch.equal(kk, torch_gather(k, idx)) and torch.equal(vk, torch_gather(v, idx))
    # the snap policies equal the reference-shaped snap_select
    assert torch.equal(res[3][0], snap_select(snap, 256, 32, 5)[0])
    # uniform_recent: the last `budget` tokens
    assert torch.equal(res[6][0][0, 0], torch.arange(n - 256, n).cuda())


@pytest.mark.parametrize("n", [137, 40000, 150000])
def test_multi_policy_matches_oracle(n):
    g = torch.Generator().manual_seed(n)
    s = torch.rand(2, 3, n, generator=g)
    s[..., ::7] = s[..., 3:4]  # ties
    budgets = [1, n // 10 + 1, n // 2, n]
    recents = [0, min(16, n // 10), n // 2 - 1, n // 3]
    pools = [1, 5, 3, 1]
    res = select_tokens_multi(s.cuda(), budgets, recents, pools)
    for (idx, keep), b, r, p in zip(res, budgets, recents, pools):
        ridx, rkeep = O.select_tokens(s.numpy(), b, reserved_recent=r, pool_kernel=p)
        np.testing.assert_array_equal(idx.cpu().numpy(), ridx)
        np.testing.assert_array_equal(keep.cpu().numpy(), rkeep)


def test_eight_policies_shared_scores():
    s = torch.rand(1, 8, 32768, device="cuda")
    budgets = [64, 128, 256, 512, 1024, 2048, 4096, 8192]
    res = select_tokens_multi(s, budgets, recents=32, pool_kernels=5)
    for (idx, keep), b in zip(res, budgets):
        ridx, rkeep = select_tokens(s, b, reserved_recent=32, pool_kernel=5)
        assert torch.equal(idx, ridx) and torch.equal(keep, rkeep)
