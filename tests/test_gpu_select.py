"""GPU selection kernel against the oracle (exact, stated tie-break) and the
reference's selection fixtures (tests/golden/selection.npz)."""
import os

import numpy as np
import pytest
import torch

from common import GOLDEN
from flash_evict import select_tokens
from flash_evict.prefill import _select
from oracle import restate as O

pytestmark = pytest.mark.gpu


def check_exact(scores, budget, recent=0, pool=1):
    idx, keep = select_tokens(scores, budget, reserved_recent=recent, pool_kernel=pool)
    ref_idx, ref_keep = O.select_tokens(scores.float().cpu().numpy(), budget, reserved_recent=recent,
                                        pool_kernel=pool)
    np.testing.assert_array_equal(idx.cpu().numpy(), ref_idx)
    np.testing.assert_array_equal(keep.cpu().numpy(), ref_keep)
    _, evict_mask = _select(scores, budget, recent, pool, evict_mask=True)
    assert torch.equal(evict_mask, ~keep)
    return idx, keep


def test_reference_selection_fixtures():
    z = np.load(os.path.join(GOLDEN, "selection.npz"))
    s = torch.from_numpy(z["pin_scores"]).cuda()
    idx, keep = select_tokens(s, 48, reserved_recent=32, pool_kernel=5)
    np.testing.assert_array_equal(idx.cpu().numpy(), z["pin_idx"])
    np.testing.assert_array_equal(keep.cpu().numpy(), z["pin_keep"])
    for j in range(int(z["ncases"])):
        bud, rec, pk = (int(x) for x in z[f"c{j}_args"])
        idx, keep = select_tokens(torch.from_numpy(z[f"c{j}_scores"]).cuda(), bud, reserved_recent=rec,
                                  pool_kernel=pk)
        np.testing.assert_array_equal(idx.cpu().numpy(), z[f"c{j}_idx"])
        np.testing.assert_array_equal(keep.cpu().numpy(), z[f"c{j}_keep"])


def test_selection_contract():
    # reference tests/test_prefill.py:77-81
    scores = torch.arange(20.).reshape(1, 1, 20).cuda()
    idx, keep = select_tokens(scores, 4, recent=2)
    assert idx.tolist() == [[[16, 17, 18, 19]]]
    assert keep.sum() == 4


def test_pinning_and_pooling_contract():
    # reference tests/test_prefill.py:149-157 (snap_select equivalence is in the fixture)
    torch.manual_seed(1)
    scores = torch.randn(1, 3, 137).cuda()
    _, tail = select_tokens(scores, 64, reserved_recent=64, pool_kernel=5)
    assert tail.sum() == 3 * 64 and tail[..., -64:].all()
    check_exact(scores, 48, 32, 5)


@pytest.mark.parametrize("rows,n", [(1, 1), (3, 7), (4, 1000), (256, 4096), (4, 32768), (8, 131072), (2, 200000)])
@pytest.mark.parametrize("pool", [1, 5])
def test_random_vs_oracle(rows, n, pool):
    g = torch.Generator().manual_seed(rows * 7 + n + pool)
    s = torch.rand((rows, n), generator=g).cuda()
    for budget, recent in {(1, 0), (max(1, n // 10), 0), (max(1, n // 10), min(64, n // 10)), (n, 0), (n, n)}:
        check_exact(s, budget, recent, pool)


@pytest.mark.parametrize("n", [786432, 786433, 1000000, 3000000])
@pytest.mark.parametrize("pool", [1, 5])
def test_rows_longer_than_shared_memory(n, pool):
    # past regions above 16 x 49152 keys run the kernel variant that
    # recomputes each key from the scores on every pass (no length limit)
    g = torch.Generator().manual_seed(n + pool)
    s = torch.rand((2, n), generator=g)
    s[:, ::1000] = s[:, 7:8]  # ties across the row
    s = s.cuda()
    for budget, recent in ((4096, 0), (n // 10, 64)):
        check_exact(s, budget, recent, pool)


@pytest.mark.parametrize("n", [100, 5000, 70000])
def test_ties_lower_index_wins(n):
    g = torch.Generator().manual_seed(n)
    s = torch.randint(0, 5, (3, n), generator=g).float().cuda()
    for budget in (1, n // 7, n // 2, n - 1):
        check_exact(s, budget)
        check_exact(s, budget, pool=3)


def test_special_values():
    s = torch.tensor([[0.0, -0.0, float("nan"), 1.0, float("inf"), -float("inf"), 2.0, -0.0, 0.0, 3.0]]).cuda()
    for budget in range(1, 11):
        check_exact(s, budget)
    z = torch.zeros(2, 3000).cuda()
    z[:, ::2] = -0.0
    check_exact(z, 1000)


def test_batched_shape_and_dtypes():
    s = torch.rand(2, 3, 500).cuda()
    idx, keep = select_tokens(s, 50)
    assert idx.shape == (2, 3, 50) and idx.dtype == torch.int64
    assert keep.shape == s.shape and keep.dtype == torch.bool
    assert (idx.diff(dim=-1) > 0).all()
    idx16, _ = select_tokens(s.half(), 50)
    ref, _ = O.select_tokens(s.half().float().cpu().numpy(), 50)
    np.testing.assert_array_equal(idx16.cpu().numpy(), ref)
