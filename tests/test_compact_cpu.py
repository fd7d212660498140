"""KV compaction: the oracle against the gather the reference documents
(README.md:31), and the host-side argument contract of flash_evict.compact
(CPU only; the kernels are exercised in test_gpu_compact.py)."""
import numpy as np
import pytest
import torch

from flash_evict import evict_compact, gather_tokens, select_and_gather
from oracle import restate


@pytest.mark.parametrize("dtype", [torch.float32, torch.float16, torch.bfloat16, torch.int8])
def test_oracle_gather_matches_readme_expression(dtype):
    g = torch.Generator().manual_seed(3)
    k = (torch.randn(2, 3, 50, 24, generator=g) * 20).to(dtype)
    idx = torch.randint(0, 50, (2, 3, 17), generator=g)
    ref = k.gather(2, idx[..., None].expand(-1, -1, -1, k.shape[-1]))  # README.md:31
    src = k.float().numpy() if dtype == torch.bfloat16 else k.numpy()
    got = restate.gather_tokens(src, idx.numpy())
    np.testing.assert_array_equal(got, ref.float().numpy() if dtype == torch.bfloat16 else ref.numpy())


def test_oracle_gather_after_selection_is_the_kept_rows():
    g = torch.Generator().manual_seed(4)
    scores = torch.rand(1, 2, 40, generator=g)
    k = torch.randn(1, 2, 40, 8, generator=g)
    idx, keep = restate.select_tokens(scores.numpy(), 10, recent=3)
    kept = restate.gather_tokens(k.numpy(), idx)
    for h in range(2):
        np.testing.assert_array_equal(kept[0, h], k.numpy()[0, h][keep[0, h]])


def test_gather_argument_errors():
    x = torch.zeros(1, 2, 8, 16, dtype=torch.float16)
    idx = torch.zeros(1, 2, 4, dtype=torch.int64)
    with pytest.raises(ValueError, match="CUDA"):
        gather_tokens(x, idx)
    with pytest.raises(ValueError, match="shape"):
        gather_tokens(x[0], idx)
    scores = torch.zeros(1, 2, 8)
    with pytest.raises(ValueError, match="CUDA"):
        select_and_gather(scores, 4, x, x)
    with pytest.raises(ValueError, match="same shape"):
        select_and_gather(scores, 4, x, x[:, :1])


def test_evict_compact_keeps_the_evict_contract():
    q = torch.zeros(1, 1, 4, 16, dtype=torch.float16)
    with pytest.raises(ValueError, match="scoring"):
        evict_compact(q, q, q, 2, score=False)
    with pytest.raises(ValueError, match="CUDA"):
        evict_compact(q, q, q, 2)


def test_multi_policy_argument_errors():
    from flash_evict.policies import select_tokens_multi, select_and_gather_multi
    s = torch.zeros(1, 2, 50)
    with pytest.raises(ValueError, match="CUDA"):
        select_tokens_multi(s, [10, 20])
    with pytest.raises(ValueError, match="policies"):
        select_tokens_multi(s, list(range(1, 10)))
    with pytest.raises(ValueError, match="same shape"):
        select_tokens_multi([s, torch.zeros(1, 2, 40)], [10, 20])
    with pytest.raises(ValueError, match="one entry per policy"):
        select_tokens_multi(s, [10, 20], recents=[1, 2, 3])
    with pytest.raises(ValueError, match="budget"):
        select_tokens_multi(s, [10, 60])
    with pytest.raises(ValueError, match="recent"):
        select_tokens_multi(s, [10, 20], recents=[11, 0])
    k = torch.zeros(1, 2, 50, 8)
    with pytest.raises(ValueError, match="CUDA"):
        select_and_gather_multi(s, [10], k, k)
