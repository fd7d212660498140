"""Host logic of the multi-GPU layer on CPU ranks (gloo, world size 2).

The query-sharded pipeline (flash_evict.distributed._query_sharded) runs
with the oracle standing in for the per-rank CUDA compute, so the partition,
the all-reduce of partial scores, the row all-gather and the per-rank
selection are checked without a GPU.  A rank that fails before the
collective must make its peer's collective fail on the process-group
timeout, not hang.
"""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from flash_evict.distributed import (BLOCK, _block_cost, _query_sharded, first_scored_row, head_blocks, head_unit_plan,
                                     key_tile_plan, query_block_plan)
from oracle import restate as O

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


@pytest.mark.parametrize("n,world,causal", [(131072, 8, True), (131072, 3, True), (32768, 2, True),
                                            (4096, 4, False), (300, 2, True), (100, 4, True)])
def test_query_block_plan_partitions_and_balances(n, world, causal):
    plan = query_block_plan(n, world, causal)
    nblk = (n + BLOCK - 1) // BLOCK
    flat = sorted(b for p in plan for b in p)
    assert flat == list(range(nblk))
    costs = [sum(_block_cost(b, n, causal) for b in p) for p in plan]
    max_block = max(_block_cost(b, n, causal) for b in range(nblk))
    assert max(costs) - min(costs) <= max_block
    for p in plan:
        c = [_block_cost(b, n, causal) for b in p]
        assert c == sorted(c, reverse=True)


@pytest.mark.parametrize("batch,heads,world", [(8, 32, 8), (8, 32, 3), (1, 8, 8), (2, 3, 4)])
def test_head_unit_plan_covers_units(batch, heads, world):
    plan = head_unit_plan(batch, heads, world)
    units = [(b, h) for runs in plan for (b, h0, h1) in runs for h in range(h0, h1)]
    assert sorted(units) == [(b, h) for b in range(batch) for h in range(heads)]
    sizes = [sum(h1 - h0 for _, h0, h1 in runs) for runs in plan]
    assert max(sizes) - min(sizes) <= 1


@pytest.mark.parametrize("batch,heads,world", [(8, 32, 8), (8, 32, 2), (8, 32, 3), (1, 8, 8), (2, 3, 4), (5, 4, 2)])
def test_head_blocks_merge_whole_batches(batch, heads, world):
    blocks = head_blocks(batch, heads, world)
    units = [(b, h) for bl in blocks for (b0, b1, h0, h1) in bl for b in range(b0, b1) for h in range(h0, h1)]
    assert sorted(units) == [(b, h) for b in range(batch) for h in range(heads)]
    for bl in blocks:
        for b0, b1, h0, h1 in bl:
            assert b1 > b0 and h1 > h0
            assert b1 - b0 == 1 or (h0 == 0 and h1 == heads)   # several batches only when whole
        whole = [x for x in bl if x[2] == 0 and x[3] == heads]
        assert all(a[1] != c[0] for a, c in zip(whole, whole[1:]))  # no two adjacent whole blocks left unmerged
    if world == 2 and batch == 8:
        assert blocks == [[(0, 4, 0, heads)], [(4, 8, 0, heads)]]


def _oracle_attend(q, k, v, blocks, causal, scale):
    """Attention rows of the given query blocks and their softmax statistics
    {m (log2 units), l}, computed in numpy (float64); other rows zero."""
    qn, kn, vn = (t.double().numpy() for t in (q, k, v))
    b, h, n, d = qn.shape
    g = h // kn.shape[1]
    out = np.zeros(qn.shape)
    stats = np.zeros((b, h, n, 2))
    rows = [r for blk in blocks for r in range(blk * BLOCK, min(n, (blk + 1) * BLOCK))]
    for bi in range(b):
        for hi in range(h):
            for r in rows:
                x = (kn[bi, hi // g] @ qn[bi, hi, r]) * scale * np.log2(np.e)
                if causal:
                    x[r + 1:] = -np.inf
                m = x.max()
                p = np.exp2(x - m)
                stats[bi, hi, r] = (m, p.sum())
                out[bi, hi, r] = p @ vn[bi, hi // g] / p.sum()
    return torch.from_numpy(out).float(), torch.from_numpy(stats).float()


def _oracle_replay(q, k, v, row_stats, key_tiles, causal, scale, decay, window, weighted):
    """Importance of keys in the given key tiles from every scored row, using
    the exchanged statistics (the replay of prefill.py:61-83); zeros elsewhere."""
    qn, kn, vn = (t.double().numpy() for t in (q, k, v))
    st = row_stats.double().numpy()
    b, h, n, d = qn.shape
    hk = kn.shape[1]
    g = h // hk
    imp = np.zeros((b, hk, n))
    k0, k1 = key_tiles[0] * 128, min(n, key_tiles[1] * 128)
    w = O.recency_weights(n, decay, window, np.float64)
    for r in range(first_scored_row(n, decay, window), n):
        for bi in range(b):
            for hi in range(h):
                x = (kn[bi, hi // g, k0:k1] @ qn[bi, hi, r]) * scale * np.log2(np.e)
                if causal:
                    x[np.arange(k0, k1) > r] = -np.inf
                imp[bi, hi // g, k0:k1] += w[r] * np.exp2(x - st[bi, hi, r, 0]) / st[bi, hi, r, 1]
    if weighted:
        imp *= np.abs(vn).sum(-1)
    return torch.from_numpy(imp).float()


def _oracle_select(importance, budget, recent, pool):
    idx, keep = O.select_tokens(importance.numpy(), budget, reserved_recent=recent, pool_kernel=pool)
    return torch.from_numpy(idx), torch.from_numpy(~keep)


def _worker(rank, world, port, result_dir, mode, decay=0.01, window=0):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    import datetime
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=8))
    g = torch.Generator().manual_seed(0)
    n, h, hk, d = 700, 4, 2, 32
    q = torch.randn(1, h, n, d, generator=g)
    k = torch.randn(1, hk, n, d, generator=g)
    v = torch.randn(1, hk, n, d, generator=g)
    try:
        if mode == "fail" and rank == 1:
            raise RuntimeError("injected failure before the score all-reduce")
        out, imp, idx, mask, blocks = _query_sharded(
            q, k, v, 64, 8, 5, True, d ** -0.5, decay, window, True, True, None, _oracle_attend, _oracle_replay,
            _oracle_select)
        np.savez(os.path.join(result_dir, f"r{rank}.npz"), out=out.numpy(), imp=imp.numpy(), idx=idx.numpy(),
                 mask=mask.numpy(), blocks=np.array(blocks))
    except Exception as e:  # noqa: BLE001
        with open(os.path.join(result_dir, f"r{rank}.err"), "w") as f:
            f.write(type(e).__name__ + ": " + str(e))
    finally:
        try:
            dist.destroy_process_group()
        except Exception:  # noqa: BLE001
            pass


def _spawn(mode, tmp_path, world=2, decay=0.01, window=0):
    port = _free_port()
    ctx = mp.get_context("spawn")
    procs = [ctx.Process(target=_worker, args=(r, world, port, str(tmp_path), mode, decay, window))
             for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(60)
        if p.is_alive():
            p.kill()
            pytest.fail("rank did not finish")


def test_query_sharded_pipeline_gloo(tmp_path):
    _spawn("ok", tmp_path)
    r0 = np.load(tmp_path / "r0.npz")
    r1 = np.load(tmp_path / "r1.npz")
    g = torch.Generator().manual_seed(0)
    n, h, hk, d = 700, 4, 2, 32
    q = torch.randn(1, h, n, d, generator=g)
    k = torch.randn(1, hk, n, d, generator=g)
    v = torch.randn(1, hk, n, d, generator=g)
    ref_out, ref_imp = O.chunked(q, k, v, recency_decay=0.01)
    np.testing.assert_allclose(r0["imp"], ref_imp, rtol=1e-5, atol=1e-6)
    np.testing.assert_array_equal(r0["imp"], r1["imp"])
    np.testing.assert_allclose(r0["out"], ref_out, rtol=1e-5, atol=1e-6)
    np.testing.assert_array_equal(r0["idx"], r1["idx"])
    ref_idx, ref_keep = O.select_tokens(ref_imp, 64, reserved_recent=8, pool_kernel=5)
    np.testing.assert_array_equal(r0["idx"], ref_idx)
    assert sorted(np.r_[r0["blocks"], r1["blocks"]].tolist()) == list(range((n + BLOCK - 1) // BLOCK))


@pytest.mark.parametrize("world,decay,window", [(3, 0.0, 300), (4, 0.05, 0)])
def test_query_sharded_more_ranks_than_blocks_gloo(tmp_path, world, decay, window):
    # 700 tokens = 3 query blocks and 6 key tiles: with 4 ranks one rank owns
    # no query block (its rows contribute nothing to the exchanges); the
    # window starts inside a block
    _spawn("ok", tmp_path, world, decay, window)
    g = torch.Generator().manual_seed(0)
    n, h, hk, d = 700, 4, 2, 32
    q = torch.randn(1, h, n, d, generator=g)
    k = torch.randn(1, hk, n, d, generator=g)
    v = torch.randn(1, hk, n, d, generator=g)
    ref_out, ref_imp = O.chunked(q, k, v, recency_decay=decay, observation_window=window)
    res = [np.load(tmp_path / f"r{r}.npz") for r in range(world)]
    for r in res:
        np.testing.assert_allclose(r["imp"], ref_imp, rtol=1e-5, atol=1e-6)
        np.testing.assert_array_equal(r["idx"], res[0]["idx"])
    np.testing.assert_allclose(res[0]["out"], ref_out, rtol=1e-5, atol=1e-6)
    blocks = sorted(b for r in res for b in r["blocks"].tolist())
    assert blocks == list(range((n + BLOCK - 1) // BLOCK))


def test_failed_rank_surfaces_as_error_not_hang(tmp_path):
    _spawn("fail", tmp_path)
    assert (tmp_path / "r1.err").exists()
    err0 = tmp_path / "r0.err"
    assert err0.exists(), "surviving rank should see its collective fail"


@pytest.mark.parametrize("n,world", [(1, 1), (700, 2), (131072, 8), (300, 4)])
def test_key_tile_plan_covers_all_tiles(n, world):
    plan = key_tile_plan(n, world)
    nkt = (n + 127) // 128
    assert plan[0][0] == 0 and plan[-1][1] == nkt
    for (a, b), (c, _) in zip(plan, plan[1:]):
        assert b == c and a <= b
    assert max(b - a for a, b in plan) - min(b - a for a, b in plan) <= 1


def test_first_scored_row_matches_oracle():
    # The last five decays round to FP32 across an integer reach: a cut computed
    # from the double decay would differ by one row from the kernel's.
    for n, decay, window in [(700, 0.0, 0), (700, 0.01, 0), (131072, 0.1, 0), (8192, 0.0, 128), (100, 0.0, 500),
                             (32768, 0.05, 4096), (65536, 0.008793296665318385, 0), (8192, 0.0675592410264192, 0),
                             (8192, 0.1343964723079836, 0), (65536, 0.0035870458270285334, 0),
                             (4096, 0.15552949112389214, 0)]:
        assert first_scored_row(n, decay, window) == int(O.scored_rows(n, decay, window)[0]), (n, decay)
