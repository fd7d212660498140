"""Multi-GPU evict, checked against single-GPU evict on the same inputs
(bitwise: outputs, importance, selection).

The NCCL test (one process per GPU) runs only when at least two GPUs are
visible.  The thread-rank tests run the same sharded entry points with the
ranks as threads on one GPU and the two collectives done by torch ops, so the
per-rank work split (query blocks, key-tile ranges, statistics exchange,
score reduction) is checked on any GPU box, c4 at its full size included."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _worker(rank, world, port, out_dir):
    import datetime
    import torch.distributed as dist
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=dev)
    try:
        from flash_evict import evict
        from flash_evict.distributed import evict_head_sharded, evict_query_sharded
        g = torch.Generator().manual_seed(5)
        q = torch.randn(1, 8, 3000, 128, generator=g).to(torch.bfloat16).to(dev)
        k = torch.randn(1, 2, 3000, 128, generator=g).to(torch.bfloat16).to(dev)
        v = torch.randn(1, 2, 3000, 128, generator=g).to(torch.bfloat16).to(dev)
        out, imp, idx, mask, blocks = evict_query_sharded(q, k, v, 300, reserved_recent=16, recency_decay=0.01,
                                                          gather_output=True)
        ref = evict(q, k, v, 300, reserved_recent=16, recency_decay=0.01)
        qb = torch.randn(4, 3000, 4, 64, generator=g).to(torch.float16).to(dev).transpose(1, 2)
        kb = torch.randn(4, 4, 3000, 64, generator=g).to(torch.float16).to(dev)
        vb = torch.randn(4, 4, 3000, 64, generator=g).to(torch.float16).to(dev)
        runs = evict_head_sharded(qb, kb, vb, 256, causal=False, value_weighted=False)
        refb = evict(qb, kb, vb, 256, causal=False, value_weighted=False)
        head_ok = True
        for b0, b1, h0, h1, o, i, ix, m in runs:
            head_ok &= torch.equal(o, refb[0][b0:b1, h0:h1]) and torch.equal(i, refb[1][b0:b1, h0:h1])
            head_ok &= torch.equal(ix, refb[2][b0:b1, h0:h1]) and torch.equal(m, refb[3][b0:b1, h0:h1])
        torch.cuda.synchronize()
        np.savez(os.path.join(out_dir, f"r{rank}.npz"), out_equal=torch.equal(out, ref[0]),
                 imp_equal=torch.equal(imp, ref[1]),
                 imp_err=(imp - ref[1]).abs().max().item(), imp_max=ref[1].abs().max().item(),
                 idx=idx.cpu().numpy(), ref_idx=ref[2].cpu().numpy(), blocks=np.array(blocks), head_ok=head_ok)
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_query_and_head_sharding_match_single_gpu(tmp_path):
    world = 2
    ctx = mp.get_context("spawn")
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, str(tmp_path))) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(240)
        assert p.exitcode == 0, f"rank exit code {p.exitcode}"
    for r in range(world):
        z = np.load(tmp_path / f"r{r}.npz")
        assert bool(z["out_equal"]), "gathered output rows differ from single-GPU evict"
        # each key's importance is computed by one rank exactly as on one GPU
        assert bool(z["imp_equal"]), float(z["imp_err"])
        np.testing.assert_array_equal(z["idx"], z["ref_idx"])
        assert bool(z["head_ok"])
    b0 = np.load(tmp_path / "r0.npz")["blocks"]
    b1 = np.load(tmp_path / "r1.npz")["blocks"]
    assert sorted(np.r_[b0, b1].tolist()) == list(range((3000 + 255) // 256))


class _ThreadRanks:
    """Ranks as threads of this process, all on cuda:0, with the two
    collectives the sharded paths use (all_reduce SUM, all_gather) done by
    torch ops over the ranks' tensors.  Lets a one-GPU box run the real
    evict_query_sharded / evict_head_sharded code (block lists, key-tile
    ranges, statistics exchange, score reduction, selection on every rank)."""

    def __init__(self, world):
        import threading
        self.world = world
        self.barrier = threading.Barrier(world, timeout=300)
        self.slots = [None] * world

    def handle(self, rank):
        return (self, rank)

    def all_reduce(self, tensor, op=None, group=None):
        shared, rank = group
        assert shared is self and (op is None or op == dist_sum())
        torch.cuda.synchronize()
        self.slots[rank] = tensor.clone()
        self.barrier.wait()
        total = self.slots[0].clone()
        for r in range(1, self.world):
            total += self.slots[r]
        torch.cuda.synchronize()
        self.barrier.wait()
        tensor.copy_(total)

    def all_gather(self, recv, send, group=None):
        shared, rank = group
        torch.cuda.synchronize()
        self.slots[rank] = send.clone()
        self.barrier.wait()
        for r in range(self.world):
            recv[r].copy_(self.slots[r])
        torch.cuda.synchronize()
        self.barrier.wait()

    def run(self, fn):
        """fn(rank, group) on every rank's thread; returns the results by rank."""
        import threading
        results, errors = [None] * self.world, []

        def body(r):
            try:
                results[r] = fn(r, self.handle(r))
            except BaseException as e:  # noqa: BLE001 - reported below
                errors.append(e)
                self.barrier.abort()

        threads = [threading.Thread(target=body, args=(r,)) for r in range(self.world)]
        for t in threads:
            t.start()
        for t in threads:
            t.join()
        if errors:
            raise errors[0]
        return results


def dist_sum():
    import torch.distributed as dist
    return dist.ReduceOp.SUM


def _patch_ranks(monkeypatch, ranks):
    import flash_evict.distributed as D
    monkeypatch.setattr(D, "_world", lambda group: (group[1], group[0].world))
    monkeypatch.setattr(D.dist, "all_reduce", ranks.all_reduce)
    monkeypatch.setattr(D.dist, "all_gather", ranks.all_gather)


@pytest.mark.parametrize("world,n,hq,hkv,decay,window,gather", [
    (2, 3000, 8, 2, 0.01, 0, True),
    (3, 5000, 4, 1, 0.0, 700, True),
    (4, 8192, 8, 2, 0.1, 0, True),
    # BASELINE c4 at full size (B1 Hq32 Hkv8 N131072 D128 bf16, decay 0.1,
    # budget 1024, reserved 64) on eight ranks
    (8, 131072, 32, 8, 0.1, 0, False),
])
def test_query_sharded_ranks_on_one_gpu_match_single_gpu(monkeypatch, world, n, hq, hkv, decay, window, gather):
    """evict_query_sharded with `world` thread ranks on one GPU: every rank's
    importance, indices and mask, and the gathered output rows, are bit for
    bit those of a single evict() on the same inputs."""
    from flash_evict import evict
    from flash_evict.distributed import BLOCK, evict_query_sharded
    dev = torch.device("cuda", 0)
    g = torch.Generator(device=dev).manual_seed(11 + world)
    q = torch.randn(1, hq, n, 128, generator=g, device=dev).to(torch.bfloat16)
    k = torch.randn(1, hkv, n, 128, generator=g, device=dev).to(torch.bfloat16)
    v = torch.randn(1, hkv, n, 128, generator=g, device=dev).to(torch.bfloat16)
    budget = 1024 if n > 4096 else 300
    ref = evict(q, k, v, budget, reserved_recent=64, recency_decay=decay, observation_window=window)
    torch.cuda.synchronize()
    ranks = _ThreadRanks(world)
    _patch_ranks(monkeypatch, ranks)
    res = ranks.run(lambda r, grp: evict_query_sharded(q, k, v, budget, group=grp, reserved_recent=64,
                                                       recency_decay=decay, observation_window=window,
                                                       gather_output=gather))
    torch.cuda.synchronize()
    blocks = sorted(b for r in range(world) for b in res[r][4])
    assert blocks == list(range((n + BLOCK - 1) // BLOCK))
    for r in range(world):
        out, imp, idx, mask, mine = res[r]
        assert torch.equal(imp, ref[1]), f"rank {r}: importance differs from single-GPU evict"
        assert torch.equal(idx, ref[2]) and torch.equal(mask, ref[3]), f"rank {r}: selection differs"
        if gather:
            assert torch.equal(out, ref[0]), f"rank {r}: gathered output differs"
        else:
            for blk in mine:
                lo, hi = blk * BLOCK, min(n, (blk + 1) * BLOCK)
                assert torch.equal(out[:, :, lo:hi], ref[0][:, :, lo:hi]), f"rank {r}: rows of block {blk} differ"


@pytest.mark.parametrize("world", [2, 3, 8])
def test_head_sharded_ranks_on_one_gpu_match_single_gpu(monkeypatch, world):
    """evict_head_sharded on BASELINE c5's layout (B8 Hq=Hkv=32 N4096 D128
    fp16, [B,N,H,D]-transposed views, q x30, 5 % of v rows zero, noncausal,
    H2O mass, budget 10 % of N) with `world` thread ranks on one GPU: the
    ranks' blocks cover every (batch, kv head) once and each equals the
    single-GPU evict() of the whole tensor bit for bit."""
    from flash_evict import evict
    from flash_evict.distributed import evict_head_sharded
    dev = torch.device("cuda", 0)
    g = torch.Generator(device=dev).manual_seed(7)
    q = (torch.randn(8, 4096, 32, 128, generator=g, device=dev) * 30).to(torch.float16).transpose(1, 2)
    k = torch.randn(8, 4096, 32, 128, generator=g, device=dev).to(torch.float16).transpose(1, 2)
    v = torch.randn(8, 4096, 32, 128, generator=g, device=dev)
    v[torch.rand(8, 4096, generator=g, device=dev) < 0.05] = 0
    v = v.to(torch.float16).transpose(1, 2)
    ref = evict(q, k, v, 409, causal=False, value_weighted=False)
    torch.cuda.synchronize()
    ranks = _ThreadRanks(world)
    _patch_ranks(monkeypatch, ranks)
    res = ranks.run(lambda r, grp: evict_head_sharded(q, k, v, 409, group=grp, causal=False, value_weighted=False))
    torch.cuda.synchronize()
    covered = torch.zeros(8, 32, dtype=torch.int32)
    for r in range(world):
        for b0, b1, h0, h1, o, i, ix, m in res[r]:
            covered[b0:b1, h0:h1] += 1
            assert torch.equal(o, ref[0][b0:b1, h0:h1]) and torch.equal(i, ref[1][b0:b1, h0:h1])
            assert torch.equal(ix, ref[2][b0:b1, h0:h1]) and torch.equal(m, ref[3][b0:b1, h0:h1])
    assert covered.eq(1).all()


@pytest.mark.parametrize("world", [3, 8])
def test_head_sharded_c4_ranks_on_one_gpu_match_single_gpu(monkeypatch, world):
    """The control plan for BASELINE c4 (B1 Hq32 Hkv8 N131072 D128 bf16,
    causal, decay 0.1, reserved 64, budget 1024): its KV heads split over
    `world` thread ranks on one GPU with evict_head_sharded, each rank's
    outputs (its KV heads' 4 query heads each), importance, indices and mask
    bitwise equal to one evict() of the whole tensor."""
    from flash_evict import evict
    from flash_evict.distributed import evict_head_sharded
    dev = torch.device("cuda", 0)
    g = torch.Generator(device=dev).manual_seed(23)
    q = torch.randn(1, 32, 131072, 128, generator=g, device=dev).to(torch.bfloat16)
    k = torch.randn(1, 8, 131072, 128, generator=g, device=dev).to(torch.bfloat16)
    v = torch.randn(1, 8, 131072, 128, generator=g, device=dev).to(torch.bfloat16)
    kw = dict(reserved_recent=64, recency_decay=0.1)
    ref = evict(q, k, v, 1024, **kw)
    torch.cuda.synchronize()
    ranks = _ThreadRanks(world)
    _patch_ranks(monkeypatch, ranks)
    res = ranks.run(lambda r, grp: evict_head_sharded(q, k, v, 1024, group=grp, **kw))
    torch.cuda.synchronize()
    covered = torch.zeros(1, 8, dtype=torch.int32)
    for r in range(world):
        for b0, b1, h0, h1, o, i, ix, m in res[r]:
            covered[b0:b1, h0:h1] += 1
            assert torch.equal(o, ref[0][b0:b1, h0 * 4:h1 * 4]), f"rank {r}: output rows differ"
            assert torch.equal(i, ref[1][b0:b1, h0:h1]), f"rank {r}: importance differs"
            assert torch.equal(ix, ref[2][b0:b1, h0:h1]) and torch.equal(m, ref[3][b0:b1, h0:h1])
    assert covered.eq(1).all()
