"""Multi-GPU evict (NCCL, one process per GPU), checked against single-GPU
evict on the same inputs (bitwise: outputs, importance, selection).  Runs
only when at least two GPUs are visible."""
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
