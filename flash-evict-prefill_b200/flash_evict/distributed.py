"""Multi-GPU evict(): one process per GPU, torch.distributed for the plumbing.

The reference is single-GPU (no torch.distributed anywhere).  Two
partitionings of the same computation are provided:

head  -- the (batch, kv-head) units are independent: every rank takes a
         contiguous range of them (with their G query heads) and runs the
         whole evict() path locally.  No communication.
query -- for long contexts: query rows are dealt out in 256-row blocks
         (FE_QUERY_BLOCK) in a causal-balanced snake order.  Every rank holds
         the full K/V and computes the attention output and softmax row
         statistics of its own rows.  The scored rows (the observation
         window, or the rows a recency decay leaves above FP32 underflow)
         usually sit in a few blocks at the end, so the replay is balanced
         separately: the statistics of the scored rows are exchanged (one
         small all_reduce), every rank replays all scored rows against its
         own contiguous range of key tiles, and one all_reduce(SUM) of the
         FP32 [B, Hkv, N] scores (each key written by exactly one rank,
         zeros elsewhere) gives every rank the full importance; each rank
         then runs the (identical) selection.  The attention output can
         optionally be all-gathered.

Each importance value is computed by one rank with the same kernel, inputs
and summation order as on a single GPU, so the result is bitwise equal to
single-GPU evict() for any world size.
"""
import torch
import torch.distributed as dist

from . import _lib
from .prefill import (_attention, _check_prefill_args, _check_select_args, _replay, _select, _tma_view,
                      _validate)

__all__ = ["query_block_plan", "head_unit_plan", "head_blocks", "key_tile_plan", "first_scored_row",
           "evict_query_sharded", "evict_head_sharded"]

BLOCK = _lib.QUERY_BLOCK


def _block_cost(i, n, causal):
    """Attention work of query block i in 128-key tiles (both 128-row tiles)."""
    nkv = (n + 127) // 128
    cost = 0
    for t in (2 * i, 2 * i + 1):
        if t * 128 >= n:
            continue
        cost += min(nkv, t + 1) if causal else nkv
    return cost


def query_block_plan(n_tokens, world, causal=True):
    """Deal the query blocks of an n_tokens sequence to `world` ranks.

    Blocks are sorted by cost (descending) and dealt in a snake order
    (0..P-1, P-1..0, ...), which balances the causal triangle to within one
    block.  Each rank's list is heaviest first, the order its kernel wants.
    Returns a list (one per rank) of block-index lists.
    """
    nblk = (n_tokens + BLOCK - 1) // BLOCK
    order = sorted(range(nblk), key=lambda i: (-_block_cost(i, n_tokens, causal), i))
    plan = [[] for _ in range(world)]
    for j, blk in enumerate(order):
        rnd, pos = divmod(j, world)
        rank = pos if rnd % 2 == 0 else world - 1 - pos
        plan[rank].append(blk)
    return plan


def key_tile_plan(n_tokens, world):
    """Split the ceil(n_tokens/128) key tiles into `world` contiguous ranges
    (begin, end), one per rank."""
    nkt = (n_tokens + 127) // 128
    return [(nkt * r // world, nkt * (r + 1) // world) for r in range(world)]


def first_scored_row(n_tokens, recency_decay=0.0, observation_window=0):
    """First query row that carries weight in the replay: the start of the
    observation window, raised past rows whose FP32 weight
    exp(-decay * distance) is below 2^-127 (the rows the replay kernel skips).
    Computed by the library itself (the kernel receives the decay as FP32), so
    the rows exchanged here are exactly the rows the kernel reads."""
    return int(_lib.load().fe_replay_first_scored_row(int(n_tokens), float(recency_decay),
                                                      int(observation_window)))


def head_unit_plan(batch, kv_heads, world):
    """Split the batch*kv_heads units into `world` contiguous ranges.
    Returns, per rank, a list of (b, h0, h1) runs (kv heads h0..h1-1 of batch b)."""
    total = batch * kv_heads
    plan = []
    for r in range(world):
        lo = total * r // world
        hi = total * (r + 1) // world
        runs = []
        u = lo
        while u < hi:
            b, h0 = divmod(u, kv_heads)
            h1 = min(kv_heads, h0 + (hi - u))
            runs.append((b, h0, h1))
            u += h1 - h0
        plan.append(runs)
    return plan


def head_blocks(batch, kv_heads, world):
    """head_unit_plan with consecutive whole batches merged: per rank a list
    of (b0, b1, h0, h1) blocks -- batches b0..b1-1, kv heads h0..h1-1 -- so a
    rank whose range spans whole batches runs them as one evict() call (three
    launches) instead of one call per batch."""
    out = []
    for runs in head_unit_plan(batch, kv_heads, world):
        blocks = []
        for b, h0, h1 in runs:
            whole = h0 == 0 and h1 == kv_heads
            if whole and blocks and blocks[-1][2] == 0 and blocks[-1][3] == kv_heads and blocks[-1][1] == b:
                blocks[-1] = (blocks[-1][0], b + 1, 0, kv_heads)
            else:
                blocks.append((b, b + 1, h0, h1))
        out.append(blocks)
    return out


def _world(group):
    if group is None and not dist.is_initialized():
        return 0, 1
    return dist.get_rank(group), dist.get_world_size(group)


def evict_head_sharded(q, k, v, budget, *, group=None, recent=0, reserved_recent=None, pool_kernel=1,
                       **prefill_kwargs):
    """Run evict() on this rank's (batch, kv-head) units; no communication.

    q/k/v are the full [B, H, N, D] tensors (views are taken, nothing is
    copied).  Returns a list of (b0, b1, h0, h1, out, importance, indices,
    mask) for the blocks this rank owns (head_blocks): batches b0..b1-1 and kv
    heads h0..h1-1; `out` covers query heads h0*G..h1*G-1 of those batches.
    """
    from .prefill import evict
    rank, world = _world(group)
    g = q.shape[1] // k.shape[1]
    results = []
    for b0, b1, h0, h1 in head_blocks(q.shape[0], k.shape[1], world)[rank]:
        res = evict(q[b0:b1, h0 * g:h1 * g], k[b0:b1, h0:h1], v[b0:b1, h0:h1], budget, recent=recent,
                    reserved_recent=reserved_recent, pool_kernel=pool_kernel, **prefill_kwargs)
        results.append((b0, b1, h0, h1) + tuple(res))
    return results


def _cuda_attend(q, k, v, blocks, causal, scale):
    """This rank's attention rows and their softmax row statistics."""
    b, h, n, d = q.shape
    out = torch.empty(q.shape, dtype=q.dtype, device=q.device)
    row_stats = torch.empty((b, h, n, 2), dtype=torch.float32, device=q.device)
    if len(blocks):
        blk = torch.tensor(blocks, dtype=torch.int32, device=q.device)
        with torch.cuda.device(q.device):
            _attention(_tma_view(q), _tma_view(k), _tma_view(v), out, row_stats, causal, scale, query_blocks=blk)
    return out, row_stats


def _cuda_replay(q, k, v, row_stats, key_tiles, causal, scale, recency_decay, observation_window, value_weighted):
    """Importance of this rank's key tiles from every scored row; zeros for
    the other keys."""
    importance = torch.zeros((q.shape[0], k.shape[1], q.shape[2]), dtype=torch.float32, device=q.device)
    with torch.cuda.device(q.device):
        _replay(_tma_view(q), _tma_view(k), _tma_view(v), row_stats, importance, causal, scale, recency_decay,
                observation_window, value_weighted, key_tiles=key_tiles)
    return importance


def _exchange_stats(row_stats, blocks, r0, group):
    """Give every rank the statistics of all scored rows [r0, n): each rank
    contributes the rows of its own blocks, zeros elsewhere, all_reduce(SUM)."""
    n = row_stats.shape[2]
    if r0 >= n:
        return
    part = torch.zeros_like(row_stats[:, :, r0:])
    for blk in blocks:
        lo, hi = max(r0, blk * BLOCK), min(n, (blk + 1) * BLOCK)
        if lo < hi:
            part[:, :, lo - r0:hi - r0] = row_stats[:, :, lo:hi]
    dist.all_reduce(part, op=dist.ReduceOp.SUM, group=group)
    row_stats[:, :, r0:] = part


def _gather_rows(out, plan, rank, group):
    """All-gather every rank's query blocks into a full output tensor."""
    world = len(plan)
    n = out.shape[2]
    nb_max = max(len(p) for p in plan)
    b, h, _, d = out.shape
    send = torch.zeros((nb_max, b, h, BLOCK, d), dtype=out.dtype, device=out.device)
    for j, blk in enumerate(plan[rank]):
        lo, hi = blk * BLOCK, min(n, (blk + 1) * BLOCK)
        send[j, :, :, :hi - lo] = out[:, :, lo:hi]
    recv = [torch.empty_like(send) for _ in range(world)]
    dist.all_gather(recv, send, group=group)
    full = torch.empty_like(out)
    for r in range(world):
        for j, blk in enumerate(plan[r]):
            lo, hi = blk * BLOCK, min(n, (blk + 1) * BLOCK)
            full[:, :, lo:hi] = recv[r][j, :, :, :hi - lo]
    return full


def _query_sharded(q, k, v, budget, recent, pool_kernel, causal, scale, recency_decay, observation_window,
                   value_weighted, gather_output, group, attend_fn, replay_fn, select_fn, marks=None):
    rank, world = _world(group)
    n = q.shape[2]
    plan = query_block_plan(n, world, causal)
    if marks:
        marks("start")
    out, row_stats = attend_fn(q, k, v, plan[rank], causal, scale)
    if marks:
        marks("attention")
    if world > 1:
        _exchange_stats(row_stats, plan[rank], first_scored_row(n, recency_decay, observation_window), group)
        if marks:
            marks("stats")
    importance = replay_fn(q, k, v, row_stats, key_tile_plan(n, world)[rank], causal, scale, recency_decay,
                           observation_window, value_weighted)
    if marks:
        marks("replay")
    if world > 1:
        dist.all_reduce(importance, op=dist.ReduceOp.SUM, group=group)
    if marks:
        marks("allreduce")
    indices, mask = select_fn(importance, budget, recent, pool_kernel)
    if marks:
        marks("select")
    if gather_output and world > 1:
        out = _gather_rows(out, plan, rank, group)
    return out, importance, indices, mask, plan[rank]


def evict_query_sharded(q, k, v, budget, *, group=None, recent=0, reserved_recent=None, pool_kernel=1,
                        gather_output=False, causal=True, value_weighted=True, scale=None, block_q=32,
                        block_k=64, recency_decay=0., observation_window=0, _marks=None):
    """Query-block-sharded evict() for long contexts.

    Every rank passes the same full q/k/v (on its own GPU).  Returns
    (out, importance, indices, eviction_mask, my_blocks): importance, indices
    and the mask are complete and identical on every rank; `out` holds valid
    rows only for this rank's query blocks unless gather_output=True.
    """
    _validate(q, k, v)
    recency_decay, scale = _check_prefill_args(recency_decay, observation_window, block_q, block_k, scale,
                                               q.shape[-1])
    recent = _check_select_args(q.shape[2], budget, recent, reserved_recent, pool_kernel)

    def select_fn(importance, budget_, recent_, pool_):
        return _select(importance, budget_, recent_, pool_, evict_mask=True)

    return _query_sharded(q, k, v, budget, recent, pool_kernel, causal, scale, recency_decay, observation_window,
                          value_weighted, gather_output, group, _cuda_attend, _cuda_replay, select_fn, marks=_marks)
