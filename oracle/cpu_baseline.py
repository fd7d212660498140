"""CPU baseline of the evict() path -- BASELINE/TEST INFRASTRUCTURE ONLY.

The reference's CPU path is its materialized FP32 torch arithmetic
(flash_evict/reference.py:5-25): logits = Q K^T * scale in FP32, causal mask,
row softmax, out = P V, importance = sum over rows of w_q * P, times ||v||_1.
This module runs that arithmetic with torch on the host cores, over query
chunks (N x N does not fit at 32K and beyond), on a fixed sample of one
workload: the last R query rows of the G query heads of (batch 0, kv head 0),
then (batch 0, kv head 1), ... until about `target_flops` of algorithmic work.
Only bench.py's cpu_baseline leg and `bench.py --impl reference` run it; the
product path never imports it.

FLOPs are counted with the same formula as the GPU metric: 4*D per (row, key)
of attention plus 2*D per (scored row, key) of importance.
"""
import os

import torch


def host_threads():
    """All cores this process may run on (the affinity mask), so a rank
    launched with OMP_NUM_THREADS=1 still measures the whole host."""
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:  # pragma: no cover
        return os.cpu_count() or 1


def sample_plan(b, hq, hkv, n, d, causal, target_flops=4e11):
    """[(b, h, rows_lo)]: units and the first sampled row of each (rows
    rows_lo..n-1), chosen to reach about target_flops of attention work."""
    g = hq // hkv
    plan, left = [], float(target_flops)
    for u in range(b * hkv):
        bi, h = divmod(u, hkv)
        per_row = 4.0 * d * g * n  # an upper bound: rows near the end see ~n keys
        rows = min(n, max(256, int(left / per_row) // 256 * 256))
        plan.append((bi, h, n - rows))
        left -= rows * per_row
        if left <= 0:
            break
    return plan


def prepare(q, k, v, plan):
    """float32 host copies of the sampled units (setup, not timed)."""
    g = q.shape[1] // k.shape[1]
    out = []
    for bi, h, lo in plan:
        out.append((q[bi, h * g:(h + 1) * g, lo:].float().cpu().contiguous(),
                    k[bi, h].float().cpu().contiguous(), v[bi, h].float().cpu().contiguous(), lo))
    return out


def run(units, n, causal, scale, recency_decay, observation_window, value_weighted, chunk=256):
    """One pass over the prepared sample.  Returns (algorithmic FLOPs, outputs
    checksum).  The importance sums run over the sampled rows only."""
    flops = 0
    check = 0.0
    pos = torch.arange(n)
    w_all = torch.exp(torch.tensor(float(recency_decay)) * (pos.float() - (n - 1)))
    if observation_window:
        w_all = w_all * (pos >= n - observation_window)
    sc = torch.tensor(scale, dtype=torch.float32)
    for qs, ks, vs, lo in units:
        d = ks.shape[-1]
        mass = torch.zeros(n)
        for hh in range(qs.shape[0]):
            for s in range(0, qs.shape[1], chunk):
                r = torch.arange(lo + s, min(n, lo + s + chunk))
                logits = (qs[hh, s:s + len(r)] @ ks.T) * sc
                if causal:
                    logits.masked_fill_(pos[None, :] > r[:, None], float("-inf"))
                p = torch.softmax(logits, -1)
                out = p @ vs
                w = w_all[r]
                scored = w > 0
                if bool(scored.any()):
                    mass += (p * w[:, None]).sum(0)
                keys = int((r + 1).sum()) if causal else len(r) * n
                keys_scored = int((r[scored] + 1).sum()) if causal else int(scored.sum()) * n
                flops += 4 * d * keys + 2 * d * keys_scored
                check += float(out[-1, 0])
        if value_weighted:
            mass = mass * vs.abs().sum(-1)
        check += float(mass.sum())
    return flops, check
