"""CPU restatement of the reference's evict() path -- TEST INFRASTRUCTURE ONLY.

This module is the checker for the CUDA kernels: only tests/, the smoke test
in __graft_entry__.py and the CPU-baseline leg of bench.py may import it.  The
product path (flash_evict) never calls it.

Parity is pinned against the reference itself: tests/golden/make_golden.py
imports the reference package (flash_evict/reference.py, flash_evict/prefill.py
select_tokens, flash_evict/baselines.py snap_select) and records its outputs on
seeded inputs; tests/test_oracle_golden.py checks this restatement against
those fixtures.

Functions (numpy, float32 like the reference or float64 for ground truth):
  materialized  -- reference.py:5-25 (N x N softmax, weighted column sums)
  chunked       -- the same math per query chunk, for N where N x N does not fit
  avg_pool      -- F.avg_pool1d(k, stride 1, pad k//2) as used at prefill.py:161-163
  select_tokens -- prefill.py:140-170 with a stated tie-break
  uniform_analytic / weighted_analytic -- the Q=K=0 closed forms the reference
                   tests use (tests/test_prefill.py:88-102, 134-146)
"""
import math

import numpy as np

LOG2E = 1.4426950408889634


def _as_np(x):
    if hasattr(x, "detach"):  # torch tensor
        x = x.detach().cpu()
        if str(x.dtype) in ("torch.bfloat16", "torch.float16"):
            x = x.float()
        x = x.numpy()
    return np.asarray(x)


def recency_weights(n, recency_decay=0.0, observation_window=0, dtype=np.float32):
    """w_q = exp(decay * (q - (n-1))) * [q >= n - window]  (reference.py:19-22)."""
    pos = np.arange(n, dtype=dtype)
    w = np.exp(dtype(recency_decay) * (pos - dtype(n - 1))).astype(dtype)
    if observation_window:
        w = w * (np.arange(n) >= n - observation_window)
    return w.astype(dtype)


def _softmax_rows(logits):
    m = logits.max(-1, keepdims=True)
    e = np.exp(logits - m)
    return e / e.sum(-1, keepdims=True)


def materialized(q, k, v, *, causal=True, value_weighted=True, scale=None, recency_decay=0.0,
                 observation_window=0, dtype=np.float32):
    """Restates flash_evict/reference.py:5-25 (`materialized`).

    q [B,Hq,N,D], k/v [B,Hkv,N,D] -> (out [B,Hq,N,D], mass [B,Hkv,N]).
    """
    q, k, v = (_as_np(t).astype(dtype) for t in (q, k, v))
    b, hq, n, d = q.shape
    hkv = k.shape[1]
    groups = hq // hkv
    kr = np.repeat(k, groups, axis=1)          # repeat_interleave (reference.py:8)
    vr = np.repeat(v, groups, axis=1)
    logits = q @ np.swapaxes(kr, -1, -2)      # reference.py:10
    logits *= dtype(d ** -0.5 if scale is None else scale)
    if causal:                                 # reference.py:12-14
        pos = np.arange(n)
        logits = np.where(pos[None, :] > pos[:, None], -np.inf, logits)
    p = _softmax_rows(logits).astype(dtype)    # reference.py:15
    out = p @ vr                               # reference.py:16
    w = recency_weights(n, recency_decay, observation_window, dtype)
    mass = (p * w[:, None]).sum(-2).reshape(b, hkv, groups, n).sum(2)  # reference.py:22
    if value_weighted:
        mass = mass * np.abs(v).sum(-1)        # reference.py:23-24
    return out.astype(dtype), mass.astype(dtype)


def chunked(q, k, v, *, causal=True, value_weighted=True, scale=None, recency_decay=0.0,
            observation_window=0, out_rows=None, chunk=256, dtype=np.float64, weight_floor=0.0,
            score_rows=None):
    """Query-chunked restatement of reference.py:5-25 for long sequences.

    Row softmax is exact per query chunk (all keys at once); the weighted
    column sums accumulate in float64.  out_rows: None -> outputs for every
    row; an index array -> outputs only for those rows (others left NaN);
    an empty list -> no outputs.  Rows whose weight is <= weight_floor are
    not visited for the importance.  score_rows restricts the importance
    sum to those query rows (a partial sum, as one rank of a query-sharded
    job computes it).
    Returns (out [B,Hq,N,D] float32, mass [B,Hkv,N] float32).
    """
    q, k, v = (_as_np(t) for t in (q, k, v))
    b, hq, n, d = q.shape
    hkv = k.shape[1]
    groups = hq // hkv
    sc = d ** -0.5 if scale is None else scale
    w = recency_weights(n, recency_decay, observation_window, np.float64)
    if score_rows is not None:
        keep = np.zeros(n, dtype=bool)
        keep[np.asarray(score_rows, dtype=np.int64)] = True
        w = np.where(keep, w, 0.0)
    scored = np.nonzero(w > weight_floor)[0]
    if out_rows is None:
        want_out = np.arange(n)
    else:
        want_out = np.asarray(out_rows, dtype=np.int64)
    out = np.full((b, hq, n, d), np.nan, dtype=np.float32) if len(want_out) else None
    rows = np.union1d(scored, want_out).astype(np.int64)
    out_flag = np.zeros(n, dtype=bool)
    out_flag[want_out] = True
    mass = np.zeros((b, hkv, n), dtype=np.float64)
    for bi in range(b):
        for h in range(hkv):
            kk = k[bi, h].astype(dtype)
            vv = v[bi, h].astype(dtype)
            for g in range(groups):
                qh = h * groups + g
                for s in range(0, len(rows), chunk):
                    r = rows[s:s + chunk]
                    logits = (q[bi, qh, r].astype(dtype) @ kk.T) * dtype(sc)
                    if causal:
                        logits = np.where(np.arange(n)[None, :] > r[:, None], -np.inf, logits)
                    p = _softmax_rows(logits)
                    sel = out_flag[r]
                    if out is not None and sel.any():
                        out[bi, qh, r[sel]] = (p[sel] @ vv).astype(np.float32)
                    wr = w[r]
                    if (wr > weight_floor).any():
                        mass[bi, h] += (p * wr[:, None]).sum(0)
            if value_weighted:
                mass[bi, h] *= np.abs(v[bi, h].astype(np.float64)).sum(-1)
    return out, mass.astype(np.float32)


def avg_pool(past, kernel):
    """F.avg_pool1d(past, kernel, stride=1, padding=kernel//2) in float32
    (count_include_pad: divisor = kernel).  Taps are summed left to right,
    out-of-range taps skipped, then one IEEE division -- the accumulation order
    of PyTorch's avg_pool kernels."""
    past = np.asarray(past, dtype=np.float32)
    r = kernel // 2
    p = past.shape[-1]
    acc = np.zeros_like(past)
    for t in range(-r, r + 1):
        shifted = np.zeros_like(past)
        if t < 0:
            shifted[..., -t:] = past[..., :p + t] if p + t > 0 else shifted[..., -t:]
        elif t > 0:
            shifted[..., :p - t] = past[..., t:] if p - t > 0 else shifted[..., :p - t]
        else:
            shifted = past
        acc = (acc + shifted).astype(np.float32)
    return (acc / np.float32(kernel)).astype(np.float32)


def order_keys(x):
    """Order-preserving uint32 keys: larger float -> larger key, NaN largest,
    -0.0 equal to +0.0."""
    x = np.asarray(x, dtype=np.float32).copy()
    x[x == 0] = 0.0
    u = x.view(np.uint32)
    key = np.where(u & np.uint32(0x80000000), ~u, u | np.uint32(0x80000000)).astype(np.uint32)
    key[np.isnan(x)] = np.uint32(0xFFFFFFFF)
    return key


def _check_select_args(n, budget, recent, reserved_recent, pool_kernel):
    # prefill.py:150-159
    if reserved_recent is not None:
        if recent != 0 and recent != reserved_recent:
            raise ValueError("recent and reserved_recent disagree")
        recent = reserved_recent
    if isinstance(budget, bool) or not isinstance(budget, int) or not 1 <= budget <= n:
        raise ValueError("budget must be an integer in [1, sequence length]")
    if isinstance(recent, bool) or not isinstance(recent, int) or not 0 <= recent <= budget:
        raise ValueError("recent must be an integer in [0, budget]")
    if isinstance(pool_kernel, bool) or not isinstance(pool_kernel, int) or pool_kernel < 1 or pool_kernel % 2 != 1:
        raise ValueError("pool_kernel must be a positive odd integer")
    return recent


def select_tokens(importance, budget, *, recent=0, reserved_recent=None, pool_kernel=1):
    """Restates prefill.py:140-170 with the tie-break stated by the CUDA
    kernel: larger value first, among equal values the lower index.

    Returns (indices int64 [..., budget] ascending, keep bool [..., N]).
    """
    imp = np.asarray(_as_np(importance), dtype=np.float32)
    n = imp.shape[-1]
    recent = _check_select_args(n, budget, recent, reserved_recent, pool_kernel)
    lead = imp.shape[:-1]
    flat = imp.reshape(-1, n)
    past = flat[:, :n - recent]
    if pool_kernel > 1 and budget > recent:
        past = avg_pool(past, pool_kernel)
    kk = budget - recent
    idx = np.empty((flat.shape[0], budget), dtype=np.int64)
    keep = np.zeros((flat.shape[0], n), dtype=bool)
    tail = np.arange(n - recent, n, dtype=np.int64)
    for r in range(flat.shape[0]):
        if kk:
            keys = order_keys(past[r])
            order = np.lexsort((np.arange(past.shape[1]), ~keys))
            top = np.sort(order[:kk])
        else:
            top = np.empty(0, dtype=np.int64)
        idx[r] = np.concatenate([top, tail])
        keep[r, idx[r]] = True
    return idx.reshape(lead + (budget,)), keep.reshape(imp.shape)


def gather_tokens(x, indices):
    """KV compaction: x[b, h, indices[b, h, j], :] (README.md:31,
    `k.gather(2, indices[..., None].expand(-1, -1, -1, k.shape[-1]))`; the
    adapters call it through kv_distill's gather_tokens at
    kv_distill_adapter.py:38-39, streaming_adapter.py:86,
    quality_adapter.py:109-110)."""
    x = np.asarray(x)
    idx = np.asarray(indices, dtype=np.int64)
    return np.take_along_axis(x, idx[..., None], axis=2)


def round_to_dtype(x, dtype_name):
    """Round float32 values to float16/bfloat16 and back, round to nearest
    even (what a matmul that writes its output in that dtype does)."""
    x = np.asarray(x, dtype=np.float32)
    if dtype_name == "float16":
        return x.astype(np.float16).astype(np.float32)
    if dtype_name == "bfloat16":
        u = x.view(np.uint32).astype(np.uint64)
        r = ((u + 0x7FFF + ((u >> 16) & 1)) & 0xFFFF0000).astype(np.uint32)
        return r.view(np.float32)
    return x


def snap_scores(q, k, window=32, dtype_name="bfloat16"):
    """SnapKV observation-window scores (baselines.py:12-26).

    q [B,Hq,N,D], k [B,Hkv,N,D] hold the fp16/bf16 input values as floats.
    logits = round_to_dtype(q[:, :, -w:] @ k^T) (the reference's matmul runs in
    the input dtype), then * D**-0.5 in float32, keys after the query's
    position masked, softmax over the keys (float64 here), summed over the w
    window rows and averaged over the G query heads of each KV head.  One
    query head at a time, so memory stays at w x N.
    """
    q = np.asarray(q, dtype=np.float64)
    k = np.asarray(k, dtype=np.float64)
    b, h, n, d = q.shape
    hk = k.shape[1]
    g = h // hk
    w = min(window, n)
    qpos = np.arange(n - w, n)
    masked = np.arange(n)[None, :] > qpos[:, None]
    scale = np.float32(d ** -0.5)
    out = np.zeros((b, hk, n), dtype=np.float64)
    for bi in range(b):
        for hi in range(h):
            logits = q[bi, hi, n - w:] @ k[bi, hi // g].T
            logits = round_to_dtype(logits.astype(np.float32), dtype_name) * scale
            logits = np.where(masked, -np.inf, logits.astype(np.float64))
            p = np.exp(logits - logits.max(-1, keepdims=True))
            p /= p.sum(-1, keepdims=True)
            out[bi, hi // g] += p.sum(0)
    return (out / g).astype(np.float32)


def snap_select(scores, budget, window=32, kernel=5):
    """baselines.py:29-43: all tokens when N <= budget, else the window
    suffix plus the top of the average-pooled past (select_tokens with
    recent = min(window, N, budget-1) and pool_kernel = kernel)."""
    scores = np.asarray(scores)
    n = scores.shape[-1]
    if n <= budget:
        idx = np.broadcast_to(np.arange(n), scores.shape[:-1] + (n,))
        return idx, np.ones(scores.shape, dtype=bool)
    window = min(window, n, budget - 1)
    return select_tokens(scores, budget, recent=window, pool_kernel=kernel)


def uniform_analytic(v, groups):
    """Q = K = 0, causal: P[q,k] = 1/(q+1) for k <= q.  Returns (out, importance)
    for value-weighted scoring (tests/test_prefill.py:88-102 of the reference).
    v: [B,Hkv,N,D] -> out [B,Hkv,N,D] (per KV head), importance [B,Hkv,N]."""
    v = _as_np(v).astype(np.float64)
    n = v.shape[2]
    pos = np.arange(1, n + 1, dtype=np.float64)
    out = np.cumsum(v, axis=2) / pos[None, None, :, None]
    harmonic = np.cumsum((1.0 / pos)[::-1])[::-1]
    imp = np.abs(v).sum(-1) * harmonic * groups
    return out, imp


def weighted_analytic(n, recency_decay, observation_window, groups, vnorm):
    """Q = K = 0, causal, V = 1: I_k = vnorm * groups * sum_{q>=k} w_q/(q+1)
    (tests/test_prefill.py:134-146 of the reference)."""
    pos = np.arange(n, dtype=np.float64)
    w = np.exp(recency_decay * (pos - (n - 1)))
    if observation_window:
        w = w * (pos >= n - observation_window)
    return np.cumsum((w / (pos + 1))[::-1])[::-1] * vnorm * groups


def attention_flops(b, hq, n, d, causal):
    """4 * B * Hq * D * sum_q K(q): QK^T and PV, each 2 flops per MAC."""
    keys = n * (n + 1) // 2 if causal else n * n
    return 4 * b * hq * d * keys


def replay_flops(b, hq, n, d, causal, scored_rows):
    """2 * B * Hq * D * sum over scored rows of their key counts."""
    rows = np.asarray(scored_rows, dtype=np.int64)
    keys = (rows + 1).sum() if causal else len(rows) * n
    return 2 * b * hq * d * int(keys)


def scored_rows(n, recency_decay=0.0, observation_window=0, skip_underflow=True):
    """Rows that carry weight: the window, minus rows whose FP32 weight is
    below 2^-127 when skip_underflow (what the CUDA replay skips)."""
    w_lo = n - (observation_window if observation_window and observation_window < n else n)
    lo = w_lo
    if skip_underflow and recency_decay > 0:
        # the kernel receives the decay as FP32
        reach = 127.0 / (float(np.float32(recency_decay)) * LOG2E)
        if reach < n:
            lo = max(lo, n - 1 - int(math.floor(reach)))
    return np.arange(lo, n)


def parity_figures(out_got, out_ref, imp_got, imp_ref, rel_floor=1e-6):
    """Error figures of a GPU result against this oracle (float64 truth).

    out_got/out_ref: sampled attention-output rows (any matching shape).
    imp_got/imp_ref: importance [..., N].  The relative importance error is
    taken over keys whose reference importance is at least `rel_floor` times
    the largest of its row (smaller ones sit at the FP32 underflow edge of
    exp2, where a relative figure means nothing); their absolute error is
    reported relative to that row maximum instead.
    """
    og = np.asarray(out_got, dtype=np.float64)
    orf = np.asarray(out_ref, dtype=np.float64)
    ig = np.asarray(imp_got, dtype=np.float64).reshape(-1, np.asarray(imp_got).shape[-1])
    ir = np.asarray(imp_ref, dtype=np.float64).reshape(ig.shape)
    err = np.abs(ig - ir)
    rowmax = np.maximum(np.abs(ir).max(-1, keepdims=True), 1e-300)
    big = np.abs(ir) >= rel_floor * rowmax
    rel = np.where(big, err / np.maximum(np.abs(ir), 1e-300), 0.0)
    return {
        "out_max_abs": float(np.abs(og - orf).max()) if og.size else 0.0,
        "out_max_rel": float(np.abs(og - orf).max() / max(np.abs(orf).max(), 1e-300)) if og.size else 0.0,
        "importance_max_rel": float(rel.max()),
        "importance_rel_floor": rel_floor,
        "importance_keys_checked": int(big.sum()),
        "importance_small_max_abs_over_rowmax": float((np.where(big, 0.0, err) / rowmax).max()),
        "importance_nonfinite": int((~np.isfinite(ig)).sum()),
    }


def selection_figures(keep_got, imp_ref, budget, *, recent=0, reserved_recent=None, pool_kernel=1, tie_rtol=1e-5):
    """Keep-mask differences between a GPU selection and this oracle's
    selection on the reference importance, and how many of the differing
    tokens are near ties: their reference selection score (the pooled past
    score when pool_kernel > 1) lies within tie_rtol (relative) of the row's
    threshold, the smallest reference score that was kept."""
    imp = np.asarray(imp_ref, dtype=np.float32)
    n = imp.shape[-1]
    recent = _check_select_args(n, budget, recent, reserved_recent, pool_kernel)
    _, ref_keep = select_tokens(imp, budget, recent=recent, pool_kernel=pool_kernel)
    got = np.asarray(keep_got, dtype=bool).reshape(-1, n)
    ref_keep = ref_keep.reshape(-1, n)
    past = imp.reshape(-1, n)[:, :n - recent]
    if pool_kernel > 1 and budget > recent:
        past = avg_pool(past, pool_kernel)
    diff = got != ref_keep
    ties = 0
    for r in np.nonzero(diff.any(1))[0]:
        kept = past[r][ref_keep[r, :n - recent]]
        thr = float(kept.min()) if kept.size else 0.0
        for c in np.nonzero(diff[r])[0]:
            if c < n - recent and abs(float(past[r, c]) - thr) <= tie_rtol * abs(thr):
                ties += 1
    return {"mask_mismatches": int(diff.sum()), "mismatches_near_ties": ties, "tie_rtol": tie_rtol,
            "index_rows_equal": int((~diff.any(1)).sum()), "rows": int(diff.shape[0])}
