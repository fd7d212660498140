"""Drop-in `prefill`, `select_tokens` and `evict` for B200 (sm_100a).

Same module path, signatures, defaults, return values and ValueError contract
as the reference's flash_evict/prefill.py (prefill.py:86-180).  The compute
runs in the native library (include/flash_evict.h) on the current CUDA stream:

  prefill  -> fe_attention_fwd (tcgen05/TMA attention, writes O and row stats)
              fe_replay_scores (key-stationary exact importance, no atomics)
  select_tokens -> fe_select_tokens (pool + radix top-k + mask, one launch)

Differences from the reference, all deliberate:
  * importance is bitwise reproducible (no FP32 atomics), and score=False
    output is bitwise equal to the scored output because it is the same
    kernel launch;
  * top-k ties are broken deterministically (larger value, then lower index)
    where torch.topk leaves the order unspecified;
  * select_tokens needs a CUDA tensor: there is no CPU path.
  * block_q / block_k are validated as in the reference but do not change the
    tiling (the sm_100a kernels use fixed 128-row tiles).
"""
import math

import torch

from . import _lib

__all__ = ["prefill", "select_tokens", "evict"]


def _validate(q, k, v):
    # Same checks and messages as the reference (prefill.py:86-99).
    if any(t.ndim != 4 for t in (q, k, v)):
        raise ValueError("Q/K/V must have shape [batch, heads, tokens, channels]")
    b, h, n, d = q.shape
    if min(b, h, n, d, k.shape[1]) < 1 or k.shape != v.shape or k.shape[0] != b or k.shape[2:] != (n, d):
        raise ValueError("Expected nonempty self-attention Q/K/V with equal sequence and channel dimensions")
    if h % k.shape[1] or d > 256:
        raise ValueError("Query heads must be divisible by KV heads; head dimension must be <= 256")
    if any(t.device != q.device or t.dtype != q.dtype for t in (k, v)):
        raise ValueError("Q/K/V must have the same device and dtype")
    if not q.is_cuda or q.dtype not in (torch.float16, torch.bfloat16):
        raise ValueError("CUDA fp16 or bf16 inputs required")
    if torch.is_grad_enabled() and any(t.requires_grad for t in (q, k, v)):
        raise ValueError("Inference only: no backward implementation")


def _check_prefill_args(recency_decay, observation_window, block_q, block_k, scale, d):
    # prefill.py:117-126
    recency_decay = float(recency_decay)
    if not math.isfinite(recency_decay) or recency_decay < 0:
        raise ValueError("recency_decay must be finite and nonnegative")
    if isinstance(observation_window, bool) or not isinstance(observation_window, int) or observation_window < 0:
        raise ValueError("observation_window must be a nonnegative integer; 0 means all queries")
    if block_q not in (16, 32, 64) or block_k not in (32, 64, 128):
        raise ValueError("Unsupported tile dimensions")
    scale = d ** -0.5 if scale is None else float(scale)
    if not math.isfinite(scale):
        raise ValueError("scale must be finite")
    return recency_decay, scale


def _check_select_args(n, budget, recent, reserved_recent, pool_kernel):
    # prefill.py:149-159
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


def _tma_view(t):
    """A view (or, if unavoidable, a copy) the TMA tensor maps accept:
    channel stride 1, other strides multiples of 8 elements, 16-byte base."""
    def ok(x):
        if x.stride(-1) != 1 and x.shape[-1] != 1:
            return False
        if x.data_ptr() % 16:
            return False
        return all(s % 8 == 0 or sz == 1 for s, sz in zip(x.stride()[:3], x.shape[:3]))

    if ok(t) and t.stride(-1) == 1:
        return t
    c = t.contiguous()
    if ok(c) and c.stride(-1) == 1:
        return c
    # channels not a multiple of 8: pad the row pitch; the kernels read only
    # the first `channels` values of each row.
    d = t.shape[-1]
    d8 = (d + 7) // 8 * 8
    padded = torch.zeros(t.shape[:-1] + (d8,), dtype=t.dtype, device=t.device)
    padded[..., :d].copy_(t)
    return padded[..., :d]


def _stream(device):
    return torch.cuda.current_stream(device).cuda_stream


def _dtype_code(dtype):
    return _lib.DTYPE_BF16 if dtype == torch.bfloat16 else _lib.DTYPE_F16


def _blocks_arg(query_blocks):
    if query_blocks is None:
        return None, 0
    return query_blocks.data_ptr(), int(query_blocks.numel())


def _attention(q, k, v, out, row_stats, causal, scale, query_blocks=None):
    lib = _lib.load()
    b, h, n, d = q.shape
    qb, nqb = _blocks_arg(query_blocks)
    _lib.check(lib.fe_attention_fwd(
        q.data_ptr(), _lib.strides(q), k.data_ptr(), _lib.strides(k), v.data_ptr(), _lib.strides(v),
        out.data_ptr(), row_stats.data_ptr(), b, h, k.shape[1], n, d, _dtype_code(q.dtype), 1 if causal else 0,
        float(scale), qb, nqb, _stream(q.device)))


def _replay(q, k, v, row_stats, importance, causal, scale, recency_decay, observation_window, value_weighted,
            query_blocks=None, key_tiles=None):
    """Importance replay; key_tiles=(begin, end) restricts it to those
    128-key tiles (the rest of `importance` is left untouched)."""
    lib = _lib.load()
    b, h, n, d = q.shape
    qb, nqb = _blocks_arg(query_blocks)
    kt0, kt1 = key_tiles if key_tiles is not None else (0, (n + 127) // 128)
    _lib.check(lib.fe_replay_scores_range(
        q.data_ptr(), _lib.strides(q), k.data_ptr(), _lib.strides(k), v.data_ptr(), _lib.strides(v),
        row_stats.data_ptr(), importance.data_ptr(), b, h, k.shape[1], n, d, _dtype_code(q.dtype),
        1 if causal else 0, float(scale), float(recency_decay), int(observation_window),
        1 if value_weighted else 0, qb, nqb, int(kt0), int(kt1), _stream(q.device)))


def _select(importance, budget, recent, pool_kernel, evict_mask):
    lib = _lib.load()
    n = importance.shape[-1]
    scores = importance if importance.dtype == torch.float32 else importance.float()
    scores = scores.contiguous()
    rows = scores.numel() // n
    indices = torch.empty(importance.shape[:-1] + (budget,), dtype=torch.int64, device=importance.device)
    mask = torch.empty(importance.shape, dtype=torch.bool, device=importance.device)
    if rows:
        with torch.cuda.device(importance.device):
            _lib.check(lib.fe_select_tokens(
                scores.data_ptr(), rows, n, budget, recent, pool_kernel, indices.data_ptr(), mask.data_ptr(),
                1 if evict_mask else 0, _stream(importance.device)))
    return indices, mask


def prefill(q, k, v, *, causal=True, value_weighted=True, score=True,
            scale=None, block_q=32, block_k=64, recency_decay=0., observation_window=0):
    """Return (attention output, FP32 importance [B, Hkv, N] or None).

    I[b,h,k] = ||V[b,h,k]||_1 * sum_(g,q) w[q] softmax(Q K^T)[b,h,g,q,k],
    w[q] = exp(recency_decay * (q - (N-1))), restricted to the last
    observation_window queries when it is nonzero.  value_weighted=False gives
    the H2O attention mass.  Same contract as the reference's prefill
    (prefill.py:102-137); importance is deterministic (no atomics).
    """
    _validate(q, k, v)
    recency_decay, scale = _check_prefill_args(recency_decay, observation_window, block_q, block_k, scale,
                                               q.shape[-1])
    b, h, n, d = q.shape
    out = torch.empty(q.shape, dtype=q.dtype, device=q.device)
    row_stats = torch.empty((b, h, n, 2), dtype=torch.float32, device=q.device)
    importance = torch.empty((b, k.shape[1], n), dtype=torch.float32, device=q.device) if score else None
    qv, kv, vv = _tma_view(q), _tma_view(k), _tma_view(v)
    with torch.cuda.device(q.device):
        _attention(qv, kv, vv, out, row_stats, causal, scale)
        if score:
            _replay(qv, kv, vv, row_stats, importance, causal, scale, recency_decay, observation_window,
                    value_weighted)
    return out, importance


def select_tokens(importance, budget, *, recent=0, reserved_recent=None, pool_kernel=1):
    """Return chronologically sorted kept indices and a bool KEEP mask.

    Same contract as the reference (prefill.py:140-170); ties are broken by
    larger value, then lower index.  `recent` reserves a suffix inside the
    budget (`reserved_recent` is an alias); pool_kernel > 1 average-pools the
    past scores as SnapKV does.
    """
    n = importance.shape[-1]
    recent = _check_select_args(n, budget, recent, reserved_recent, pool_kernel)
    if not importance.is_cuda:
        raise ValueError("select_tokens requires a CUDA importance tensor")
    return _select(importance, budget, recent, pool_kernel, evict_mask=False)


def evict(q, k, v, budget, *, recent=0, reserved_recent=None, pool_kernel=1, **kwargs):
    """Return output, importance, kept indices, and bool eviction mask (True=evict)."""
    return _evict_impl(q, k, v, budget, recent, reserved_recent, pool_kernel, None, kwargs)


def _evict_impl(q, k, v, budget, recent, reserved_recent, pool_kernel, marks, kwargs, compact=False):
    """Body of `evict` (reference prefill.py:173-180): prefill then selection,
    with the eviction mask written directly by the selection kernel.
    `marks`, when given, is called with a stage name before the first launch
    and after each launch (bench.py places CUDA events there).  With
    compact=True the selection launch also gathers the kept K/V rows and two
    more tensors are returned (flash_evict.compact.evict_compact)."""
    if kwargs.get("score") is False:
        raise ValueError("evict requires importance scoring")
    kwargs = dict(kwargs)
    kwargs.pop("score", None)
    causal = kwargs.pop("causal", True)
    value_weighted = kwargs.pop("value_weighted", True)
    recency_decay = kwargs.pop("recency_decay", 0.)
    observation_window = kwargs.pop("observation_window", 0)
    block_q = kwargs.pop("block_q", 32)
    block_k = kwargs.pop("block_k", 64)
    scale = kwargs.pop("scale", None)
    if kwargs:
        raise TypeError(f"prefill() got unexpected keyword arguments {sorted(kwargs)}")
    _validate(q, k, v)
    recency_decay, scale = _check_prefill_args(recency_decay, observation_window, block_q, block_k, scale,
                                               q.shape[-1])
    b, h, n, d = q.shape
    hk = k.shape[1]
    recent = _check_select_args(n, budget, recent, reserved_recent, pool_kernel)
    out = torch.empty(q.shape, dtype=q.dtype, device=q.device)
    row_stats = torch.empty((b, h, n, 2), dtype=torch.float32, device=q.device)
    importance = torch.empty((b, hk, n), dtype=torch.float32, device=q.device)
    indices = torch.empty((b, hk, budget), dtype=torch.int64, device=q.device)
    eviction_mask = torch.empty((b, hk, n), dtype=torch.bool, device=q.device)
    qv, kv, vv = _tma_view(q), _tma_view(k), _tma_view(v)
    lib = _lib.load()
    with torch.cuda.device(q.device):
        if marks:
            marks("start")
        _attention(qv, kv, vv, out, row_stats, causal, scale)
        if marks:
            marks("attention")
        _replay(qv, kv, vv, row_stats, importance, causal, scale, recency_decay, observation_window,
                value_weighted)
        if marks:
            marks("replay")
        if compact:
            k_kept = torch.empty((b, hk, budget, d), dtype=k.dtype, device=q.device)
            v_kept = torch.empty_like(k_kept)
            _lib.check(lib.fe_select_gather(
                importance.data_ptr(), b, hk, n, budget, recent, pool_kernel, indices.data_ptr(),
                eviction_mask.data_ptr(), 1, kv.data_ptr(), _lib.strides(kv), vv.data_ptr(), _lib.strides(vv),
                k_kept.data_ptr(), v_kept.data_ptr(), d, kv.element_size(), _stream(q.device)))
        else:
            _lib.check(lib.fe_select_tokens(
                importance.data_ptr(), b * hk, n, budget, recent, pool_kernel, indices.data_ptr(),
                eviction_mask.data_ptr(), 1, _stream(q.device)))
        if marks:
            marks("select")
    if compact:
        return out, importance, indices, eviction_mask, k_kept, v_kept
    return out, importance, indices, eviction_mask
