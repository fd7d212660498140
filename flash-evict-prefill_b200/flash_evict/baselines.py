"""Drop-in for the reference's SnapKV baseline (flash_evict/baselines.py).

Same names, signatures, defaults and return values as the reference:

  flash_attention(q, k, v)                   causal GQA attention (baselines.py:7-9;
                                             the reference forces torch's flash SDPA)
                                             -> fe_attention_fwd
  snap_scores(q, k, window=32)               baselines.py:12-26 -> fe_snap_scores
  snap_select(scores, budget, window=32, kernel=5)
                                             baselines.py:29-43 -> fe_select_tokens
  flash_snap(q, k, v, budget, window=32)     baselines.py:46-50

snap_scores keeps the reference's arithmetic: the window logits are rounded
to the input dtype (its matmul runs in fp16/bf16) before the FP32 scale,
causal mask and softmax; the w x N matrix is never materialised.  Arguments
the reference would reject only deep inside torch (window 0, an even pooling
kernel) raise ValueError here.
"""
import torch

from . import _lib
from .prefill import _attention, _select, _stream, _tma_view, _validate, _dtype_code

__all__ = ["flash_attention", "snap_scores", "snap_select", "flash_snap"]


def flash_attention(q, k, v):
    """Causal attention with grouped KV heads, scale D**-0.5 (baselines.py:7-9)."""
    _validate(q, k, v)
    b, h, n, d = q.shape
    out = torch.empty(q.shape, dtype=q.dtype, device=q.device)
    row_stats = torch.empty((b, h, n, 2), dtype=torch.float32, device=q.device)
    with torch.cuda.device(q.device):
        _attention(_tma_view(q), _tma_view(k), _tma_view(v), out, row_stats, True, d ** -0.5)
    return out


def _check_window(window):
    if isinstance(window, bool) or not isinstance(window, int) or window < 1:
        raise ValueError("window must be a positive integer")


def snap_scores(q, k, window=32):
    """Observation-window attention mass per KV token, mean over grouped heads.

    FP32 [B, Hkv, N]: for the last min(window, N) queries, softmax of the
    causal logits (native-dtype QK^T, then FP32 * D**-0.5), summed over the
    window rows and averaged over the G query heads of each KV head.
    """
    _validate(q, k, k)
    _check_window(window)
    b, h, n, d = q.shape
    hk = k.shape[1]
    lib = _lib.load()
    wsz = lib.fe_snap_workspace_floats(b, h, hk, n, window)
    if wsz < 0:
        _lib.check(_lib.STATUS_INVALID)
    scores = torch.empty((b, hk, n), dtype=torch.float32, device=q.device)
    workspace = torch.empty(max(int(wsz), 2), dtype=torch.float32, device=q.device)
    qv, kv = _tma_view(q), _tma_view(k)
    with torch.cuda.device(q.device):
        _lib.check(lib.fe_snap_scores(
            qv.data_ptr(), _lib.strides(qv), kv.data_ptr(), _lib.strides(kv), scores.data_ptr(),
            workspace.data_ptr(), workspace.numel(), b, h, hk, n, d, _dtype_code(q.dtype), float(d ** -0.5),
            window, _stream(q.device)))
    return scores


def _snap_select(scores, budget, window, kernel, evict_mask):
    if isinstance(budget, bool) or not isinstance(budget, int) or budget < 1:
        raise ValueError("budget must be a positive integer")
    if isinstance(window, bool) or not isinstance(window, int) or window < 0:
        raise ValueError("window must be a nonnegative integer")
    if isinstance(kernel, bool) or not isinstance(kernel, int) or kernel < 1 or kernel % 2 != 1:
        raise ValueError("kernel must be a positive odd integer")
    if not scores.is_cuda:
        raise ValueError("snap_select requires a CUDA score tensor")
    n = scores.shape[-1]
    if n <= budget:
        # baselines.py:31-32: every token kept
        idx = torch.arange(n, device=scores.device).expand(*scores.shape[:-1], n)
        keep = torch.ones(scores.shape, dtype=torch.bool, device=scores.device)
        return idx, (~keep if evict_mask else keep)
    # baselines.py:34-39: the window suffix is reserved inside the budget and
    # the past is average-pooled before the top-k (kernel 1 pools as identity)
    window = min(window, n, budget - 1)
    return _select(scores, budget, window, kernel, evict_mask=evict_mask)


def snap_select(scores, budget, window=32, kernel=5):
    """Sorted kept indices and a bool KEEP mask (baselines.py:29-43)."""
    return _snap_select(scores, budget, window, kernel, evict_mask=False)


def flash_snap(q, k, v, budget, window=32):
    """(out, scores, indices, eviction_mask) of FlashAttention + SnapKV (baselines.py:46-50)."""
    out = flash_attention(q, k, v)
    scores = snap_scores(q, k, window)
    idx, evict_mask = _snap_select(scores, budget, window, 5, evict_mask=True)
    return out, scores, idx, evict_mask
