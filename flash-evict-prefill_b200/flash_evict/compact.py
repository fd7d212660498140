"""KV compaction after selection.

The reference's adapters shrink the cache right after selecting: they call
`select_tokens` and then `gather_tokens(k, indices)` / `gather_tokens(v, indices)`
from their kv_distill dependency (flash_evict/kv_distill_adapter.py:35-39,
flash_evict/streaming_adapter.py:84-86, flash_evict/quality_adapter.py:109-110).
README.md:31 states the gather as
`k.gather(2, indices[..., None].expand(-1, -1, -1, k.shape[-1]))`.

  gather_tokens(x, indices)               -> fe_gather_tokens
  select_and_gather(importance, budget, k, v, ...)
                                          -> fe_select_gather (selection and both
                                             gathers in one launch)
  evict_compact(q, k, v, budget, ...)     -> evict() whose selection launch also
                                             writes the compacted K and V

The copies are bitwise.  An index outside [0, tokens) does not fault the GPU
(torch.gather would stop it with a device assert): the destination row is
zero-filled and the device status word reports FE_STATUS_BAD_INDEX
(`flash_evict._lib.device_status`).
"""
import torch

from . import _lib
from .prefill import _check_select_args, _evict_impl, _stream

__all__ = ["gather_tokens", "select_and_gather", "evict_compact"]


def _gather_src(x):
    """A view whose channel stride is 1 (copied only when it is not)."""
    return x if x.stride(-1) == 1 else x.contiguous()


def _check_kv(k, v):
    if k.ndim != 4:
        raise ValueError("K/V must have shape [batch, heads, tokens, channels]")
    if v is not None and (v.shape != k.shape or v.dtype != k.dtype or v.device != k.device):
        raise ValueError("K and V must have the same shape, dtype and device")
    if not k.is_cuda:
        raise ValueError("KV compaction requires CUDA tensors")


def gather_tokens(x, indices):
    """x[b, h, indices[b, h, j], :] for every j: a contiguous [B, H, budget, D] copy.

    Same result as `x.gather(2, indices[..., None].expand(-1, -1, -1, x.shape[-1]))`.
    indices: int64 [B, H, budget] on x's device, any order, repeats allowed.
    """
    _check_kv(x, None)
    if indices.ndim != 3 or tuple(indices.shape[:2]) != tuple(x.shape[:2]):
        raise ValueError("indices must have shape [batch, heads, budget] matching x")
    if indices.dtype != torch.int64 or indices.device != x.device:
        raise ValueError("indices must be an int64 tensor on x's device")
    b, h, n, d = x.shape
    budget = indices.shape[2]
    out = torch.empty((b, h, budget, d), dtype=x.dtype, device=x.device)
    if out.numel() == 0:
        return out
    if n == 0:
        raise ValueError("cannot gather from an empty token dimension")
    src = _gather_src(x)
    idx = indices.contiguous()
    lib = _lib.load()
    with torch.cuda.device(x.device):
        _lib.check(lib.fe_gather_tokens(
            src.data_ptr(), _lib.strides(src), None, None, idx.data_ptr(), out.data_ptr(), None, b, h, n, budget,
            d, src.element_size(), _stream(x.device)))
    return out


def select_and_gather(importance, budget, k, v, *, recent=0, reserved_recent=None, pool_kernel=1):
    """`select_tokens` followed by the gather of K and V, in one launch.

    importance: [B, H, N] scores for k/v [B, H, N, D].  Returns
    (indices, keep, k_kept, v_kept); indices and keep are exactly those of
    `select_tokens` with the same arguments, k_kept/v_kept are contiguous
    [B, H, budget, D].
    """
    _check_kv(k, v)
    if importance.ndim != 3 or tuple(importance.shape) != tuple(k.shape[:3]):
        raise ValueError("importance must have shape [batch, heads, tokens] matching K/V")
    if importance.device != k.device:
        raise ValueError("importance and K/V must be on the same device")
    b, h, n, d = k.shape
    recent = _check_select_args(n, budget, recent, reserved_recent, pool_kernel)
    scores = (importance if importance.dtype == torch.float32 else importance.float()).contiguous()
    indices = torch.empty((b, h, budget), dtype=torch.int64, device=k.device)
    keep = torch.empty((b, h, n), dtype=torch.bool, device=k.device)
    k_kept = torch.empty((b, h, budget, d), dtype=k.dtype, device=k.device)
    v_kept = torch.empty_like(k_kept)
    ks, vs = _gather_src(k), _gather_src(v)
    lib = _lib.load()
    with torch.cuda.device(k.device):
        _lib.check(lib.fe_select_gather(
            scores.data_ptr(), b, h, n, budget, recent, pool_kernel, indices.data_ptr(), keep.data_ptr(), 0,
            ks.data_ptr(), _lib.strides(ks), vs.data_ptr(), _lib.strides(vs), k_kept.data_ptr(), v_kept.data_ptr(),
            d, ks.element_size(), _stream(k.device)))
    return indices, keep, k_kept, v_kept


def evict_compact(q, k, v, budget, *, recent=0, reserved_recent=None, pool_kernel=1, **prefill_kwargs):
    """`evict` plus the compacted cache.

    Returns (out, importance, indices, eviction_mask, k_kept, v_kept): the
    first four exactly as `evict` with the same arguments; k_kept/v_kept are
    the kept K/V rows, [B, Hkv, budget, D], written by the selection launch.
    """
    return _evict_impl(q, k, v, budget, recent, reserved_recent, pool_kernel, None, prefill_kwargs, compact=True)
