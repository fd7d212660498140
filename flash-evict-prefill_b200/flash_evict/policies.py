"""Several selection policies in one launch.

The reference's paired controller scores a prompt once and then selects for
every method that shares the prefill, one `select_tokens` (or `snap_select`)
call per method, and gathers a compact cache for each
(flash_evict/quality_adapter.py:95-111, choose_indices at :39-51).  Here all
of them run in one selection launch (fe_select_multi); with K/V given, the
same launch also writes each policy's compacted cache.

A policy is (importance, budget, recent, pool_kernel): `importance` may be a
different score tensor per policy (fused importance, SnapKV scores, value
norms), all of one [B, H, N] shape; `recent` is the reserved suffix inside
the budget (select_tokens' `recent` / `reserved_recent`).  Each policy's
indices and mask are exactly those of `select_tokens` with the same
arguments.  Up to 8 policies per launch.
"""
import ctypes

import torch

from . import _lib
from .compact import _check_kv, _gather_src
from .prefill import _check_select_args, _stream

__all__ = ["select_tokens_multi", "select_and_gather_multi", "MAX_POLICIES"]

MAX_POLICIES = 8


def _as_list(x, n, name):
    if isinstance(x, (list, tuple)):
        if len(x) != n:
            raise ValueError(f"{name} must have one entry per policy")
        return list(x)
    return [x] * n


def _prepare(importances, budgets, recents, pool_kernels):
    if isinstance(budgets, int) and not isinstance(budgets, bool):
        budgets = [budgets]
    budgets = list(budgets)
    npol = len(budgets)
    if not 1 <= npol <= MAX_POLICIES:
        raise ValueError(f"between 1 and {MAX_POLICIES} policies per launch")
    imps = _as_list(importances, npol, "importances")
    recents = _as_list(0 if recents is None else recents, npol, "recents")
    pools = _as_list(1 if pool_kernels is None else pool_kernels, npol, "pool_kernels")
    shape, dev = imps[0].shape, imps[0].device
    if len(shape) < 1 or any(t.shape != shape or t.device != dev for t in imps):
        raise ValueError("every policy's importance must have the same shape and device")
    n = shape[-1]
    recents = [_check_select_args(n, b, r, None, p) for b, r, p in zip(budgets, recents, pools)]
    if not imps[0].is_cuda:
        raise ValueError("select_tokens_multi requires CUDA importance tensors")
    scores = [(t if t.dtype == torch.float32 else t.float()).contiguous() for t in imps]
    return npol, n, shape, dev, budgets, recents, pools, scores


def _launch(npol, n, shape, dev, budgets, recents, pools, scores, k=None, v=None):
    rows = scores[0].numel() // n
    idx = [torch.empty(shape[:-1] + (b,), dtype=torch.int64, device=dev) for b in budgets]
    keep = [torch.empty(shape, dtype=torch.bool, device=dev) for _ in budgets]
    kk = vk = None
    if k is not None:
        b_, h_, _, d = k.shape
        kk = [torch.empty((b_, h_, bud, d), dtype=k.dtype, device=dev) for bud in budgets]
        vk = [torch.empty_like(t) for t in kk]
    if rows == 0:
        return idx, keep, kk, vk
    P = ctypes.c_void_p * npol
    I = ctypes.c_int64 * npol
    lib = _lib.load()
    args_k = (None, None, None, None, None, None, 0, 0)
    if k is not None:
        ks, vs = _gather_src(k), _gather_src(v)
        args_k = (ks.data_ptr(), _lib.strides(ks), vs.data_ptr(), _lib.strides(vs),
                  P(*[t.data_ptr() for t in kk]), P(*[t.data_ptr() for t in vk]), k.shape[-1], ks.element_size())
    bh = (shape[0], rows // shape[0]) if len(shape) >= 2 else (1, rows)
    with torch.cuda.device(dev):
        _lib.check(lib.fe_select_multi(
            P(*[t.data_ptr() for t in scores]), bh[0], bh[1], n, npol, I(*budgets), I(*recents), I(*pools),
            P(*[t.data_ptr() for t in idx]), P(*[t.data_ptr() for t in keep]), 0, *args_k, _stream(dev)))
    return idx, keep, kk, vk


def select_tokens_multi(importances, budgets, recents=None, pool_kernels=None):
    """[(indices, keep)] for each policy, one launch.

    importances: one [..., N] score tensor shared by all policies, or a list
    with one per policy; budgets: list of ints; recents / pool_kernels: a
    value for all policies or a list.
    """
    npol, n, shape, dev, budgets, recents, pools, scores = _prepare(importances, budgets, recents, pool_kernels)
    idx, keep, _, _ = _launch(npol, n, shape, dev, budgets, recents, pools, scores)
    return list(zip(idx, keep))


def select_and_gather_multi(importances, budgets, k, v, recents=None, pool_kernels=None):
    """[(indices, keep, k_kept, v_kept)] for each policy, one launch.

    importances are [B, H, N] for k/v [B, H, N, D]; k_kept/v_kept are the
    policy's compact cache, contiguous [B, H, budget, D].
    """
    _check_kv(k, v)
    npol, n, shape, dev, budgets, recents, pools, scores = _prepare(importances, budgets, recents, pool_kernels)
    if tuple(shape) != tuple(k.shape[:3]) or dev != k.device:
        raise ValueError("importance must have shape [batch, heads, tokens] matching K/V, on their device")
    idx, keep, kk, vk = _launch(npol, n, shape, dev, budgets, recents, pools, scores, k, v)
    return list(zip(idx, keep, kk, vk))
