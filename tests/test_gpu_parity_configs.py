"""GPU parity at the BASELINE configurations c2-c5, full sizes, against the
float64 oracle (oracle/restate.py, a query-chunked restatement of the
reference's flash_evict/reference.py:5-25), with the tolerances stated here.

Per configuration: sampled attention-output rows, every key's importance of
the sampled KV heads (all of their scored query rows), and the keep mask of
those heads against the oracle's selection on the oracle's importance (the
reference's select_tokens, prefill.py:140-170).  The figures are printed in
the terminal summary.

Stated tolerances (importance relative error over keys whose reference
importance is at least 1e-9 of its row's largest; below that, absolute error
at most 1e-6 of the row's largest):
  c2, c3, c4: importance rtol 1e-5 (measured on B200: 1.6e-6, 4.7e-6, 1.9e-6);
  c5: importance rtol 1e-4 (measured 4.0e-5).  Its queries are scaled x30,
      so the unscaled dot products reach |q.k| ~ 300-400 and the log2-domain
      exponents ~150: FP32 accumulation of the dot products (what the tensor
      cores, like the reference's Triton kernel, do) and the FP32 rounding of
      exponent arguments of that size (ulp 1.5e-5) put a few 1e-5 of relative
      error into every exponential.
  Attention output: max-abs <= 2e-2 (the north star's bound), and max-abs
      relative to the largest |output| <= 5e-3 (bf16 output rounding is
      2^-9 relative).
  Keep masks: exact except near ties (reference scores within 1e-5 of the
      selection threshold); the mismatch count is recorded.
"""
import numpy as np
import pytest
import torch

from common import record_figures
from flash_evict import evict
from oracle import restate as O

pytestmark = pytest.mark.gpu

REL_FLOOR = 1e-9


def _gen(shape, seed, dtype, scale=1.0):
    g = torch.Generator().manual_seed(seed)
    return (torch.randn(shape, generator=g) * scale).to(dtype)


def _parity(name, q, k, v, budget, units, rows, imp_rtol, **kw):
    causal = kw.pop("causal", True)
    pool = kw.pop("pool_kernel", 1)
    recent = kw.pop("reserved_recent", 0)
    out, imp, idx, mask = evict(q, k, v, budget, causal=causal, pool_kernel=pool, reserved_recent=recent, **kw)
    torch.cuda.synchronize()
    d = q.shape[-1]
    g = q.shape[1] // k.shape[1]
    scale = float(np.float32(d ** -0.5))  # the reference multiplies FP32 logits by an FP32 scale
    total = {"out_max_abs": 0.0, "out_max_rel": 0.0, "importance_max_rel": 0.0, "importance_keys_checked": 0,
             "mask_mismatches": 0, "mismatches_near_ties": 0}
    for b, h in units:
        ro, ri = O.chunked(q[b:b + 1, h * g:(h + 1) * g].cpu(), k[b:b + 1, h:h + 1].cpu(),
                           v[b:b + 1, h:h + 1].cpu(), causal=causal, out_rows=rows, scale=scale,
                           recency_decay=kw.get("recency_decay", 0.0),
                           observation_window=kw.get("observation_window", 0),
                           value_weighted=kw.get("value_weighted", True), weight_floor=1e-30)
        figs = O.parity_figures(out[b, h * g:(h + 1) * g][:, rows].float().cpu().numpy(), ro[0][:, rows],
                                imp[b, h].cpu().numpy(), ri[0, 0], rel_floor=REL_FLOOR)
        sel = O.selection_figures((~mask[b, h]).cpu().numpy(), ri[0, 0], budget, reserved_recent=recent,
                                  pool_kernel=pool, tie_rtol=imp_rtol)
        assert figs["importance_nonfinite"] == 0
        assert figs["importance_small_max_abs_over_rowmax"] <= 1e-6, figs
        for key in ("out_max_abs", "out_max_rel", "importance_max_rel"):
            total[key] = max(total[key], figs[key])
        total["importance_keys_checked"] += figs["importance_keys_checked"]
        total["mask_mismatches"] += sel["mask_mismatches"]
        total["mismatches_near_ties"] += sel["mismatches_near_ties"]
        assert sel["mask_mismatches"] == sel["mismatches_near_ties"], (name, b, h, sel)
        assert torch.equal(idx[b, h], torch.nonzero(~mask[b, h]).flatten())
    record_figures(f"{name} ({len(units)} kv heads)", total)
    assert total["out_max_abs"] <= 2e-2, total
    assert total["out_max_rel"] <= 5e-3, total
    assert total["importance_max_rel"] <= imp_rtol, total
    assert (~mask).sum(-1).eq(budget).all()
    return total


def test_config2_llama_8k():
    # B1 Hq32 Hkv8 N8192 D128 bf16 causal, q,k ~ N(0,1)/D^0.25, decay 0.1, reserved 64, budget 1024
    n, d = 8192, 128
    q = (_gen((1, 32, n, d), 0, torch.float32) / d ** 0.25).to(torch.bfloat16).cuda()
    k = (_gen((1, 8, n, d), 1, torch.float32) / d ** 0.25).to(torch.bfloat16).cuda()
    v = _gen((1, 8, n, d), 2, torch.bfloat16).cuda()
    rows = np.unique(np.r_[0, 1, 127, 128, 4095, n - 1, np.random.default_rng(0).integers(0, n, 10)])
    _parity("c2", q, k, v, 1024, [(0, 0), (0, 5)], rows, 1e-5, recency_decay=0.1, reserved_recent=64)


def test_config3_qwen_32k():
    # B1 Hq28 Hkv4 N32768 D128 fp16 causal, 1% of k rows x8, window 128, pool 5, budget 2048
    n, d = 32768, 128
    q = _gen((1, 28, n, d), 0, torch.float16).cuda()
    k = _gen((1, 4, n, d), 1, torch.float32)
    sink = torch.randperm(n, generator=torch.Generator().manual_seed(3))[: n // 100]
    k[:, :, sink] *= 8
    k = k.to(torch.float16).cuda()
    v = _gen((1, 4, n, d), 2, torch.float16).cuda()
    rows = np.unique(np.r_[0, 255, 256, n - 129, n - 1, np.random.default_rng(1).integers(0, n, 8)])
    _parity("c3", q, k, v, 2048, [(0, 0), (0, 3)], rows, 1e-5, observation_window=128, pool_kernel=5)


def test_config4_131k():
    # B1 Hq32 Hkv8 N131072 D128 bf16 causal, q/k/v ~ N(0,1), decay 0.1, reserved 64, budget 1024.
    # Every scored row (weight above 1e-30: the last ~690 rows) of kv heads 0
    # and 7 (four query heads each) enters the oracle's importance.
    n, d = 131072, 128
    q = _gen((1, 32, n, d), 0, torch.bfloat16).cuda()
    k = _gen((1, 8, n, d), 1, torch.bfloat16).cuda()
    v = _gen((1, 8, n, d), 2, torch.bfloat16).cuda()
    rows = np.unique(np.r_[0, 1, 255, 65535, n - 1000, n - 2, n - 1, np.random.default_rng(2).integers(0, n, 6)])
    _parity("c4", q, k, v, 1024, [(0, 0), (0, 7)], rows, 1e-5, recency_decay=0.1, reserved_recent=64)


def test_config5_batched_mha_noncausal_h2o():
    # B8 Hq=Hkv=32 N4096 D128 fp16 noncausal, [B,N,H,D] strides, q x30, 5% zero v rows, H2O, budget 410
    b, h, n, d = 8, 32, 4096, 128
    q = (_gen((b, n, h, d), 0, torch.float32) * 30).to(torch.float16).cuda().transpose(1, 2)
    k = _gen((b, n, h, d), 1, torch.float16).cuda().transpose(1, 2)
    v = _gen((b, n, h, d), 2, torch.float32)
    zero = torch.randperm(n, generator=torch.Generator().manual_seed(4))[: n * 5 // 100]
    v[:, zero] = 0
    v = v.to(torch.float16).cuda().transpose(1, 2)
    tot = _parity("c5", q, k, v, 410, [(0, 0), (3, 17), (7, 31), (5, 2)], np.r_[0, 1, 2047, n - 1], 1e-4,
                  causal=False, value_weighted=False)
    assert tot["importance_keys_checked"] > 4 * 3500
    # size-independent over every unit: the H2O mass of each (b, h) sums to N
    _, imp, _, _ = evict(q, k, v, 410, causal=False, value_weighted=False)
    torch.testing.assert_close(imp.double().sum(-1), torch.full((b, h), float(n), dtype=torch.float64,
                                                                device="cuda"), rtol=1e-5, atol=1e-3)
