"""Pins the CPU oracle (oracle/restate.py) to the reference's own outputs.

The fixtures in tests/golden/ were produced by the reference package
(tests/golden/make_golden.py): reference.py:materialized, prefill.py:
select_tokens, baselines.snap_select, and the reference's Triton kernel run
by the Triton CPU interpreter.  CPU only.
"""
import math
import os

import numpy as np
import pytest
import torch
import torch.nn.functional as F

from common import GOLDEN, golden_cases, load_case, snap_cases
from oracle import restate as O


@pytest.mark.parametrize("name", golden_cases())
def test_oracle_materialized_matches_reference(name):
    c = load_case(name)
    out, mass = O.materialized(c["q_t"], c["k_t"], c["v_t"], causal=c["causal"], **c["kwargs"])
    np.testing.assert_allclose(out, c["out"], atol=2e-5, rtol=1e-5)
    np.testing.assert_allclose(mass, c["mass"], atol=1e-4, rtol=2e-5)


@pytest.mark.parametrize("name", golden_cases())
def test_oracle_chunked_matches_reference(name):
    c = load_case(name)
    # float64 here: closer to the truth than the reference's float32, so the
    # extreme-logit case (logits ~1e3) differs from it by ~1e-4.
    out, mass = O.chunked(c["q_t"], c["k_t"], c["v_t"], causal=c["causal"], chunk=64, **c["kwargs"])
    np.testing.assert_allclose(out, c["out"], atol=2e-4, rtol=1e-5)
    np.testing.assert_allclose(mass, c["mass"], atol=1e-3, rtol=1e-4)


@pytest.mark.parametrize("name", golden_cases())
def test_oracle_selection_on_reference_scores(name):
    c = load_case(name)
    for bud in c["budgets"]:
        idx, keep = O.select_tokens(c["mass"], int(bud))
        np.testing.assert_array_equal(idx, c[f"idx_{bud}"])
        np.testing.assert_array_equal(keep, c[f"keep_{bud}"])


def test_oracle_selection_fixtures():
    z = np.load(os.path.join(GOLDEN, "selection.npz"))
    idx, keep = O.select_tokens(z["pin_scores"], 48, reserved_recent=32, pool_kernel=5)
    np.testing.assert_array_equal(idx, z["pin_idx"])
    np.testing.assert_array_equal(keep, z["pin_keep"])
    for j in range(int(z["ncases"])):
        bud, rec, pk = (int(x) for x in z[f"c{j}_args"])
        idx, keep = O.select_tokens(z[f"c{j}_scores"], bud, reserved_recent=rec, pool_kernel=pk)
        np.testing.assert_array_equal(idx, z[f"c{j}_idx"])
        np.testing.assert_array_equal(keep, z[f"c{j}_keep"])
    idx, keep = O.select_tokens(np.arange(20.).reshape(1, 1, 20), 4, recent=2)
    np.testing.assert_array_equal(idx, z["contract_idx"])
    assert idx.tolist() == [[[16, 17, 18, 19]]]


def test_oracle_matches_reference_triton_kernel():
    """The reference kernel (two traversals, FP32 atomics) run by the Triton
    interpreter agrees with the materialized restatement."""
    z = np.load(os.path.join(GOLDEN, "triton_interp.npz"))
    for j in range(int(z["ncases"])):
        n, h, hk, d, causal, weighted, decay, window = z[f"i{j}_args"]
        q, k, v = (torch.from_numpy(z[f"i{j}_{x}"].view(np.int16)).view(torch.float16) for x in "qkv")
        out, mass = O.materialized(q, k, v, causal=bool(causal), value_weighted=bool(weighted),
                                   recency_decay=float(decay), observation_window=int(window))
        np.testing.assert_allclose(z[f"i{j}_out"], out, atol=2e-3, rtol=6e-3)
        np.testing.assert_allclose(z[f"i{j}_imp"], mass, atol=3e-3 if weighted else 3e-5, rtol=3e-4)


@pytest.mark.parametrize("kernel", [3, 5, 7, 9])
def test_avg_pool_bitexact_vs_torch(kernel):
    g = torch.Generator().manual_seed(kernel)
    x = torch.randn(5, 777, generator=g) * 100
    ref = F.avg_pool1d(x.reshape(-1, 1, 777), kernel, stride=1, padding=kernel // 2).reshape_as(x).numpy()
    mine = O.avg_pool(x.numpy(), kernel)
    assert np.array_equal(ref.view(np.uint32), mine.view(np.uint32))


def test_order_keys():
    x = np.array([-np.inf, -3.5, -1e-30, -0.0, 0.0, 1e-30, 2.0, np.inf, np.nan], dtype=np.float32)
    k = O.order_keys(x)
    assert (np.diff(k[:4].astype(np.int64)) > 0).all()
    assert k[3] == k[4]                      # -0.0 ties +0.0
    assert (np.diff(k[4:].astype(np.int64)) > 0).all()
    assert k[-1] == 0xFFFFFFFF               # NaN is the largest


def test_selection_tie_break_lower_index():
    s = np.array([[1., 3., 3., 2., 3., 0.]], dtype=np.float32)
    idx, keep = O.select_tokens(s, 2)
    assert idx.tolist() == [[1, 2]]
    idx, _ = O.select_tokens(s, 4)
    assert idx.tolist() == [[1, 2, 3, 4]]


def test_normalization_counterexample():
    # Restates tests/test_prefill.py:62-74 of the reference: column sums need
    # each query's final normaliser.
    logits = torch.tensor([[0., 0.], [0., math.log(9.)]])
    normalized = logits.softmax(-1).sum(0)
    prematurely_summed = logits.exp().sum(0)
    assert torch.allclose(normalized, torch.tensor([.6, 1.4]))
    assert not torch.allclose(normalized, prematurely_summed / prematurely_summed.sum() * 2)
    causal_logits = torch.tensor([[math.log(9.), -torch.inf], [math.log(100.), math.log(200.)]])
    assert causal_logits.softmax(-1).sum(0).argmax() == 0
    assert causal_logits.exp().sum(0).argmax() == 1


def test_analytic_forms_match_materialized():
    n, g = 300, 2
    v = torch.randn(1, 1, n, 16, generator=torch.Generator().manual_seed(3))
    q = torch.zeros(1, g, n, 16)
    k = torch.zeros(1, 1, n, 16)
    out, mass = O.materialized(q, k, v, dtype=np.float64)
    aout, amass = O.uniform_analytic(v, g)
    np.testing.assert_allclose(out[0, 0], aout[0, 0], rtol=1e-10, atol=1e-12)
    np.testing.assert_allclose(mass, amass, rtol=1e-10)
    for decay, window in ((.01, 0), (0., 128), (.1, 65)):
        _, m = O.materialized(q, k, torch.ones_like(v), recency_decay=decay, observation_window=window,
                              dtype=np.float64)
        exp = O.weighted_analytic(n, decay, window, g, 16.0)
        np.testing.assert_allclose(m[0, 0], exp, rtol=1e-8, atol=1e-14)


def test_flop_and_row_accounting():
    assert O.attention_flops(1, 28, 32768, 128, True) == 4 * 28 * 128 * (32768 * 32769 // 2)
    rows = O.scored_rows(32768, 0.0, 128)
    assert rows[0] == 32768 - 128 and len(rows) == 128
    rows = O.scored_rows(8192, 0.1, 0)
    assert 860 < len(rows) < 890
    assert O.replay_flops(1, 28, 32768, 128, True, O.scored_rows(32768, 0.0, 128)) > 2.9e10


def test_oracle_snap_matches_reference_fixtures():
    # the reference's baselines.snap_scores / snap_select run here (torch, CPU)
    for c in snap_cases():
        s = O.snap_scores(c["q"].float().numpy(), c["k"].float().numpy(), c["window"], c["dtype_name"])
        np.testing.assert_allclose(s, c["scores"], rtol=2e-5, atol=1e-7, err_msg=c["name"])
        idx, keep = O.snap_select(c["scores"], c["budget"], c["window"])
        np.testing.assert_array_equal(idx, c["idx"], err_msg=c["name"])
        np.testing.assert_array_equal(keep, c["keep"], err_msg=c["name"])


def test_round_to_dtype_matches_torch():
    x = (torch.randn(10000, generator=torch.Generator().manual_seed(2)) * 300).float()
    for name, dt in (("float16", torch.float16), ("bfloat16", torch.bfloat16)):
        np.testing.assert_array_equal(O.round_to_dtype(x.numpy(), name), x.to(dt).float().numpy())


def test_parity_and_selection_figures_helpers():
    # The figure helpers the GPU parity tests and bench.py report with.
    ref = np.array([[4.0, 3.0, 2.0, 1.0, 1e-12, 0.5]], dtype=np.float64)
    got = ref * (1 + np.array([[1e-6, -2e-6, 0, 0, 0.5, 3e-6]]))
    f = O.parity_figures(np.ones(3), np.ones(3) * 1.001, got, ref, rel_floor=1e-9)
    assert abs(f["importance_max_rel"] - 3e-6) < 1e-12
    assert f["importance_keys_checked"] == 5          # 1e-12 < 1e-9 * 4
    assert f["importance_small_max_abs_over_rowmax"] == pytest.approx(0.5e-12 / 4.0)
    assert f["out_max_abs"] == pytest.approx(0.001)
    # a keep mask that swaps the threshold token with a near tie
    imp = np.array([[5.0, 4.0, 3.0, 3.0 * (1 - 1e-7), 1.0]], dtype=np.float32)
    keep = np.array([[True, True, False, True, False]])
    s = O.selection_figures(keep, imp, 3, tie_rtol=1e-5)
    assert s["mask_mismatches"] == 2 and s["mismatches_near_ties"] == 2
    s = O.selection_figures(np.array([[True, False, True, True, False]]), imp, 3, tie_rtol=1e-5)
    assert s["mask_mismatches"] == 2 and s["mismatches_near_ties"] == 1


def test_cpu_baseline_sample_and_flops():
    # The timed CPU baseline (bench.py): a fixed sample, FLOPs counted with
    # the GPU metric's formula, and the arithmetic of the oracle.
    from oracle import cpu_baseline as C
    plan = C.sample_plan(1, 4, 2, 512, 64, True, target_flops=4 * 64 * 2 * 512 * 300)
    assert plan[0][:2] == (0, 0) and plan[0][2] % 256 == 0
    g = torch.Generator().manual_seed(1)
    q = torch.randn(1, 4, 512, 64, generator=g)
    k = torch.randn(1, 2, 512, 64, generator=g)
    v = torch.randn(1, 2, 512, 64, generator=g)
    units = C.prepare(q, k, v, [(0, 0, 0)])
    fl, _ = C.run(units, 512, True, 0.125, 0.0, 0, True)
    keys = 512 * 513 // 2
    assert fl == 2 * (4 * 64 * keys + 2 * 64 * keys)
