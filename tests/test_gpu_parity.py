"""GPU parity of prefill/evict against the oracle and the reference's goldens.

Restates the reference's tests/test_prefill.py cases (file:line cited per
test) with the CPU oracle (oracle/restate.py) as the ground truth.  The
tolerances are the reference's own.
"""
import math

import numpy as np
import pytest
import torch

from common import golden_cases, load_case, selection_mismatch, strided_like_model
from flash_evict import evict, prefill, select_tokens
from oracle import restate as O

pytestmark = pytest.mark.gpu


@pytest.fixture(autouse=True)
def precision():
    torch.manual_seed(731)
    torch.backends.cuda.matmul.allow_tf32 = False


def oracle(q, k, v, **kw):
    out, mass = O.materialized(q, k, v, **kw)
    return torch.from_numpy(out).cuda(), torch.from_numpy(mass).cuda()


def assert_keep_matches(keep, ref_keep, scores, ref_scores, atol, rtol):
    mism, explained = selection_mismatch(keep.cpu().numpy(), ref_keep.cpu().numpy() if torch.is_tensor(ref_keep)
                                         else ref_keep, scores.cpu().numpy(),
                                         ref_scores.cpu().numpy() if torch.is_tensor(ref_scores) else ref_scores,
                                         atol, rtol)
    assert explained, f"{mism} keep-mask mismatches not explained by near ties"
    return mism


@pytest.mark.parametrize("name", golden_cases())
def test_golden_reference_outputs(name):
    """Outputs of the reference's materialized path (tests/golden) on the same inputs."""
    c = load_case(name)
    q, k, v = (strided_like_model(c[x]).cuda() for x in ("q_t", "k_t", "v_t"))
    out, imp = prefill(q, k, v, causal=c["causal"], **c["kwargs"])
    bf = c["dtype"] == torch.bfloat16
    extreme = "x15" in name
    atol_o = 0.004 if extreme else (0.012 if bf else 0.002)
    atol_s, rtol_s = (0.01, 0.001) if extreme else (3e-3, 3e-4)
    if c["kwargs"].get("value_weighted") is False:
        atol_s = 3e-5
    torch.testing.assert_close(out.float().cpu(), torch.from_numpy(c["out"]), atol=atol_o, rtol=0.006)
    torch.testing.assert_close(imp.cpu(), torch.from_numpy(c["mass"]), atol=atol_s, rtol=rtol_s)
    for bud in c["budgets"]:
        idx, keep = select_tokens(imp, int(bud))
        assert_keep_matches(keep, c[f"keep_{int(bud)}"], imp, c["mass"], atol_s, rtol_s)
        assert keep.sum(-1).eq(int(bud)).all()


@pytest.mark.parametrize("n,h,hk,d,dtype,causal", [
    (512, 4, 4, 64, torch.float16, True),
    (1024, 4, 2, 64, torch.bfloat16, True),
    (4096, 4, 2, 128, torch.bfloat16, True),
    (137, 6, 2, 80, torch.float16, False),
    (65, 4, 1, 32, torch.bfloat16, True),
    (1, 2, 1, 16, torch.float16, True),
    # more than 128 channels: two attention launches (one per 128-channel half of V)
    (512, 4, 2, 256, torch.bfloat16, True),
    (300, 4, 2, 192, torch.float16, True),
    (257, 2, 1, 160, torch.bfloat16, False),
])
def test_exact(n, h, hk, d, dtype, causal):
    # reference tests/test_prefill.py:15-41
    q = torch.randn((1, n, h, d), device="cuda", dtype=dtype).transpose(1, 2)
    k, v = [torch.randn((1, n, hk, d), device="cuda", dtype=dtype).transpose(1, 2) for _ in range(2)]
    out, importance = prefill(q, k, v, causal=causal)
    expected, scores = oracle(q, k, v, causal=causal)
    torch.testing.assert_close(out.float(), expected, atol=0.012 if dtype == torch.bfloat16 else 0.002, rtol=0.006)
    torch.testing.assert_close(importance, scores, atol=3e-3, rtol=3e-4)
    for rate in (.05, .1, .2):
        budget = max(1, math.ceil(n * rate))
        idx, keep = select_tokens(importance, budget)
        ref_idx, ref_keep = O.select_tokens(scores.cpu().numpy(), budget)
        assert_keep_matches(keep, ref_keep, importance, scores, 3e-3, 3e-4)
        if np.array_equal(keep.cpu().numpy(), ref_keep):
            assert np.array_equal(idx.cpu().numpy(), ref_idx)
    _, hh = prefill(q, k, v, causal=causal, value_weighted=False)
    _, hh_ref = oracle(q, k, v, causal=causal, value_weighted=False)
    torch.testing.assert_close(hh, hh_ref, atol=3e-5, rtol=3e-4)
    torch.testing.assert_close(hh.sum(-1), torch.full_like(hh.sum(-1), n * h / hk), rtol=1e-5, atol=1e-4)


def test_extreme_logits_batches_and_zero_values():
    # reference tests/test_prefill.py:44-59
    q = torch.randn(2, 4, 97, 64, device="cuda", dtype=torch.float16) * 15
    k = torch.randn(2, 2, 97, 64, device="cuda", dtype=torch.float16) * 15
    v = torch.randn_like(k)
    out, scores, idx, mask = evict(q, k, v, 17, recent=5)
    ref, refscore = oracle(q, k, v)
    torch.testing.assert_close(out.float(), ref, atol=0.004, rtol=0.006)
    torch.testing.assert_close(scores, refscore, atol=0.01, rtol=0.001)
    assert torch.isfinite(scores).all()
    assert (~mask).sum(-1).eq(17).all()
    assert not mask[..., -5:].any()
    zero, zeroscore = prefill(q, k, torch.zeros_like(v))
    assert zero.count_nonzero() == 0 and zeroscore.count_nonzero() == 0
    plain, _ = prefill(q, k, v, score=False)
    assert torch.equal(plain, out)


@pytest.mark.parametrize("n,decay,window", [
    (512, .01, 0), (1024, .1, 0), (4096, 1., 0),
    (137, 0., 32), (1024, 0., 64), (4096, 0., 128),
    (137, .1, 65), (65, 1., 128), (1, .1, 32),
])
@pytest.mark.parametrize("value_weighted", [True, False])
def test_query_weighted_exact(n, decay, window, value_weighted):
    # reference tests/test_prefill.py:105-131
    q = torch.randn(1, n, 4, 64, device="cuda", dtype=torch.bfloat16).transpose(1, 2)
    k, v = [torch.randn(1, n, 2, 64, device="cuda", dtype=q.dtype).transpose(1, 2) for _ in range(2)]
    kwargs = dict(recency_decay=decay, observation_window=window, value_weighted=value_weighted)
    out, scores = prefill(q, k, v, **kwargs)
    expected, ref = oracle(q, k, v, **kwargs)
    torch.testing.assert_close(out.float(), expected, atol=.012, rtol=.006)
    torch.testing.assert_close(scores, ref, atol=3e-5, rtol=4e-4)
    plain, _ = prefill(q, k, v, score=False)
    assert torch.equal(out, plain)
    if not value_weighted:
        pos = torch.arange(n, device="cuda")
        weight = (decay * (pos.float() - (n - 1))).exp()
        if window:
            weight *= pos >= n - window
        torch.testing.assert_close(scores.sum(-1), weight.sum().expand(1, 2) * 2, rtol=1e-5, atol=1e-4)
    budget = min(n, 128)
    recent = min(64, budget)
    _, keep = select_tokens(scores, budget, reserved_recent=recent)
    _, reference_keep = O.select_tokens(ref.cpu().numpy(), budget, reserved_recent=recent)
    assert_keep_matches(keep, reference_keep, scores, ref, 3e-5, 4e-4)
    assert keep.sum(-1).eq(budget).all() and keep[..., -recent:].all()


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
def test_normalization_counterexample_through_kernels(dtype):
    # reference tests/test_prefill.py:62-74 through the kernels: logits
    # [[log 9, -], [log 100, log 200]] (causal).  Normalised column sums
    # rank key 0 first (1 + 1/3 against 2/3); unnormalised exp sums would
    # rank key 1 first.
    q = torch.zeros(1, 1, 2, 16)
    k = torch.zeros(1, 1, 2, 16)
    q[0, 0, 0, 0] = math.log(9.)
    q[0, 0, 1, 0] = math.log(100.)
    q[0, 0, 1, 1] = math.log(200.)
    k[0, 0, 0, 0] = 1.
    k[0, 0, 1, 1] = 1.
    v = torch.ones(1, 1, 2, 16)
    q, k, v = (t.to(dtype).cuda() for t in (q, k, v))
    out, scores = prefill(q, k, v, scale=1.0, value_weighted=False)
    _, ref = O.materialized(q.float().cpu().numpy(), k.float().cpu().numpy(), v.float().cpu().numpy(), scale=1.0,
                            value_weighted=False)
    np.testing.assert_allclose(scores.cpu().numpy(), ref, rtol=3e-4, atol=3e-5)
    assert scores[0, 0].argmax().item() == 0
    idx, keep = select_tokens(scores, 1)
    assert idx.flatten().tolist() == [0]
    logits = (q.float() @ k.float().transpose(-1, -2))[0, 0]
    assert torch.tril(logits.exp()).sum(0).argmax().item() == 1


@pytest.mark.parametrize("n", [8192, 32768, 131072])
def test_long_uniform_analytic(n):
    # reference tests/test_prefill.py:88-102: Q=K=0 closed form
    q = torch.zeros(1, 2, n, 16, device="cuda", dtype=torch.bfloat16)
    k = torch.zeros(1, 1, n, 16, device="cuda", dtype=q.dtype)
    v = torch.randn_like(k)
    out, scores = prefill(q, k, v)
    positions = torch.arange(1, n + 1, device="cuda", dtype=torch.float64)
    expected_out = (v.double().cumsum(2) / positions[None, None, :, None]).expand_as(out)
    harmonic = positions.reciprocal().flip(0).cumsum(0).flip(0)
    expected_scores = (v.double().abs().sum(-1) * harmonic * 2).float()
    torch.testing.assert_close(out.float(), expected_out.float(), atol=.008, rtol=.008)
    torch.testing.assert_close(scores, expected_scores, atol=.002, rtol=.0003)


def test_evict_one_million_tokens():
    # Q=K=0 closed form at N = 2^20 through evict(): uniform causal attention,
    # H2O importance = sum over q >= k of 1/(q+1); the past region is longer
    # than the selection's shared-memory slices
    n = 1 << 20
    q = torch.zeros(1, 1, n, 16, device="cuda", dtype=torch.float16)
    k = torch.zeros(1, 1, n, 16, device="cuda", dtype=q.dtype)
    v = torch.randn(1, 1, n, 16, generator=torch.Generator().manual_seed(5)).to(q.dtype).cuda()
    out, scores, idx, mask = evict(q, k, v, 4096, reserved_recent=64, value_weighted=False)
    positions = torch.arange(1, n + 1, device="cuda", dtype=torch.float64)
    rows = torch.tensor([0, 1, 4095, 777777, n - 1], device="cuda")
    expected_out = v.double().cumsum(2)[:, :, rows] / positions[rows][None, None, :, None]
    torch.testing.assert_close(out[:, :, rows].float(), expected_out.float(), atol=.004, rtol=.004)
    expected = positions.reciprocal().flip(0).cumsum(0).flip(0).float()
    torch.testing.assert_close(scores[0, 0], expected, atol=1e-6, rtol=3e-4)
    # the scores fall with the key index: the first 4032 keys and the suffix are kept
    _, ref_keep = O.select_tokens(scores.cpu().numpy(), 4096, reserved_recent=64)
    np.testing.assert_array_equal((~mask).cpu().numpy(), ref_keep)
    assert idx[0, 0, :4032].eq(torch.arange(4032, device="cuda")).all()


@pytest.mark.parametrize("decay,window", [(.01, 0), (0., 128), (.1, 65)])
def test_long_weighted_analytic(decay, window):
    # reference tests/test_prefill.py:134-146
    n = 131072
    q = torch.zeros(1, 2, n, 16, device="cuda", dtype=torch.bfloat16)
    k = torch.zeros(1, 1, n, 16, device="cuda", dtype=q.dtype)
    v = torch.ones_like(k)
    _, scores = prefill(q, k, v, recency_decay=decay, observation_window=window)
    pos = torch.arange(n, device="cuda", dtype=torch.float64)
    weight = (decay * (pos - (n - 1))).exp()
    if window:
        weight *= pos >= n - window
    expected = (weight / (pos + 1)).flip(0).cumsum(0).flip(0) * 32
    torch.testing.assert_close(scores[0, 0], expected.float(), atol=1e-7, rtol=5e-4)


def test_reference_triton_kernel_outputs():
    """The reference's own Triton kernel (run by the interpreter when the
    fixture was made) on the same fp16 inputs."""
    import os
    from common import GOLDEN
    z = np.load(os.path.join(GOLDEN, "triton_interp.npz"))
    for j in range(int(z["ncases"])):
        n, h, hk, d, causal, weighted, decay, window = z[f"i{j}_args"]
        q, k, v = (torch.from_numpy(z[f"i{j}_{x}"].view(np.int16)).view(torch.float16).cuda() for x in "qkv")
        out, imp = prefill(q, k, v, causal=bool(causal), value_weighted=bool(weighted), recency_decay=float(decay),
                           observation_window=int(window))
        torch.testing.assert_close(out.float().cpu(), torch.from_numpy(z[f"i{j}_out"]), atol=2e-3, rtol=6e-3)
        torch.testing.assert_close(imp.cpu(), torch.from_numpy(z[f"i{j}_imp"]), atol=3e-3 if weighted else 3e-5,
                                   rtol=3e-4)
