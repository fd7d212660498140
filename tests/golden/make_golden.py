"""Generate golden fixtures from the reference implementation.

Runs only where the reference package is importable (pass its checkout with
--reference); the GPU box and the tests never import the reference.  Writes
tests/golden/*.npz:

  materialized_<case>.npz  inputs (raw fp16/bf16 bits) and the outputs of the
                           reference's flash_evict/reference.py:materialized,
                           plus flash_evict/prefill.py:select_tokens (torch,
                           CPU) on those scores at several budgets
  selection.npz            select_tokens / baselines.snap_select on seeded
                           score tensors (pooling, reserved suffix, ties-free)
  triton_interp.npz        the reference's own Triton kernel `_prefill` run by
                           the Triton CPU interpreter (fp16 only; the
                           interpreter mishandles bf16), output and importance
  snap.npz                 the reference's flash_evict/baselines.py:snap_scores
                           and snap_select (torch, CPU) on seeded q/k, windows
                           inside one 256-row group, several groups, and a
                           window longer than 256 rows

Usage: python tests/golden/make_golden.py --reference /path/to/reference [--only NAME ...]
"""
import argparse
import math
import os
import subprocess
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))

# (name, B, n, h, hk, d, dtype, causal, kwargs, transposed, q_scale)
CASES = [
    ("n256_h4_hk4_d64_f16", 1, 256, 4, 4, 64, torch.float16, True, {}, True, 1.0),
    ("n256_h4_hk2_d64_bf16", 1, 256, 4, 2, 64, torch.bfloat16, True, {}, True, 1.0),
    ("n137_h6_hk2_d80_f16_noncausal", 1, 137, 6, 2, 80, torch.float16, False, {}, True, 1.0),
    ("n65_h4_hk1_d32_bf16", 1, 65, 4, 1, 32, torch.bfloat16, True, {}, True, 1.0),
    ("n1_h2_hk1_d16_f16", 1, 1, 2, 1, 16, torch.float16, True, {}, True, 1.0),
    ("b2_n97_h4_hk2_d64_f16_x15", 2, 97, 4, 2, 64, torch.float16, True, {}, False, 15.0),
    ("n137_d01_w65_bf16", 1, 137, 4, 2, 64, torch.bfloat16, True,
     {"recency_decay": 0.1, "observation_window": 65}, True, 1.0),
    ("n300_d001_bf16_h2o", 1, 300, 4, 2, 64, torch.bfloat16, True,
     {"recency_decay": 0.01, "value_weighted": False}, True, 1.0),
    ("n200_w32_f16", 1, 200, 4, 2, 64, torch.float16, True, {"observation_window": 32}, True, 1.0),
]


def bits(t):
    return t.contiguous().view(torch.int16).numpy().view(np.uint16)


def make_inputs(seed, b, n, h, hk, d, dtype, transposed, q_scale):
    g = torch.Generator().manual_seed(seed)
    if transposed:
        q = torch.randn((b, n, h, d), generator=g).to(dtype).transpose(1, 2)
        k = torch.randn((b, n, hk, d), generator=g).to(dtype).transpose(1, 2)
        v = torch.randn((b, n, hk, d), generator=g).to(dtype).transpose(1, 2)
    else:
        q = torch.randn((b, h, n, d), generator=g).to(dtype)
        k = torch.randn((b, hk, n, d), generator=g).to(dtype)
        v = torch.randn((b, hk, n, d), generator=g).to(dtype)
    if q_scale != 1.0:
        q = (q.float() * q_scale).to(dtype)
        k = (k.float() * q_scale).to(dtype)
    return q, k, v


def materialized_fixtures(ref):
    from flash_evict.prefill import select_tokens
    from flash_evict.reference import materialized
    for i, (name, b, n, h, hk, d, dtype, causal, kw, tr, qs) in enumerate(CASES):
        q, k, v = make_inputs(1000 + i, b, n, h, hk, d, dtype, tr, qs)
        out, mass = materialized(q, k, v, causal=causal, **kw)
        budgets = sorted({max(1, math.ceil(n * r)) for r in (.05, .1, .2)})
        sel = {}
        for bud in budgets:
            idx, keep = select_tokens(mass, bud)
            sel[f"idx_{bud}"] = idx.numpy()
            sel[f"keep_{bud}"] = keep.numpy()
        np.savez_compressed(
            os.path.join(HERE, f"materialized_{name}.npz"),
            q=bits(q), k=bits(k), v=bits(v), dtype=np.array(str(dtype).split(".")[-1]),
            causal=np.array(causal), kwargs=np.array(repr(kw)), out=out.numpy().astype(np.float32),
            mass=mass.numpy().astype(np.float32), budgets=np.array(budgets), **sel)
        print("wrote", name)


def selection_fixtures():
    from flash_evict.baselines import snap_select
    from flash_evict.prefill import select_tokens
    rec = {}
    torch.manual_seed(1)
    scores = torch.randn(1, 3, 137)                  # tests/test_prefill.py:151-155
    idx, keep = select_tokens(scores, 48, reserved_recent=32, pool_kernel=5)
    sidx, skeep = snap_select(scores, 48, 32, 5)
    assert torch.equal(idx, sidx) and torch.equal(keep, skeep)
    rec["pin_scores"], rec["pin_idx"], rec["pin_keep"] = scores.numpy(), idx.numpy(), keep.numpy()
    g = torch.Generator().manual_seed(7)
    cases = [(2, 4, 1000, 100, 0, 1), (2, 4, 1000, 100, 16, 5), (1, 2, 4096, 410, 0, 1), (1, 2, 4096, 512, 64, 7),
             (1, 1, 50, 50, 10, 3), (1, 1, 50, 5, 5, 5), (3, 1, 333, 1, 0, 1)]
    for j, (b, hk, n, bud, rec_, pk) in enumerate(cases):
        s = torch.rand((b, hk, n), generator=g) * 10
        idx, keep = select_tokens(s, bud, reserved_recent=rec_, pool_kernel=pk)
        rec[f"c{j}_scores"] = s.numpy()
        rec[f"c{j}_args"] = np.array([bud, rec_, pk])
        rec[f"c{j}_idx"] = idx.numpy()
        rec[f"c{j}_keep"] = keep.numpy()
    rec["ncases"] = np.array(len(cases))
    # the reference's own contract example (tests/test_prefill.py:77-81)
    idx, keep = select_tokens(torch.arange(20.).reshape(1, 1, 20), 4, recent=2)
    rec["contract_idx"], rec["contract_keep"] = idx.numpy(), keep.numpy()
    np.savez_compressed(os.path.join(HERE, "selection.npz"), **rec)
    print("wrote selection")


# (name, B, Hq, Hkv, N, D, dtype, window, q_scale, budget)
SNAP_CASES = [
    ("ref_test_w32", 1, 6, 2, 137, 32, torch.bfloat16, 32, 1.0, 48),     # tests/test_baselines.py:11-14 shape
    ("ref_test_full", 1, 6, 2, 137, 32, torch.bfloat16, 137, 1.0, 48),  # tests/test_baselines.py:21
    ("f16_g2_w32", 1, 4, 2, 300, 64, torch.float16, 32, 1.0, 30),
    ("bf16_g4_w48_b2", 2, 8, 2, 200, 64, torch.bfloat16, 48, 1.0, 20),
    ("bf16_g7_w32_d128", 1, 28, 4, 400, 128, torch.bfloat16, 32, 1.0, 40),
    ("bf16_w300_pieces", 1, 2, 1, 600, 64, torch.bfloat16, 300, 1.0, 60),
    ("f16_window_gt_n", 1, 4, 1, 100, 64, torch.float16, 500, 1.0, 10),
    ("bf16_x8_logits", 1, 4, 2, 260, 64, torch.bfloat16, 40, 8.0, 26),
    ("f16_n1", 1, 2, 1, 1, 16, torch.float16, 32, 1.0, 1),
]


def snap_fixtures():
    from flash_evict.baselines import snap_scores, snap_select
    rec = {}
    for j, (name, b, h, hk, n, d, dtype, window, qs, budget) in enumerate(SNAP_CASES):
        g = torch.Generator().manual_seed(3000 + j)
        q = (torch.randn((b, h, n, d), generator=g) * qs).to(dtype)
        k = torch.randn((b, hk, n, d), generator=g).to(dtype)
        scores = snap_scores(q, k, window)
        idx, keep = snap_select(scores, budget, window)
        rec[f"s{j}_name"] = np.array(name)
        # only the window rows of q enter the scores; the rest are not stored
        w = min(window, n)
        rec[f"s{j}_qwin"], rec[f"s{j}_k"] = bits(q[:, :, n - w:]), bits(k)
        rec[f"s{j}_shape"] = np.array([b, h, hk, n, d])
        rec[f"s{j}_dtype"] = np.array(str(dtype).split(".")[-1])
        rec[f"s{j}_args"] = np.array([window, budget])
        rec[f"s{j}_scores"] = scores.numpy()
        rec[f"s{j}_idx"] = idx.numpy()
        rec[f"s{j}_keep"] = keep.numpy()
    rec["ncases"] = np.array(len(SNAP_CASES))
    np.savez_compressed(os.path.join(HERE, "snap.npz"), **rec)
    print("wrote snap")


INTERP_SNIPPET = r"""
import sys, math, numpy as np, torch
sys.path.insert(0, sys.argv[1])
import triton
from flash_evict.prefill import _prefill
res = {}
for j, (n, h, hk, d, causal, weighted, decay, window) in enumerate(
        [(200, 4, 2, 64, True, True, 0.0, 0), (130, 2, 1, 32, False, True, 0.0, 0),
         (160, 4, 2, 64, True, False, 0.05, 48)]):
    g = torch.Generator().manual_seed(500 + j)
    q = torch.randn((1, h, n, d), generator=g).half()
    k = torch.randn((1, hk, n, d), generator=g).half()
    v = torch.randn((1, hk, n, d), generator=g).half()
    out = torch.empty_like(q)
    imp = torch.zeros((1, hk, n), dtype=torch.float32)
    bq, bk = 32, 64
    _prefill[(triton.cdiv(n, bq), h)](q, k, v, out, imp, *q.stride(), *k.stride(), *v.stride(), h, hk, n, d,
        d ** -0.5 * math.log2(math.e), causal, weighted, True, decay, min(n, window or n), bq, bk,
        max(16, triton.next_power_of_2(d)))
    res[f"i{j}_q"] = q.view(torch.int16).numpy().view(np.uint16)
    res[f"i{j}_k"] = k.view(torch.int16).numpy().view(np.uint16)
    res[f"i{j}_v"] = v.view(torch.int16).numpy().view(np.uint16)
    res[f"i{j}_out"] = out.float().numpy()
    res[f"i{j}_imp"] = imp.numpy()
    res[f"i{j}_args"] = np.array([n, h, hk, d, int(causal), int(weighted), decay, window])
res["ncases"] = np.array(3)
np.savez_compressed(sys.argv[2], **res)
print("wrote triton_interp")
"""


def triton_fixture(reference):
    env = dict(os.environ, TRITON_INTERPRET="1")
    subprocess.run([sys.executable, "-c", INTERP_SNIPPET, reference, os.path.join(HERE, "triton_interp.npz")],
                   check=True, env=env)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True, help="checkout of anishesg/flash-evict-prefill")
    ap.add_argument("--only", nargs="*", choices=["materialized", "selection", "triton", "snap"],
                    help="regenerate only these fixture files")
    args = ap.parse_args()
    sys.path.insert(0, args.reference)
    torch.set_num_threads(8)
    only = set(args.only or ["materialized", "selection", "triton", "snap"])
    if "materialized" in only:
        materialized_fixtures(args.reference)
    if "selection" in only:
        selection_fixtures()
    if "triton" in only:
        triton_fixture(args.reference)
    if "snap" in only:
        snap_fixtures()


if __name__ == "__main__":
    main()
