"""Shared helpers for the tests: fixture loading and selection comparison."""
import ast
import glob
import os

import numpy as np
import torch

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")

DTYPES = {"float16": torch.float16, "bfloat16": torch.bfloat16}


def from_bits(arr, dtype):
    """uint16 raw bits -> torch tensor of dtype (fp16/bf16)."""
    return torch.from_numpy(np.ascontiguousarray(arr).view(np.int16)).view(dtype)


def golden_cases():
    return sorted(os.path.basename(p)[len("materialized_"):-4]
                  for p in glob.glob(os.path.join(GOLDEN, "materialized_*.npz")))


def load_case(name):
    z = np.load(os.path.join(GOLDEN, f"materialized_{name}.npz"), allow_pickle=False)
    dtype = DTYPES[str(z["dtype"])]
    rec = {key: z[key] for key in z.files}
    rec["dtype"] = dtype
    rec["q_t"] = from_bits(z["q"], dtype)
    rec["k_t"] = from_bits(z["k"], dtype)
    rec["v_t"] = from_bits(z["v"], dtype)
    rec["causal"] = bool(z["causal"])
    rec["kwargs"] = ast.literal_eval(str(z["kwargs"]))
    return rec


def snap_cases():
    """The SnapKV fixtures (tests/golden/snap.npz, from the reference's
    baselines.snap_scores / snap_select): list of dicts with torch q/k (q
    zero outside the window rows, which do not enter the scores)."""
    z = np.load(os.path.join(GOLDEN, "snap.npz"), allow_pickle=False)
    cases = []
    for j in range(int(z["ncases"])):
        dtype = DTYPES[str(z[f"s{j}_dtype"])]
        b, h, hk, n, d = (int(x) for x in z[f"s{j}_shape"])
        window, budget = (int(x) for x in z[f"s{j}_args"])
        qwin = from_bits(z[f"s{j}_qwin"], dtype)
        q = torch.zeros((b, h, n, d), dtype=dtype)
        q[:, :, n - qwin.shape[2]:] = qwin
        cases.append(dict(name=str(z[f"s{j}_name"]), dtype=dtype, dtype_name=str(z[f"s{j}_dtype"]), q=q,
                          k=from_bits(z[f"s{j}_k"], dtype), window=window, budget=budget,
                          scores=z[f"s{j}_scores"], idx=z[f"s{j}_idx"], keep=z[f"s{j}_keep"]))
    return cases


def strided_like_model(t):
    """Same values in the adapters' layout: a [B,H,N,D] view of a [B,N,H,D]
    buffer (noncontiguous strides)."""
    return t.transpose(1, 2).contiguous().transpose(1, 2)


def selection_mismatch(keep, ref_keep, scores, ref_scores, tol_abs, tol_rel):
    """Count keep-mask differences and check each one is a near tie.

    A difference is acceptable only when the reference score of every token
    that changed side lies within tolerance of the reference's selection
    threshold (the smallest kept reference score of that row).
    Returns (mismatches, all_explained).
    """
    keep = np.asarray(keep).reshape(-1, np.asarray(keep).shape[-1])
    ref_keep = np.asarray(ref_keep).reshape(keep.shape)
    ref_scores = np.asarray(ref_scores, dtype=np.float64).reshape(keep.shape)
    diff = keep != ref_keep
    mism = int(diff.sum())
    ok = True
    for r in np.nonzero(diff.any(1))[0]:
        kept = ref_scores[r][ref_keep[r]]
        thr = kept.min() if kept.size else 0.0
        for c in np.nonzero(diff[r])[0]:
            if abs(ref_scores[r, c] - thr) > tol_abs + tol_rel * abs(thr):
                ok = False
    return mism, ok


# Parity figures recorded by the GPU tests (one line per configuration),
# printed in the terminal summary by conftest.py.
PARITY_FIGURES = []


def record_figures(name, figs):
    keys = ("out_max_abs", "out_max_rel", "importance_max_rel", "importance_keys_checked", "mask_mismatches",
            "mismatches_near_ties")
    PARITY_FIGURES.append(name + ": " + ", ".join(f"{k}={figs[k]:.3g}" if isinstance(figs[k], float)
                                                 else f"{k}={figs[k]}" for k in keys if k in figs))
