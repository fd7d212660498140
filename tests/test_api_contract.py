"""Host-side contract of the drop-in API and the C ABI (CPU only).

Mirrors the ValueError contract of the reference (prefill.py:86-99,
117-126, 149-159, 175-176 and tests/test_prefill.py:77-84, 149-159), checks
that the native library loads and exports every entry point declared in
include/flash_evict.h, and that a missing library fails loudly.
"""
import ctypes
import os
import re

import pytest
import torch

import flash_evict
from flash_evict import _lib, evict, prefill, select_tokens
import importlib

prefill_mod = importlib.import_module("flash_evict.prefill")

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "flash_evict.h")


def header_functions():
    text = open(HEADER).read()
    return re.findall(r"FE_API\s+[\w\s\*]+?\b(fe_\w+)\s*\(", text)


def test_library_exports_every_header_symbol():
    names = header_functions()
    assert len(names) >= 8
    lib = ctypes.CDLL(_lib.LIB_PATH)
    for name in names:
        assert hasattr(lib, name), name
        assert name in _lib.SIGNATURES, name
    assert set(_lib.SIGNATURES) == set(names)


def test_header_constants_match_binding():
    text = open(HEADER).read()
    defs = dict(re.findall(r"#define (FE_\w+) (\d+)", text))
    assert int(defs["FE_STATUS_OK"]) == _lib.STATUS_OK
    assert int(defs["FE_STATUS_INVALID"]) == _lib.STATUS_INVALID
    assert int(defs["FE_STATUS_UNSUPPORTED"]) == _lib.STATUS_UNSUPPORTED
    assert int(defs["FE_STATUS_CUDA"]) == _lib.STATUS_CUDA
    assert int(defs["FE_STATUS_TIMEOUT"]) == _lib.STATUS_TIMEOUT
    assert int(defs["FE_STATUS_BAD_INDEX"]) == _lib.STATUS_BAD_INDEX
    assert int(defs["FE_DTYPE_F16"]) == _lib.DTYPE_F16
    assert int(defs["FE_DTYPE_BF16"]) == _lib.DTYPE_BF16
    assert int(defs["FE_QUERY_BLOCK"]) == _lib.QUERY_BLOCK


def test_library_host_calls_without_gpu():
    lib = _lib.load()
    assert lib.fe_abi_version() == 3
    # argument checks run on the host before any device work
    rc = lib.fe_select_tokens(None, 1, 10, 0, 0, 1, None, None, 1, None)
    assert rc == _lib.STATUS_INVALID
    assert b"budget" in lib.fe_last_error()
    rc = lib.fe_select_tokens(None, 1, 10, 4, 0, 2, None, None, 1, None)
    assert rc == _lib.STATUS_INVALID and b"pool_kernel" in lib.fe_last_error()
    st = (ctypes.c_int64 * 4)(8, 8, 8, 2)
    fake = 256  # never dereferenced: the argument checks fail first
    rc = lib.fe_gather_tokens(fake, st, None, None, fake, fake, None, 1, 1, 8, 4, 8, 3, None)
    assert rc == _lib.STATUS_INVALID and b"elem_bytes" in lib.fe_last_error()
    rc = lib.fe_gather_tokens(fake, st, fake, st, fake, fake, None, 1, 1, 8, 4, 8, 2, None)
    assert rc == _lib.STATUS_INVALID and b"both" in lib.fe_last_error()
    rc = lib.fe_gather_tokens(fake, st, None, None, fake, fake, None, 1, 1, 8, 4, 8, 2, None)
    assert rc == _lib.STATUS_UNSUPPORTED and b"channel stride" in lib.fe_last_error()
    rc = lib.fe_gather_tokens(None, st, None, None, None, None, None, 1, 1, 8, 0, 8, 2, None)
    assert rc == _lib.STATUS_OK  # nothing to gather
    rc = lib.fe_select_gather(None, 1, 1, 10, 11, 0, 1, None, None, 1, None, st, None, st, None, None, 8, 2, None)
    assert rc == _lib.STATUS_INVALID and b"budget" in lib.fe_last_error()
    # key-tile range of the replay: 300 tokens = 3 tiles of 128 keys
    for lo, hi in ((-1, 2), (0, 4), (2, 1)):
        rc = lib.fe_replay_scores_range(fake, st, fake, st, fake, st, fake, fake, 1, 2, 1, 300, 64, _lib.DTYPE_BF16,
                                        1, 0.125, 0.0, 0, 1, None, 0, lo, hi, None)
        assert rc == _lib.STATUS_INVALID and b"key tile range" in lib.fe_last_error(), (lo, hi)
    # an empty range is a no-op that touches nothing
    rc = lib.fe_replay_scores_range(fake, st, fake, st, fake, st, fake, fake, 1, 2, 1, 300, 64, _lib.DTYPE_BF16,
                                    1, 0.125, 0.0, 0, 1, None, 0, 2, 2, None)
    assert rc == _lib.STATUS_OK


def test_public_api_surface():
    assert flash_evict.__all__[:3] == ["prefill", "evict", "select_tokens"]
    assert set(flash_evict.__all__[3:]) == {"gather_tokens", "select_and_gather", "evict_compact", "check_status"}
    import inspect
    sig = inspect.signature(prefill)
    assert list(sig.parameters) == ["q", "k", "v", "causal", "value_weighted", "score", "scale", "block_q",
                                    "block_k", "recency_decay", "observation_window"]
    assert sig.parameters["block_q"].default == 32 and sig.parameters["block_k"].default == 64
    assert list(inspect.signature(select_tokens).parameters) == ["importance", "budget", "recent",
                                                                 "reserved_recent", "pool_kernel"]
    assert list(inspect.signature(evict).parameters) == ["q", "k", "v", "budget", "recent", "reserved_recent",
                                                         "pool_kernel", "kwargs"]


def test_validate_errors():
    q = torch.zeros(1, 4, 8, 16, dtype=torch.float16)
    k = torch.zeros(1, 2, 8, 16, dtype=torch.float16)
    with pytest.raises(ValueError, match="shape"):
        prefill(q[0], k, k)
    with pytest.raises(ValueError, match="nonempty"):
        prefill(q, k, k[:, :, :4])
    with pytest.raises(ValueError, match="divisible"):
        prefill(q, torch.zeros(1, 3, 8, 16, dtype=torch.float16), torch.zeros(1, 3, 8, 16, dtype=torch.float16))
    with pytest.raises(ValueError, match="<= 256"):
        big = torch.zeros(1, 1, 8, 272, dtype=torch.float16)
        prefill(big, big, big)
    with pytest.raises(ValueError, match="same device and dtype"):
        prefill(q, k, k.float())
    with pytest.raises(ValueError, match="CUDA fp16 or bf16"):
        prefill(q, k, k)
    with pytest.raises(ValueError, match="CUDA fp16 or bf16"):
        prefill(q.float(), k.float(), k.float())
    with pytest.raises(ValueError, match="nonempty"):
        prefill(q[:, :, :0], k[:, :, :0], k[:, :, :0])


def test_prefill_argument_errors():
    check = prefill_mod._check_prefill_args
    assert check(0.1, 0, 32, 64, None, 64) == (0.1, 0.125)
    for bad in (-1.0, float("inf"), float("nan")):
        with pytest.raises(ValueError, match="recency_decay"):
            check(bad, 0, 32, 64, None, 64)
    for bad in (True, -1, 2.0):
        with pytest.raises(ValueError, match="observation_window"):
            check(0., bad, 32, 64, None, 64)
    with pytest.raises(ValueError, match="tile"):
        check(0., 0, 128, 64, None, 64)
    with pytest.raises(ValueError, match="tile"):
        check(0., 0, 32, 16, None, 64)
    with pytest.raises(ValueError, match="scale"):
        check(0., 0, 32, 64, float("inf"), 64)


def test_selection_contract_errors():
    # tests/test_prefill.py:77-84 and 149-159 of the reference
    scores = torch.arange(20.).reshape(1, 1, 20)
    for budget in (0, 21, True, 2.5):
        with pytest.raises(ValueError):
            select_tokens(scores, budget)
    with pytest.raises(ValueError):
        select_tokens(scores, 2, recent=3)
    s = torch.randn(1, 3, 137)
    for kwargs in ({'recent': True}, {'pool_kernel': 2}, {'recent': 1, 'reserved_recent': 2}):
        with pytest.raises(ValueError):
            select_tokens(s, 64, **kwargs)
    # valid arguments on a CPU tensor: no CPU path, fail loudly
    with pytest.raises(ValueError, match="CUDA"):
        select_tokens(scores, 4, recent=2)


def test_evict_rejects_score_false():
    q = torch.zeros(1, 1, 4, 16, dtype=torch.float16)
    with pytest.raises(ValueError, match="scoring"):
        evict(q, q, q, 2, score=False)


def test_missing_library_fails_loudly(monkeypatch):
    monkeypatch.setattr(_lib, "_lib", None)
    monkeypatch.setattr(_lib, "LIB_PATH", "/nonexistent/libflash_evict_b200.so")
    with pytest.raises(RuntimeError, match="not found"):
        _lib.load()


def test_no_oracle_on_product_path():
    pkg = os.path.join(ROOT, "flash-evict-prefill_b200")
    for dirpath, _, files in os.walk(pkg):
        for f in files:
            if f.endswith((".py", ".cu", ".cuh")):
                text = open(os.path.join(dirpath, f)).read()
                assert "oracle" not in text.replace("oracle/", ""), f


def _snap_workspace_model(b, hq, hk, n, window):
    """Restates the SnapKV row-group and key-chunk geometry of the C ABI
    (packed window rows in groups of <= 256, about one statistics CTA per SM,
    at most 32 key chunks) to check fe_snap_workspace_floats on the host."""
    g = hq // hk
    w = min(window, n)
    w8 = (w + 7) // 8 * 8
    groups = -(-g // (256 // w8)) if w8 <= 256 else g * (-(-w // 256))
    units = b * hk * groups
    ntiles = -(-n // 128)
    nchunk = max(1, min(-(-148 // units), 32, ntiles))
    tiles = -(-ntiles // nchunk)
    nchunk = -(-ntiles // tiles)
    return units * nchunk * 256 * 2


@pytest.mark.parametrize("shape", [(1, 28, 4, 32768, 32), (1, 6, 2, 137, 137), (2, 8, 2, 200, 48),
                                   (1, 2, 1, 600, 300), (8, 32, 32, 4096, 32), (1, 4, 1, 1, 32)])
def test_snap_workspace_size_on_host(shape):
    lib = _lib.load()
    assert lib.fe_snap_workspace_floats(*shape) == _snap_workspace_model(*shape)
    assert lib.fe_snap_workspace_floats(1, 28, 4, 32768, 0) < 0
    assert lib.fe_snap_workspace_floats(1, 27, 4, 32768, 32) < 0  # q_heads not a multiple of kv_heads
