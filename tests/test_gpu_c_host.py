"""The library driven from C, without Python or torch in the calling process.

tests/c_host/evict_host.c is built with gcc against include/flash_evict.h and
the in-tree libflash_evict_b200.so (plus the system CUDA runtime for its own
allocations and stream).  It runs fe_evict (caller workspace) and
fe_evict_noalloc on bf16 inputs it generates and writes inputs and outputs
to a file; both results must equal, bit for bit, what the Python evict()
returns for the same inputs.
"""
import os
import shutil
import subprocess

import numpy as np
import pytest
import torch

from flash_evict import _lib, evict

pytestmark = pytest.mark.gpu

HERE = os.path.dirname(os.path.abspath(__file__))
INCLUDE = os.path.join(HERE, "..", "include")
CUDA = "/usr/local/cuda"


def _read(f, dtype, count):
    a = np.fromfile(f, dtype=dtype, count=count)
    assert a.size == count
    return a


def test_c_host_matches_python(tmp_path):
    gcc = shutil.which("gcc")
    assert gcc is not None, "gcc is part of this image"
    libdir = os.path.dirname(_lib.LIB_PATH)
    _lib.load()  # the library must exist (built in tree)
    exe = str(tmp_path / "evict_host")
    subprocess.run([gcc, "-O2", "-std=c11", "-Wall", os.path.join(HERE, "c_host", "evict_host.c"), "-I", INCLUDE,
                    "-I", os.path.join(CUDA, "include"), "-L", libdir, "-lflash_evict_b200",
                    "-L", os.path.join(CUDA, "lib64"), "-lcudart", "-Wl,-rpath," + libdir,
                    "-Wl,-rpath," + os.path.join(CUDA, "lib64"), "-o", exe], check=True)
    r = subprocess.run([exe, str(tmp_path / "res")], capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stdout + r.stderr
    with open(tmp_path / "res.bin", "rb") as f:
        b, hq, hk, n, d, budget, recent, pool = (int(x) for x in _read(f, np.int64, 8))
        bits = lambda shape: torch.from_numpy(_read(f, np.uint16, int(np.prod(shape))).astype(np.int16)).view(
            torch.bfloat16).reshape(shape)
        q, k, v = bits((b, hq, n, d)), bits((b, hk, n, d)), bits((b, hk, n, d))
        calls = []
        for _ in range(2):
            out = bits((b, hq, n, d))
            imp = torch.from_numpy(_read(f, np.float32, b * hk * n)).reshape(b, hk, n)
            idx = torch.from_numpy(_read(f, np.int64, b * hk * budget)).reshape(b, hk, budget)
            mask = torch.from_numpy(_read(f, np.uint8, b * hk * n)).reshape(b, hk, n)
            calls.append((out, imp, idx, mask))
    ref = evict(q.cuda(), k.cuda(), v.cuda(), budget, recent=recent, pool_kernel=pool, recency_decay=0.02)
    ref = [t.cpu() for t in ref]
    for out, imp, idx, mask in calls:
        assert torch.equal(out.view(torch.int16), ref[0].view(torch.int16))
        assert torch.equal(imp.view(torch.int32), ref[1].view(torch.int32))
        assert torch.equal(idx, ref[2])
        assert torch.equal(mask.bool(), ref[3])
    assert int((~ref[3]).sum()) == b * hk * budget
