"""The C-ABI library loads and exports every function include/llama2q.h
declares; argument errors come back as status codes (CPU only, no compute)."""
import ctypes as C
import os
import re
import subprocess

import pytest

ROOT = os.path.abspath(os.path.join(os.path.dirname(__file__), ".."))
HEADER = os.path.join(ROOT, "include", "llama2q.h")


def declared_functions():
    src = open(HEADER).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    names = re.findall(r"^[A-Za-z_][\w\s\*]*?\b([A-Za-z_]\w*)\s*\(", src, flags=re.M)
    return sorted(set(n for n in names if n not in ("defined",)))


def test_header_declares_the_reference_names():
    names = declared_functions()
    for n in ("quantize", "matmul", "forward", "build_transformer", "free_transformer"):
        assert n in names


def test_library_exports_every_declared_symbol(lq):
    L = lq.lib()
    out = subprocess.run(["nm", "-D", "--defined-only", lq.LIB_PATH], capture_output=True, text=True).stdout
    exported = set(line.split()[-1] for line in out.splitlines() if " T " in line)
    missing = [n for n in declared_functions() if n not in exported]
    assert not missing, missing
    for n in declared_functions():
        assert getattr(L, n) is not None
    assert set(lq.EXPORTS) <= set(declared_functions())


def test_argument_errors_are_status_codes(lq):
    qt = lq.QuantizedTensor()
    with pytest.raises(lq.LlamaQError) as e:
        lq.quantize(qt, 0, 64)
    assert e.value.code == lq.EINVAL
    w = lq.QuantizedTensor(q=16, s=16, rows=4, cols=64, group_size=48, kind=lq.KIND_INT8)
    x = lq.QuantizedTensor(q=16, s=16, rows=1, cols=64, group_size=48, kind=lq.KIND_ACT8)
    with pytest.raises(lq.LlamaQError) as e:
        lq.matmul(16, x, w, 64, 4)
    assert e.value.code == lq.EUNSUPPORTED
    w.group_size = x.group_size = 32
    with pytest.raises(lq.LlamaQError) as e:
        lq.matmul(16, x, w, 64, 8)  # d does not match w.rows
    assert e.value.code == lq.EINVAL
    assert "shape" in lq.last_error()


def test_runner_binary_built(lq):
    assert os.access(lq.RUNNER_PATH, os.X_OK)
    r = subprocess.run([lq.RUNNER_PATH], capture_output=True, text=True)
    assert r.returncode != 0 and "Usage" in r.stderr
