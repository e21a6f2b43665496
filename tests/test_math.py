"""The project's exp (lq_expf, csrc/lq_math.h): Cody-Waite reduction plus a
degree-7 Taylor polynomial, written with IEEE +, *, fma and rint only so the
CPU and the GPU produce the same bits.  Checked here (CPU only) against the
correctly rounded float64 exp over its whole finite range: at most 2 ulp
from the true value; bit for bit equal to the oracle's restatement
(orc_expf), which the decode-step tests compare with the GPU's results."""
import ctypes as C
import os
import subprocess

import numpy as np
import pytest

import oracle as O

ROOT = os.path.abspath(os.path.join(os.path.dirname(__file__), ".."))
CSRC = os.path.join(ROOT, "llama2-min-inference_b200", "csrc")


@pytest.fixture(scope="module")
def host_expf(tmp_path_factory):
    """lq_math.h compiled for the host exactly as the library's host code is
    (-ffp-contract=off), exposing lq_expf over an array."""
    d = tmp_path_factory.mktemp("expf")
    src = d / "expf.c"
    src.write_text('#include "lq_math.h"\n'
                   "void expf_many(const float* x, float* y, long n) {\n"
                   "    for (long i = 0; i < n; i++) y[i] = lq_expf(x[i]);\n}\n")
    so = d / "libexpf.so"
    subprocess.run(["gcc", "-O2", "-ffp-contract=off", "-fPIC", "-shared", f"-I{CSRC}", "-o", str(so), str(src),
                    "-lm"], check=True)
    L = C.CDLL(str(so))
    L.expf_many.argtypes = [C.c_void_p, C.c_void_p, C.c_long]

    def f(x):
        x = np.ascontiguousarray(x, np.float32)
        y = np.empty_like(x)
        L.expf_many(x.ctypes.data, y.ctypes.data, x.size)
        return y
    return f


def _sweep():
    # every 97th float32 bit pattern of [-104, 88.7] (both signs), plus edges
    lo, hi = np.float32(-104.0), np.float32(88.7)
    pos = np.arange(0, np.float32(hi).view(np.int32), 97, dtype=np.int32).view(np.float32)
    neg = -np.arange(0, np.float32(-lo).view(np.int32), 97, dtype=np.int32).view(np.float32)
    edges = np.array([0.0, -0.0, 1e-30, -1e-30, 0.5, -0.5, 1.0, -1.0, 88.0, 88.7, -87.3, -103.9, -104.0],
                     np.float32)
    return np.concatenate([pos, neg, edges])


def _ulp_err(y, x):
    """|y - exp(x)| in units of the float32 spacing at exp(x) (float64 reference)."""
    ref = np.exp(x.astype(np.float64))
    spacing = np.spacing(ref.astype(np.float32)).astype(np.float64)
    return np.abs(y.astype(np.float64) - ref) / spacing


def test_lq_expf_within_two_ulp(host_expf):
    x = _sweep()
    y = host_expf(x)
    ok = np.exp(x.astype(np.float64)) >= np.finfo(np.float32).tiny  # normal results
    err = _ulp_err(y[ok], x[ok])
    print(f"lq_expf over {ok.sum()} arguments: max {err.max():.3f} ulp, mean {err.mean():.3f} ulp")
    assert err.max() <= 2.0


def test_lq_expf_special_values(host_expf):
    y = host_expf(np.array([-200.0, -104.5, 89.0, 200.0, np.inf, -np.inf, np.nan], np.float32))
    assert y[0] == 0.0 and y[1] == 0.0
    assert np.isinf(y[2]) and np.isinf(y[3]) and np.isinf(y[4]) and y[5] == 0.0
    assert np.isnan(y[6])


def test_lq_expf_equals_oracle_restatement(host_expf):
    x = _sweep()[::7]
    y = host_expf(x)
    z = np.array([O.orc().orc_expf(float(v)) for v in x], np.float32)
    assert np.array_equal(y.view(np.uint32), z.view(np.uint32))
