"""matmul_f32_noalloc: the allocation-free form of matmul_f32, for callers
that cannot allocate device memory while they run.  Checked through the C
ABI against matmul_f32 (the existing entry point) on two calls in a row,
with the same reordering tolerance the other GEMV tests use.  This file is
collected last so that a run stopping at the first failure has already run
every other test; it also passes alone in a fresh process."""
import numpy as np
import pytest

import oracle as O
from gpu_util import dev, gemv_tolerance, lq, weight_tensor

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("kind,gs,n,d", [(8, 64, 4096, 1024), (4, 64, 11008, 512), (8, 32, 288, 96)])
def test_noalloc_matches_matmul_f32_twice(cuda, kind, gs, n, d):
    rng = np.random.default_rng(n + kind)
    w = (rng.standard_normal((d, n)) * 0.02).astype(np.float32)
    wq, ws = O.quantize_weight(w, gs, kind)
    wt, keep = weight_tensor(cuda, wq, ws, n, gs, kind)
    for call in range(2):
        x = (rng.standard_normal(n) * (1 + call)).astype(np.float32)
        xq, xs, _ = O.quantize_act(x, gs)
        tol = gemv_tolerance(xq, xs, wq, ws, n, gs, kind)[0]
        xd = dev(cuda, x)
        y_ref = cuda.full((d,), float("nan"), dtype=cuda.float32, device="cuda")
        y_new = cuda.full((d,), float("nan"), dtype=cuda.float32, device="cuda")
        lq.matmul_f32(y_ref.data_ptr(), xd.data_ptr(), wt, n, d)
        lq.matmul_f32_noalloc(y_new.data_ptr(), xd.data_ptr(), wt, n, d)
        lq.sync()
        a, b = y_ref.cpu().numpy(), y_new.cpu().numpy()
        assert np.all(np.isfinite(b))
        assert np.all(np.abs(a - b) <= tol), f"call {call}"


def test_noalloc_rejects_oversize_and_host_memory(cuda):
    n, d, gs = 65536, 4, 64
    wq = np.zeros((d, n), np.uint8)
    ws = np.ones((d, n // gs), np.float32)
    wt, keep = weight_tensor(cuda, wq, ws, n, gs, 8)
    x = cuda.zeros(n, device="cuda")
    y = cuda.zeros(d, device="cuda")
    with pytest.raises(lq.LlamaQError) as e:
        lq.matmul_f32_noalloc(y.data_ptr(), x.data_ptr(), wt, n, d)
    assert e.value.code == lq.EINVAL and "limit" in lq.last_error()
    xh = np.zeros(4096, np.float32)
    w2, keep2 = weight_tensor(cuda, np.zeros((d, 4096), np.uint8), np.ones((d, 64), np.float32), 4096, 64, 8)
    with pytest.raises(lq.LlamaQError) as e:
        lq.matmul_f32_noalloc(y.data_ptr(), xh.ctypes.data, w2, 4096, d)
    assert e.value.code == lq.EINVAL
