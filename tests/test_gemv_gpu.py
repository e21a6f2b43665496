"""GPU parity of the hot-path operators against the CPU oracle, through the
C ABI (quantize / matmul / matmul_f32).

Bar: bit-exact int8 activations and int32 group dots; fp32 outputs within a
rigorous reordering bound (2 * groups * eps * sum of |terms|)."""
import numpy as np
import pytest

import oracle as O
from gpu_util import act_tensor, dev, gemv_tolerance, lq, weight_tensor

pytestmark = pytest.mark.gpu


def _weights(rng, d, n, gs, kind, std=0.02):
    w = (rng.standard_normal((d, n)) * std).astype(np.float32)
    return O.quantize_weight(w, gs, kind)


def _acts(rng, B, n, gs, scale=1.0):
    x = (rng.standard_normal((B, n)) * scale).astype(np.float32)
    xq, xs, _ = O.quantize_act(x, gs)
    return x, xq, xs


@pytest.mark.parametrize("n,gs,rows", [(288, 32, 1), (768, 32, 3), (4096, 64, 1), (11008, 64, 2), (4096, 128, 1)])
def test_quantize_bit_exact(cuda, n, gs, rows):
    rng = np.random.default_rng(n + gs)
    x = (rng.standard_normal((rows, n)) * 2).astype(np.float32)
    x[0, :gs] = 0.0  # all-zero group -> scale 1e-8
    xq, xs, _ = O.quantize_act(x, gs)
    tq = cuda.empty((rows, n), dtype=cuda.int8, device="cuda")
    ts = cuda.empty((rows, n // gs), dtype=cuda.float32, device="cuda")
    out = lq.QuantizedTensor(q=tq.data_ptr(), s=ts.data_ptr(), rows=rows, cols=n, group_size=gs, kind=0)
    lq.quantize(out, dev(cuda, x).data_ptr(), n)       # device input
    lq.sync()
    assert np.array_equal(tq.cpu().numpy(), xq)
    assert np.array_equal(ts.cpu().numpy().view(np.uint32), xs.view(np.uint32))
    tq.zero_()
    lq.quantize(out, x.ctypes.data, n)                 # host input
    lq.sync()
    assert np.array_equal(tq.cpu().numpy(), xq)
    assert out.kind == lq.KIND_ACT8 and out.cols == n


SHAPES = [
    # (d, n, gs): tiny config, 7B layer shapes, and shapes that take the
    # plain-load path (d % 4 != 0) or the row-slice path (long rows)
    (288, 288, 32), (768, 288, 32), (288, 768, 32),
    (4096, 4096, 64), (11008, 4096, 64), (4096, 11008, 64),
    (262, 512, 64), (64, 28672, 64), (1024, 8192, 64), (512, 4096, 128),
]


@pytest.mark.parametrize("kind", [8, 4])
@pytest.mark.parametrize("d,n,gs", SHAPES)
def test_group_dots_bit_exact(cuda, kind, d, n, gs):
    """With one-hot group scales and unit activation scales the GEMV output
    is exactly one int32 group dot (|D| < 2^24 is exact in fp32)."""
    rng = np.random.default_rng(d * 7 + n + kind)
    wq, _ = _weights(rng, d, n, gs, kind)
    xq = rng.integers(-127, 128, size=n).astype(np.int8)
    ng = n // gs
    D = O.group_dots(wq, xq, n, gs, kind)
    x, keep_x = act_tensor(cuda, xq[None], np.ones((1, ng), np.float32), gs)
    y = cuda.empty(d, dtype=cuda.float32, device="cuda")
    for g0 in sorted({0, ng // 2, ng - 1}):
        ws = np.zeros((d, ng), np.float32)
        ws[:, g0] = 1.0
        w, keep_w = weight_tensor(cuda, wq, ws, n, gs, kind)
        lq.matmul(y.data_ptr(), x, w, n, d)
        lq.sync()
        got = y.cpu().numpy()
        assert np.array_equal(got.astype(np.int64), D[:, g0].astype(np.int64)), f"group {g0}"


@pytest.mark.parametrize("kind", [8, 4])
@pytest.mark.parametrize("d,n,gs", SHAPES)
def test_matmul_matches_oracle(cuda, kind, d, n, gs):
    rng = np.random.default_rng(d + n * 3 + kind)
    wq, ws = _weights(rng, d, n, gs, kind)
    _, xq, xs = _acts(rng, 1, n, gs)
    ref = O.gemv(xq, xs, wq, ws, n, gs, kind)[0]
    tol = gemv_tolerance(xq, xs, wq, ws, n, gs, kind)[0]
    w, keep_w = weight_tensor(cuda, wq, ws, n, gs, kind)
    x, keep_x = act_tensor(cuda, xq, xs, gs)
    y = cuda.full((d,), float("nan"), dtype=cuda.float32, device="cuda")
    lq.matmul(y.data_ptr(), x, w, n, d)
    lq.sync()
    got = y.cpu().numpy()
    assert np.all(np.abs(got - ref) <= tol)


@pytest.mark.parametrize("kind", [8, 4])
@pytest.mark.parametrize("B", [2, 3, 8, 13])
def test_batched_matmul_matches_oracle(cuda, kind, B):
    d, n, gs = 1024, 4096, 64
    rng = np.random.default_rng(B * 11 + kind)
    wq, ws = _weights(rng, d, n, gs, kind)
    _, xq, xs = _acts(rng, B, n, gs)
    ref = O.gemv(xq, xs, wq, ws, n, gs, kind)
    tol = gemv_tolerance(xq, xs, wq, ws, n, gs, kind)
    w, keep_w = weight_tensor(cuda, wq, ws, n, gs, kind)
    x, keep_x = act_tensor(cuda, xq, xs, gs)
    y = cuda.empty((B, d), dtype=cuda.float32, device="cuda")
    lq.matmul(y.data_ptr(), x, w, n, d)
    lq.sync()
    assert np.all(np.abs(y.cpu().numpy() - ref) <= tol)


@pytest.mark.parametrize("kind", [8, 4])
def test_matmul_f32_host_and_device(cuda, kind):
    """quantize_act + matmul_q8 in one call (runq.c:345-346), host buffers
    (copies inside the call) and device buffers."""
    d, n, gs = 768, 4096, 64
    rng = np.random.default_rng(5 + kind)
    wq, ws = _weights(rng, d, n, gs, kind)
    x = rng.standard_normal(n).astype(np.float32)
    xq, xs, _ = O.quantize_act(x, gs)
    ref = O.gemv(xq, xs, wq, ws, n, gs, kind)[0]
    tol = gemv_tolerance(xq, xs, wq, ws, n, gs, kind)[0]
    w, keep_w = weight_tensor(cuda, wq, ws, n, gs, kind)
    out = np.full(d, np.nan, np.float32)
    lq.matmul_f32(out.ctypes.data, x.ctypes.data, w, n, d)
    assert np.all(np.abs(out - ref) <= tol)
    xd, yd = dev(cuda, x), cuda.empty(d, dtype=cuda.float32, device="cuda")
    lq.matmul_f32(yd.data_ptr(), xd.data_ptr(), w, n, d)
    lq.sync()
    assert np.array_equal(yd.cpu().numpy(), out)


@pytest.mark.parametrize("kind", [8, 4])
def test_matmul_f32_repeated_pinned_calls(cuda, kind):
    """Page-locked host x and y passed again and again (the end-to-end
    pattern): the first call runs operation by operation, the second builds
    the call's graph, later calls replay it.  Every call reads the current x
    and equals the device-buffer call bit for bit; a second weight with the
    same buffers gets its own result."""
    d, n, gs = 1024, 4096, 64
    rng = np.random.default_rng(17 + kind)
    wq, ws = _weights(rng, d, n, gs, kind)
    wq2, ws2 = _weights(rng, d, n, gs, kind)
    w, keep_w = weight_tensor(cuda, wq, ws, n, gs, kind)
    w2, keep_w2 = weight_tensor(cuda, wq2, ws2, n, gs, kind)
    hx = cuda.empty(n, dtype=cuda.float32).pin_memory()
    hy = cuda.empty(d, dtype=cuda.float32).pin_memory()
    yd = cuda.empty(d, dtype=cuda.float32, device="cuda")
    for i in range(5):
        wi = w2 if i == 3 else w
        x = rng.standard_normal(n).astype(np.float32)
        hx.copy_(cuda.from_numpy(x))
        hy.fill_(float("nan"))
        lq.matmul_f32(hy.data_ptr(), hx.data_ptr(), wi, n, d)
        lq.matmul_f32(yd.data_ptr(), dev(cuda, x).data_ptr(), wi, n, d)
        lq.sync()
        assert np.array_equal(hy.numpy(), yd.cpu().numpy()), i


def test_matmul_is_deterministic(cuda):
    d, n, gs, kind = 11008, 4096, 64, 4
    rng = np.random.default_rng(1)
    wq, ws = _weights(rng, d, n, gs, kind)
    _, xq, xs = _acts(rng, 1, n, gs)
    w, keep_w = weight_tensor(cuda, wq, ws, n, gs, kind)
    x, keep_x = act_tensor(cuda, xq, xs, gs)
    outs = []
    for _ in range(3):
        y = cuda.empty(d, dtype=cuda.float32, device="cuda")
        lq.matmul(y.data_ptr(), x, w, n, d)
        lq.sync()
        outs.append(y.cpu().numpy())
    assert np.array_equal(outs[0], outs[1]) and np.array_equal(outs[0], outs[2])
