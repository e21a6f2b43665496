"""Tensor-core GEMM (tcgen05.mma kind::i8) through the C ABI's matmul with
16 or more activation rows, against the oracle's restatement of its order.

The int32 group dots are exact and the fp32 epilogue is a fixed order
(fmaf over the groups of each stream-K piece, pieces summed in K order), so
the results are bit-exact against the oracle for the same grid size."""
import numpy as np
import pytest

import oracle as O
from gpu_util import act_tensor, gemv_tolerance, lq, weight_tensor

pytestmark = pytest.mark.gpu


def _sms(cuda):
    return cuda.cuda.get_device_properties(0).multi_processor_count


def _case(rng, B, d, n, gs, kind):
    w = (rng.standard_normal((d, n)) * 0.02).astype(np.float32)
    wq, ws = O.quantize_weight(w, gs, kind)
    x = rng.standard_normal((B, n)).astype(np.float32)
    xq, xs, _ = O.quantize_act(x, gs)
    return wq, ws, xq, xs


CASES = [
    # (B, d, n, gs): 13B / 7B layer shapes, a tile owned by two CTAs (d = 128),
    # every group size, partial 64-row chunks
    (16, 128, 256, 64), (17, 256, 512, 32), (32, 512, 1024, 128), (48, 5120, 5120, 64),
    (64, 13824, 5120, 64), (20, 5120, 13824, 64), (64, 4096, 4096, 64), (100, 1024, 4096, 64),
    (16, 32000, 4096, 64),
]


@pytest.mark.parametrize("kind", [8, 4])
@pytest.mark.parametrize("B,d,n,gs", CASES)
def test_tensor_core_matmul_bit_exact(cuda, kind, B, d, n, gs):
    rng = np.random.default_rng(B * 1000 + d + n + gs + kind)
    wq, ws, xq, xs = _case(rng, B, d, n, gs, kind)
    w, kw = weight_tensor(cuda, wq, ws, n, gs, kind)
    x, kx = act_tensor(cuda, xq, xs, gs)
    y = cuda.empty((B, d), dtype=cuda.float32, device="cuda")
    lq.matmul(y.data_ptr(), x, w, n, d)
    lq.sync()
    got = y.cpu().numpy()
    grid = min((d // 128) * (n // 128), _sms(cuda))
    ref = O.gemm_mma(xq, xs, wq, ws, n, gs, kind, 0, d // 128, grid)
    bad = np.argwhere(got.view(np.uint32) != ref.view(np.uint32))
    assert bad.size == 0, (len(bad), bad[:5].tolist(), float(np.abs(got - ref).max()))
    # and the order-free bound against the plain oracle GEMM
    tol = gemv_tolerance(xq, xs, wq, ws, n, gs, kind)
    plain = O.gemv(xq, xs, wq, ws, n, gs, kind)
    assert np.all(np.abs(got - plain) <= tol)


@pytest.mark.parametrize("kind", [8, 4])
def test_group_dots_exact_on_tensor_cores(cuda, kind):
    """One-hot group scales and unit activation scales: each output is one
    int32 group dot from the tensor cores."""
    rng = np.random.default_rng(11 + kind)
    B, d, n, gs = 24, 256, 1024, 64
    wq, _, xq, _ = _case(rng, B, d, n, gs, kind)
    xq[3] = 127
    xq[4] = -127
    ng = n // gs
    x, kx = act_tensor(cuda, xq, np.ones((B, ng), np.float32), gs)
    y = cuda.empty((B, d), dtype=cuda.float32, device="cuda")
    for g0 in (0, 7, ng - 1):
        ws = np.zeros((d, ng), np.float32)
        ws[:, g0] = 1.0
        w, kw = weight_tensor(cuda, wq, ws, n, gs, kind)
        lq.matmul(y.data_ptr(), x, w, n, d)
        lq.sync()
        got = y.cpu().numpy()
        for b in range(B):
            D = O.group_dots(wq, xq[b], n, gs, kind)[:, g0]
            assert np.array_equal(got[b].astype(np.int64), D.astype(np.int64)), (b, g0)


def test_tensor_core_rows_independent_of_batch(cuda):
    """Row b of a 16-row and of a 64-row product are bitwise equal."""
    rng = np.random.default_rng(5)
    d, n, gs = 1024, 2048, 64
    wq, ws, xq, xs = _case(rng, 64, d, n, gs, 8)
    w, kw = weight_tensor(cuda, wq, ws, n, gs, 8)
    outs = []
    for B in (16, 64):
        x, kx = act_tensor(cuda, xq[:B], xs[:B], gs)
        y = cuda.empty((B, d), dtype=cuda.float32, device="cuda")
        lq.matmul(y.data_ptr(), x, w, n, d)
        lq.sync()
        outs.append(y.cpu().numpy())
    assert np.array_equal(outs[0].view(np.uint32), outs[1][:16].view(np.uint32))


def test_tensor_core_pdl_and_graph(cuda):
    """With programmatic dependent launch and inside a captured graph the
    product is unchanged."""
    rng = np.random.default_rng(9)
    d, n, gs, B = 2048, 4096, 64, 32
    wq, ws, xq, xs = _case(rng, B, d, n, gs, 4)
    w, kw = weight_tensor(cuda, wq, ws, n, gs, 4)
    x, kx = act_tensor(cuda, xq, xs, gs)
    st = cuda.cuda.Stream()
    lq.set_stream(st.cuda_stream)
    try:
        y = cuda.empty((B, d), dtype=cuda.float32, device="cuda")
        lq.matmul(y.data_ptr(), x, w, n, d)
        lq.sync()
        ref = y.cpu().numpy().copy()
        lq.set_launch_flags(lq.LAUNCH_PDL)
        for _ in range(3):
            lq.matmul(y.data_ptr(), x, w, n, d)
        lq.sync()
        assert np.array_equal(y.cpu().numpy().view(np.uint32), ref.view(np.uint32))
        y.zero_()
        lq.graph_begin()
        lq.matmul(y.data_ptr(), x, w, n, d)
        g = lq.graph_end()
        for _ in range(3):
            lq.graph_launch(g)
        lq.sync()
        lq.graph_destroy(g)
        assert np.array_equal(y.cpu().numpy().view(np.uint32), ref.view(np.uint32))
    finally:
        lq.set_launch_flags(0)
        lq.set_stream(None)
