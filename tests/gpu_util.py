"""Helpers for the GPU tests: device buffers (torch, plumbing only) wrapped
as the C ABI's QuantizedTensor."""
from __future__ import annotations

import importlib

import numpy as np

lq = importlib.import_module("llama2-min-inference_b200")


def dev(torch, a: np.ndarray):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def weight_tensor(torch, q: np.ndarray, s: np.ndarray, cols: int, gs: int, kind: int):
    """Upload packed weights + scales; returns (QuantizedTensor, keepalive)."""
    tq, ts = dev(torch, q), dev(torch, s.astype(np.float32))
    qt = lq.QuantizedTensor(q=tq.data_ptr(), s=ts.data_ptr(), rows=q.shape[0], cols=cols, group_size=gs, kind=kind)
    return qt, (tq, ts)


def act_tensor(torch, xq: np.ndarray, xs: np.ndarray, gs: int):
    tq, ts = dev(torch, xq.astype(np.int8)), dev(torch, xs.astype(np.float32))
    rows = xq.shape[0] if xq.ndim == 2 else 1
    qt = lq.QuantizedTensor(q=tq.data_ptr(), s=ts.data_ptr(), rows=rows, cols=xq.shape[-1], group_size=gs,
                            kind=lq.KIND_ACT8)
    return qt, (tq, ts)


def gemv_tolerance(xq, xs, wq, ws, cols, gs, kind):
    """Rigorous fp32 bound for a different summation order of the same
    terms: |dy| <= 2 * ng * eps * sum_g |ws*xs*D|."""
    import oracle as O

    xq2 = np.atleast_2d(xq)
    xs2 = np.atleast_2d(xs)
    ng = cols // gs
    bounds = []
    for b in range(xq2.shape[0]):
        D = O.group_dots(wq, xq2[b], cols, gs, kind).astype(np.float64)
        terms = np.abs(ws.astype(np.float64) * xs2[b][None, :].astype(np.float64) * D)
        bounds.append(terms.sum(1))
    eps = np.finfo(np.float32).eps
    return 2 * ng * eps * np.stack(bounds) + 1e-30
