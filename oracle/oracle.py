"""ctypes bindings of the CPU oracle (liboracle.so) and of the reference's own
runq.c built into _ref/librunq.so.

TEST INFRASTRUCTURE ONLY: imported by tests/, __graft_entry__.smoke() and the
CPU-baseline leg of bench.py, never by the product.
"""
from __future__ import annotations

import ctypes as C
import os

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ORACLE_LIB = os.path.join(HERE, "liboracle.so")
REF_LIB = os.path.join(HERE, "_ref", "librunq.so")
REF_RUNQ = os.path.join(HERE, "_ref", "runq")

_P = C.c_void_p
_orc = None
_ref = None


def _ptr(a: np.ndarray) -> int:
    assert a.flags["C_CONTIGUOUS"]
    return a.ctypes.data


def orc() -> C.CDLL:
    global _orc
    if _orc is None:
        L = C.CDLL(ORACLE_LIB)
        I, I64 = C.c_int, C.c_int64
        L.orc_quantize_act.argtypes = [_P, I, I, _P, _P, _P]
        L.orc_quantize_w8.argtypes = [_P, I64, I64, I, _P, _P]
        L.orc_quantize_w4.argtypes = [_P, I64, I64, I, _P, _P]
        L.orc_group_dots.argtypes = [_P, _P, _P, I64, I64, I, I]
        L.orc_gemv.argtypes = [_P, _P, _P, _P, _P, I64, I64, I, I]
        L.orc_gemm.argtypes = [_P, _P, _P, _P, _P, I, I64, I64, I, I]
        L.orc_model_load.restype = _P
        L.orc_model_load.argtypes = [C.c_char_p, I]
        L.orc_model_free.argtypes = [_P]
        L.orc_model_info.argtypes = [_P, _P, C.POINTER(I), C.POINTER(I)]
        L.orc_forward.restype = C.POINTER(C.c_float)
        L.orc_forward.argtypes = [_P, I, I]
        L.orc_argmax.argtypes = [_P, I]
        L.orc_forward_kernel_order.restype = C.POINTER(C.c_float)
        L.orc_forward_kernel_order.argtypes = [_P, I, I]
        L.orc_gemm_mma.argtypes = [_P, _P, _P, _P, _P, I, I64, I64, I, I, I, I, I]
        L.orc_set_mma_grid.argtypes = [_P, I]
        L.orc_set_tp.argtypes = [_P, I]
        L.orc_expf.restype = C.c_float
        L.orc_expf.argtypes = [C.c_float]
        L.orc_act_trace.restype = C.c_long
        L.orc_act_trace.argtypes = [_P, _P, C.c_long]
        L.orc_act_override.restype = C.c_long
        L.orc_act_override.argtypes = [_P, _P, _P, C.c_long]
        _orc = L
    return _orc


def ref_available() -> bool:
    return os.path.exists(REF_LIB)


def ref() -> C.CDLL:
    global _ref
    if _ref is None:
        L = C.CDLL(REF_LIB)
        I = C.c_int
        L.ref_quantize_act.argtypes = [_P, I, _P, _P, _P]
        L.ref_matmul_q8.argtypes = [_P, _P, _P, _P, _P, _P, I, I]
        L.ref_build.restype = _P
        L.ref_build.argtypes = [C.c_char_p]
        L.ref_forward.restype = C.POINTER(C.c_float)
        L.ref_forward.argtypes = [_P, I, I]
        L.ref_vocab.argtypes = [_P]
        L.ref_free.argtypes = [_P]
        L.ref_set_threads.argtypes = [I]
        L.ref_tokenizer.restype = _P
        L.ref_tokenizer.argtypes = [C.c_char_p, I]
        L.ref_encode.restype = I
        L.ref_encode.argtypes = [_P, C.c_char_p, _P]
        L.ref_tokenizer_free.argtypes = [_P]
        L.ref_sample.restype = I
        L.ref_sample.argtypes = [_P, I, C.c_float, C.c_float, C.POINTER(C.c_ulonglong)]
        L.ref_act_trace.restype = C.c_long
        L.ref_act_trace.argtypes = [_P, _P, C.c_long]
        _ref = L
    return _ref


def _act_values(config) -> int:
    """int8 activation values one decode step quantizes (runq.c:345,394,400,412,418)."""
    dim, hidden, layers = config[0], config[1], config[2]
    return layers * (3 * dim + hidden) + dim


# ---- oracle wrappers -----------------------------------------------------------

def quantize_act(x: np.ndarray, gs: int):
    x = np.ascontiguousarray(x, dtype=np.float32)
    n = x.shape[-1]
    rows = x.size // n
    xq = np.empty(x.shape, np.int8)
    xs = np.empty(x.shape[:-1] + (n // gs,), np.float32)
    xt = np.empty_like(xs)
    for r in range(rows):
        orc().orc_quantize_act(_ptr(x) + r * n * 4, n, gs, _ptr(xq) + r * n, _ptr(xs) + r * (n // gs) * 4,
                               _ptr(xt) + r * (n // gs) * 4)
    return xq, xs, xt


def quantize_weight(w: np.ndarray, gs: int, kind: int):
    w = np.ascontiguousarray(w, dtype=np.float32)
    rows, cols = w.shape
    q = np.empty((rows, cols if kind == 8 else cols // 2), np.uint8)
    s = np.empty((rows, cols // gs), np.float32)
    fn = orc().orc_quantize_w8 if kind == 8 else orc().orc_quantize_w4
    fn(_ptr(w), rows, cols, gs, _ptr(q), _ptr(s))
    return q, s


def group_dots(wq: np.ndarray, xq: np.ndarray, cols: int, gs: int, kind: int) -> np.ndarray:
    rows = wq.shape[0]
    D = np.empty((rows, cols // gs), np.int32)
    orc().orc_group_dots(_ptr(D), _ptr(np.ascontiguousarray(wq)), _ptr(np.ascontiguousarray(xq)), rows, cols,
                         gs, kind)
    return D


def gemv(xq, xs, wq, ws, cols: int, gs: int, kind: int) -> np.ndarray:
    xq = np.ascontiguousarray(xq)
    xs = np.ascontiguousarray(xs, dtype=np.float32)
    rows = wq.shape[0]
    B = xq.size // cols
    out = np.empty((B, rows), np.float32)
    orc().orc_gemm(_ptr(out), _ptr(xq), _ptr(xs), _ptr(np.ascontiguousarray(wq)),
                   _ptr(np.ascontiguousarray(ws)), B, rows, cols, gs, kind)
    return out


def gemm_mma(xq, xs, wq, ws, cols: int, gs: int, kind: int, tile0: int = 0, tiles: int = 0,
             grid: int = 148) -> np.ndarray:
    """The tensor-core GEMM's fp32 order: out [B, rows] for rows of tiles
    tile0.. of a launch of `tiles` 128-row tiles on `grid` CTAs."""
    xq = np.ascontiguousarray(np.atleast_2d(xq))
    xs = np.ascontiguousarray(np.atleast_2d(xs), dtype=np.float32)
    rows = wq.shape[0]
    B = xq.shape[0]
    tiles = tiles or rows // 128
    out = np.empty((B, rows), np.float32)
    orc().orc_gemm_mma(_ptr(out), _ptr(xq), _ptr(xs), _ptr(np.ascontiguousarray(wq)),
                       _ptr(np.ascontiguousarray(ws, dtype=np.float32)), B, rows, cols, gs, kind, tile0, tiles, grid)
    return out


class OracleModel:
    """Scalar CPU forward (runq.c:320-421 with INT4 and GS as parameters)."""

    def __init__(self, path: str, max_seq: int = 0):
        self.h = orc().orc_model_load(path.encode(), max_seq)
        if not self.h:
            raise RuntimeError(f"oracle could not load {path}")
        cfg = (C.c_int * 7)()
        kind, gs = C.c_int(), C.c_int()
        orc().orc_model_info(self.h, cfg, C.byref(kind), C.byref(gs))
        self.config = tuple(cfg)
        self.vocab = cfg[5]
        self.kind, self.gs = kind.value, gs.value

    def forward(self, token: int, pos: int) -> np.ndarray:
        p = orc().orc_forward(self.h, token, pos)
        return np.ctypeslib.as_array(p, shape=(self.vocab,)).copy()

    def set_mma_grid(self, grid: int) -> None:
        """grid > 0: forward_kernel_order mirrors a batched step (products on
        the tensor-core GEMM with `grid` CTAs); 0: the batch-1 GEMV."""
        orc().orc_set_mma_grid(self.h, grid)

    def set_tp(self, tp: int) -> None:
        """tp > 1: forward_kernel_order mirrors the tensor-parallel batch-1
        step over tp processes (wo / w2 partials summed in process order)."""
        orc().orc_set_tp(self.h, tp)

    def forward_kernel_order(self, token: int, pos: int) -> np.ndarray:
        """The step in the product kernels' fp32 reduction order."""
        p = orc().orc_forward_kernel_order(self.h, token, pos)
        return np.ctypeslib.as_array(p, shape=(self.vocab,)).copy()

    def forward_kernel_order_traced(self, token: int, pos: int):
        """forward_kernel_order plus every int8 activation value of the step,
        in call order (attention input, attention output, ffn input, ffn
        hidden per layer, then the final norm)."""
        buf = np.empty(_act_values(self.config), np.int8)
        orc().orc_act_trace(self.h, _ptr(buf), buf.size)
        lg = self.forward_kernel_order(token, pos)
        n = orc().orc_act_trace(self.h, None, 0)
        assert n == buf.size, (n, buf.size)
        return lg, buf

    def forward_kernel_order_with(self, token: int, pos: int, xq: np.ndarray, xs: np.ndarray) -> np.ndarray:
        """forward_kernel_order with every int8 activation and group scale of
        the step replaced by the given ones (e.g. runq.c's, from
        RefRunq.forward_traced): isolates the fp32 summation order from int8
        rounding flips."""
        xq = np.ascontiguousarray(xq, np.int8)
        xs = np.ascontiguousarray(xs, np.float32)
        assert xq.size == _act_values(self.config) and xs.size == xq.size // self.gs
        orc().orc_act_override(self.h, _ptr(xq), _ptr(xs), xq.size)
        lg = self.forward_kernel_order(token, pos)
        n = orc().orc_act_override(self.h, None, None, 0)
        assert n == xq.size, (n, xq.size)
        return lg

    def close(self):
        if self.h:
            orc().orc_model_free(self.h)
            self.h = None

    def __del__(self):
        self.close()


class RefRunq:
    """The reference's own runq.c (build_transformer / forward)."""

    def __init__(self, path: str):
        self.h = ref().ref_build(path.encode())
        self.vocab = ref().ref_vocab(self.h)

    def forward(self, token: int, pos: int) -> np.ndarray:
        p = ref().ref_forward(self.h, token, pos)
        return np.ctypeslib.as_array(p, shape=(self.vocab,)).copy()

    def forward_traced(self, token: int, pos: int, config):
        """forward plus the int8 activations quantize_act produced in the step
        and their group scales (recorded through the shim's fabsf / lrintf
        wrappers), in call order: (logits, xq [values], xs [values / 32])."""
        nv = _act_values(config)
        q = np.empty(nv, np.int8)
        ax = np.empty(nv, np.float32)
        ref().ref_act_trace(_ptr(q), _ptr(ax), nv)
        lg = self.forward(token, pos)
        n = ref().ref_act_trace(None, None, 0)
        assert n == nv, (n, nv)
        # quantize_act's group scale (runq.c:126-127), float32 arithmetic
        amax = ax.reshape(-1, 32).max(axis=1)
        xs = (amax / np.float32(127.0)).astype(np.float32)
        xs[xs == 0] = np.float32(1e-8)
        return lg, q, xs

    def close(self):
        if self.h:
            ref().ref_free(self.h)
            self.h = None

    def __del__(self):
        self.close()


def ref_matmul_q8(xq, xs, xt, q_biased, s, rows: int, cols: int) -> np.ndarray:
    out = np.empty(rows, np.float32)
    ref().ref_matmul_q8(_ptr(out), _ptr(np.ascontiguousarray(xq)), _ptr(np.ascontiguousarray(xs)),
                        _ptr(np.ascontiguousarray(xt)), _ptr(np.ascontiguousarray(q_biased)),
                        _ptr(np.ascontiguousarray(s)), rows, cols)
    return out


def ref_sample(logits: np.ndarray, temperature: float, topp: float, state: int):
    """runq.c's sample() on a copy of the logits: (next token, new rng state)."""
    x = np.ascontiguousarray(logits, np.float32).copy()
    st = C.c_ulonglong(state)
    nxt = ref().ref_sample(_ptr(x), x.size, temperature, topp, C.byref(st))
    return nxt, st.value


def ref_encode(tokenizer_path: str, vocab: int, text: str) -> np.ndarray:
    """runq.c's encode of a prompt (BOS first, no EOS), as generate() calls it."""
    t = ref().ref_tokenizer(tokenizer_path.encode(), vocab)
    out = np.zeros(len(text.encode()) + 3, np.int32)
    n = ref().ref_encode(t, text.encode(), _ptr(out))
    ref().ref_tokenizer_free(t)
    return out[:n].copy()


def ref_quantize_act(x: np.ndarray):
    x = np.ascontiguousarray(x, dtype=np.float32)
    n = x.size
    xq = np.empty(n, np.int8)
    xs = np.empty(n // 32, np.float32)
    xt = np.empty(n // 32, np.float32)
    ref().ref_quantize_act(_ptr(x), n, _ptr(xq), _ptr(xs), _ptr(xt))
    return xq, xs, xt
