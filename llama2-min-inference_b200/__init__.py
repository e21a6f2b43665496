"""Python mirror of the llama2q C ABI (include/llama2q.h), over ctypes.

The product is the shared library lib/libllama2q.so (CUDA kernels for
sm_100a behind a plain C ABI).  This module only binds it, with the
reference's names and argument meaning:

    quantize(out, x, n)              quantize_act   v1-int8-vnni/runq.c:117
    matmul(xout, x, w, n, d)         matmul_q8      v1-int8-vnni/runq.c:142
    forward(t, token, pos)           forward        v1-int8-vnni/runq.c:320
    build_transformer / free_transformer           runq.c:280-289

Errors raise LlamaQError carrying the library's status code and message,
where the reference exits the process.  There is no CPU fallback: importing
this module fails loudly when the library has not been built.

The package directory name contains hyphens, so import it with
``importlib.import_module("llama2-min-inference_b200")``.
"""
from __future__ import annotations

import ctypes as C
import os

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "lib", "libllama2q.so")
RUNNER_PATH = os.path.join(_HERE, "bin", "run")

KIND_INT8 = 8
KIND_INT4 = 4
KIND_ACT8 = 1

OK, EINVAL, ECUDA, ENOMEM, EIO, EFORMAT, ETIMEOUT, EUNSUPPORTED = range(8)

# step-trace kernel kinds (transformer_trace_read)
TRACE_KINDS = {1: "quantize", 2: "gemv", 3: "qgemm", 4: "attention", 5: "allreduce", 6: "argmax", 7: "nccl"}

# tensor ids of the checkpoint (file order) = synthetic generator streams
T_EMB, T_RMS_ATT, T_WQ, T_WK, T_WV, T_WO, T_RMS_FFN, T_W1, T_W2, T_W3, T_RMS_FINAL, T_WCLS = range(12)


class LlamaQError(RuntimeError):
    def __init__(self, code: int, msg: str):
        super().__init__(f"llama2q error {code}: {msg}")
        self.code = code


class QuantizedTensor(C.Structure):
    """QuantizedTensor of include/llama2q.h (QWeight, runq.c:43-49)."""

    _fields_ = [
        ("q", C.c_void_p),
        ("s", C.c_void_p),
        ("rows", C.c_int64),
        ("cols", C.c_int64),
        ("group_size", C.c_int32),
        ("kind", C.c_int32),
    ]


class Config(C.Structure):
    """Config of include/llama2q.h (runq.c:33-41)."""

    _fields_ = [
        ("dim", C.c_int),
        ("hidden_dim", C.c_int),
        ("n_layers", C.c_int),
        ("n_heads", C.c_int),
        ("n_kv_heads", C.c_int),
        ("vocab_size", C.c_int),
        ("seq_len", C.c_int),
    ]

    @staticmethod
    def make(dim, hidden_dim, n_layers, n_heads, n_kv_heads, vocab_size, seq_len) -> "Config":
        return Config(dim, hidden_dim, n_layers, n_heads, n_kv_heads, vocab_size, seq_len)

    def as_tuple(self):
        return (self.dim, self.hidden_dim, self.n_layers, self.n_heads, self.n_kv_heads,
                self.vocab_size, self.seq_len)


# names the C ABI exports (checked by the CPU test suite against the header)
EXPORTS = (
    "lq_last_error", "lq_select_device", "lq_set_stream", "lq_get_stream", "lq_sync",
    "lq_set_launch_flags", "lq_set_trace", "lq_graph_begin", "lq_graph_end", "lq_graph_launch", "lq_graph_destroy",
    "lq_synth_tensor", "quantize", "matmul", "matmul_f32", "matmul_f32_noalloc",
    "build_transformer", "build_transformer_random", "forward", "forward_argmax", "forward_prompt",
    "transformer_reserve_batch", "forward_batch", "forward_batch_argmax",
    "lq_tp_unique_id", "build_transformer_tp", "build_transformer_random_tp", "lq_tp_wait_selftest",
    "free_transformer", "transformer_config", "transformer_trace", "transformer_trace_read",
    "lq_write_checkpoint_fp32", "lq_quantize_checkpoint", "lq_write_checkpoint_random", "lq_read_header",
    "lq_synth_value",
)

_lib = None


def lib() -> C.CDLL:
    """Load lib/libllama2q.so (raises if it has not been built)."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(LIB_PATH):
        raise ImportError(f"{LIB_PATH} is missing: run __graft_entry__.build() (make -C the package)")
    L = C.CDLL(LIB_PATH)
    P, I, I64, U64, F = C.c_void_p, C.c_int, C.c_int64, C.c_uint64, C.c_float
    QT = C.POINTER(QuantizedTensor)
    CFG = C.POINTER(Config)
    sig = {
        "lq_last_error": (C.c_char_p, []),
        "lq_select_device": (I, [I]),
        "lq_set_stream": (I, [P]),
        "lq_get_stream": (P, []),
        "lq_sync": (I, []),
        "lq_set_launch_flags": (I, [I]),
        "lq_set_trace": (I, [P]),
        "lq_graph_begin": (I, []),
        "lq_graph_end": (I, [C.POINTER(P)]),
        "lq_graph_launch": (I, [P]),
        "lq_graph_destroy": (None, [P]),
        "lq_synth_tensor": (I, [QT, U64, I, F]),
        "quantize": (I, [QT, P, I]),
        "matmul": (I, [P, QT, QT, I, I]),
        "matmul_f32": (I, [P, P, QT, I, I]),
        "matmul_f32_noalloc": (I, [P, P, QT, I, I]),
        "build_transformer": (I, [C.POINTER(P), C.c_char_p, I]),
        "build_transformer_random": (I, [C.POINTER(P), CFG, I, I, U64, I]),
        "forward": (C.POINTER(F), [P, I, I]),
        "forward_argmax": (I, [P, I, I, C.POINTER(I)]),
        "forward_prompt": (C.POINTER(F), [P, P, I, I]),
        "transformer_reserve_batch": (I, [P, I]),
        "lq_tp_unique_id": (I, [P]),
        "lq_tp_wait_selftest": (I, [I, I, C.POINTER(C.c_double), C.POINTER(C.c_double)]),
        "build_transformer_tp": (I, [C.POINTER(P), C.c_char_p, I, I, I, P]),
        "build_transformer_random_tp": (I, [C.POINTER(P), CFG, I, I, U64, I, I, I, P]),
        "forward_batch": (C.POINTER(F), [P, P, P, I]),
        "forward_batch_argmax": (I, [P, P, P, I, P]),
        "free_transformer": (None, [P]),
        "transformer_config": (I, [P, CFG, C.POINTER(I), C.POINTER(I)]),
        "transformer_trace": (I, [P, I]),
        "transformer_trace_read": (I, [P, I, P, P, C.POINTER(I)]),
        "lq_write_checkpoint_fp32": (I, [C.c_char_p, CFG, U64, F, I]),
        "lq_quantize_checkpoint": (I, [C.c_char_p, C.c_char_p, I, I]),
        "lq_write_checkpoint_random": (I, [C.c_char_p, CFG, I, I, U64, F]),
        "lq_read_header": (I, [C.c_char_p, CFG, C.POINTER(I), C.POINTER(I), C.POINTER(I)]),
        "lq_synth_value": (F, [U64, I, U64, F]),
    }
    for name, (res, args) in sig.items():
        fn = getattr(L, name)
        fn.restype = res
        fn.argtypes = args
    _lib = L
    return L


def last_error() -> str:
    return (lib().lq_last_error() or b"").decode(errors="replace")


def check(rc: int) -> None:
    if rc != OK:
        raise LlamaQError(rc, last_error())


# ---- operators -------------------------------------------------------------

def set_stream(stream_ptr: int | None) -> None:
    check(lib().lq_set_stream(stream_ptr))


def sync() -> None:
    check(lib().lq_sync())


LAUNCH_PDL = 1


def set_launch_flags(flags: int) -> None:
    check(lib().lq_set_launch_flags(flags))


def set_trace(device_ptr: int | None) -> None:
    check(lib().lq_set_trace(device_ptr))


def graph_begin() -> None:
    check(lib().lq_graph_begin())


def graph_end() -> int:
    h = C.c_void_p()
    check(lib().lq_graph_end(C.byref(h)))
    return h.value


def graph_launch(h: int) -> None:
    check(lib().lq_graph_launch(C.c_void_p(h)))


def graph_destroy(h: int) -> None:
    lib().lq_graph_destroy(C.c_void_p(h))


def synth_tensor(w: QuantizedTensor, seed: int, tensor_id: int, std: float = 0.02) -> None:
    check(lib().lq_synth_tensor(C.byref(w), seed, tensor_id, std))


def quantize(out: QuantizedTensor, x_ptr: int, n: int) -> None:
    """Activation quantize (quantize_act, runq.c:117-139) into device buffers."""
    check(lib().quantize(C.byref(out), C.c_void_p(x_ptr), n))


def matmul(xout_ptr: int, x: QuantizedTensor, w: QuantizedTensor, n: int, d: int) -> None:
    """xout[B, d] = W[d, n] . x[B, n] (matmul_q8, runq.c:142-159)."""
    check(lib().matmul(C.c_void_p(xout_ptr), C.byref(x), C.byref(w), n, d))


def matmul_f32(xout_ptr: int, x_ptr: int, w: QuantizedTensor, n: int, d: int) -> None:
    """quantize_act + matmul_q8 in one call; host or device pointers.  (The
    pointers go to the C function as plain integers and the weight by
    reference, through the argument types set when the library was loaded.)"""
    rc = lib().matmul_f32(xout_ptr, x_ptr, w, n, d)
    if rc != OK:
        raise LlamaQError(rc, last_error())


def matmul_f32_noalloc(xout_ptr: int, x_ptr: int, w: QuantizedTensor, n: int, d: int) -> None:
    """matmul_f32 without any device allocation (fixed library scratch, n <= 32768, device pointers)."""
    check(lib().matmul_f32_noalloc(C.c_void_p(xout_ptr), C.c_void_p(x_ptr), C.byref(w), n, d))


# ---- model -------------------------------------------------------------------

class Transformer:
    """Owns a Transformer* (build_transformer / free_transformer)."""

    def __init__(self, handle: int):
        self._h = C.c_void_p(handle)
        cfg, kind, gs = Config(), C.c_int(), C.c_int()
        check(lib().transformer_config(self._h, C.byref(cfg), C.byref(kind), C.byref(gs)))
        self.config, self.kind, self.group_size = cfg, kind.value, gs.value

    @classmethod
    def from_file(cls, path: str, max_seq_len: int = 0) -> "Transformer":
        h = C.c_void_p()
        check(lib().build_transformer(C.byref(h), path.encode(), max_seq_len))
        return cls(h.value)

    @classmethod
    def random(cls, cfg: Config, kind: int, group_size: int, seed: int, max_seq_len: int = 0) -> "Transformer":
        h = C.c_void_p()
        check(lib().build_transformer_random(C.byref(h), C.byref(cfg), kind, group_size, seed, max_seq_len))
        return cls(h.value)

    def forward(self, token: int, pos: int):
        """Returns a numpy view of the host logits (valid until the next call)."""
        import numpy as np

        p = lib().forward(self._h, token, pos)
        if not p:
            raise LlamaQError(-1, last_error())
        return np.ctypeslib.as_array(p, shape=(self.config.vocab_size,))

    def forward_prompt(self, tokens, start_pos: int = 0):
        """Prefill sequence 0 with the prompt tokens at start_pos..; returns a
        numpy view of the last token's logits (valid until the next call)."""
        import numpy as np

        t = np.ascontiguousarray(tokens, dtype=np.int32)
        p = lib().forward_prompt(self._h, t.ctypes.data, t.size, start_pos)
        if not p:
            raise LlamaQError(-1, last_error())
        return np.ctypeslib.as_array(p, shape=(self.config.vocab_size,))

    def forward_argmax(self, token: int, pos: int) -> int:
        nxt = C.c_int()
        check(lib().forward_argmax(self._h, token, pos, C.byref(nxt)))
        return nxt.value

    @classmethod
    def from_file_tp(cls, path: str, rank: int, size: int, group_id: bytes | None, max_seq_len: int = 0):
        """This process's tensor-parallel share (rank of size) of a checkpoint."""
        h = C.c_void_p()
        gid = C.create_string_buffer(group_id, 128) if group_id else None
        check(lib().build_transformer_tp(C.byref(h), path.encode(), max_seq_len, rank, size, gid))
        return cls(h.value)

    @classmethod
    def random_tp(cls, cfg: Config, kind: int, group_size: int, seed: int, rank: int, size: int,
                  group_id: bytes | None, max_seq_len: int = 0) -> "Transformer":
        h = C.c_void_p()
        gid = C.create_string_buffer(group_id, 128) if group_id else None
        check(lib().build_transformer_random_tp(C.byref(h), C.byref(cfg), kind, group_size, seed, max_seq_len,
                                                rank, size, gid))
        return cls(h.value)

    def reserve_batch(self, max_batch: int) -> None:
        """Size for up to max_batch sequences (restarts every sequence)."""
        check(lib().transformer_reserve_batch(self._h, max_batch))
        self.max_batch = max_batch

    @staticmethod
    def _rows(tokens, pos):
        import numpy as np

        t = np.ascontiguousarray(tokens, dtype=np.int32)
        p = np.ascontiguousarray(pos, dtype=np.int32)
        if t.shape != p.shape or t.ndim != 1:
            raise ValueError("tokens and pos must be 1-D and of equal length")
        return t, p

    def forward_batch(self, tokens, pos):
        """Logits [B, vocab] (a view of host memory valid until the next call)."""
        import numpy as np

        t, p = self._rows(tokens, pos)
        r = lib().forward_batch(self._h, t.ctypes.data, p.ctypes.data, t.size)
        if not r:
            raise LlamaQError(-1, last_error())
        return np.ctypeslib.as_array(r, shape=(t.size, self.config.vocab_size))

    def forward_batch_argmax(self, tokens, pos):
        import numpy as np

        t, p = self._rows(tokens, pos)
        out = np.empty(t.size, np.int32)
        check(lib().forward_batch_argmax(self._h, t.ctypes.data, p.ctypes.data, t.size, out.ctypes.data))
        return out

    def trace(self, enable: bool = True) -> None:
        """Turn the step trace on or off (the graph is captured again)."""
        check(lib().transformer_trace(self._h, 1 if enable else 0))

    def trace_read(self):
        """(kinds [K], stamps [K, 3] uint64 ns: start, past-wait, end) of the last step."""
        import numpy as np

        cnt = C.c_int()
        check(lib().transformer_trace_read(self._h, 0, None, None, C.byref(cnt)))
        k = np.zeros(cnt.value, np.int32)
        st = np.zeros((cnt.value, 3), np.uint64)
        check(lib().transformer_trace_read(self._h, cnt.value, k.ctypes.data, st.ctypes.data, C.byref(cnt)))
        return k, st

    def close(self) -> None:
        if self._h:
            lib().free_transformer(self._h)
            self._h = None

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def tp_wait_selftest(tp_size: int, wait_us: int):
    """Run the all-reduce wait's failure path on this device (see the header):
    returns (status code, first call ms, second call ms); LQ_ETIMEOUT expected."""
    a, b = C.c_double(), C.c_double()
    rc = lib().lq_tp_wait_selftest(tp_size, wait_us, C.byref(a), C.byref(b))
    return rc, a.value, b.value


def tp_unique_id() -> bytes:
    """A new tensor-parallel group id (128 bytes) to hand to every process."""
    buf = C.create_string_buffer(128)
    check(lib().lq_tp_unique_id(buf))
    return buf.raw


# ---- checkpoint files (host only) ----------------------------------------------

def write_checkpoint_fp32(path: str, cfg: Config, seed: int, std: float = 0.02, shared: bool = False) -> None:
    check(lib().lq_write_checkpoint_fp32(path.encode(), C.byref(cfg), seed, std, 1 if shared else 0))


def quantize_checkpoint(src: str, dst: str, kind: int, group_size: int) -> None:
    check(lib().lq_quantize_checkpoint(src.encode(), dst.encode(), kind, group_size))


def write_checkpoint_random(path: str, cfg: Config, kind: int, group_size: int, seed: int, std: float = 0.02) -> None:
    """Seeded quantized checkpoint written directly (same bytes as the fp32
    export + quantize_checkpoint, unshared classifier)."""
    check(lib().lq_write_checkpoint_random(path.encode(), C.byref(cfg), kind, group_size, seed, std))


def read_header(path: str):
    cfg, kind, gs, shared = Config(), C.c_int(), C.c_int(), C.c_int()
    check(lib().lq_read_header(path.encode(), C.byref(cfg), C.byref(kind), C.byref(gs), C.byref(shared)))
    return cfg, kind.value, gs.value, bool(shared.value)


def synth_value(seed: int, tensor_id: int, index: int, std: float = 0.02) -> float:
    return lib().lq_synth_value(seed, tensor_id, index, std)
