"""runq.c parity helpers shared by the tests and the fixture generator.

The reference's CPU runner (v1-int8-vnni/runq.c, built from its sources into
oracle/_ref/librunq.so) and this library compute the same arithmetic with
the fp32 sums associated differently.  The two agree to a few ulp until an
fp32 value lands within an ulp of an int8 rounding boundary in one of the
step's quantize_act calls (runq.c:117-139); from then on the two runs see
one different int8 activation and the logits drift apart.  These helpers
locate that position (the first int8 "flip") and measure the agreement
before it, and over every position with the flip removed (the kernel-order
oracle fed runq.c's own int8 activations and scales).
"""
from __future__ import annotations

import os

import numpy as np

import oracle as O
import synth


def runq_usable() -> str | None:
    """None when the reference runner can run on this host, else why not."""
    if not O.ref_available():
        return "oracle/_ref/librunq.so is not built (the reference sources were absent at build time)"
    try:
        flags = open("/proc/cpuinfo").read()
    except OSError:
        return "cannot read /proc/cpuinfo"
    if "avx512_vnni" not in flags:
        return "the host CPU lacks AVX-512 VNNI, which runq.c needs"
    return None


def rel(a: np.ndarray, b: np.ndarray) -> float:
    return float(np.abs(a - b).max() / np.abs(b).max())


def runq_greedy_stream(path: str, steps: int) -> np.ndarray:
    """runq.c's free-running greedy stream from BOS (generate with -t 0)."""
    R = O.RefRunq(path)
    stream, token = [], 1
    for pos in range(steps):
        token = int(np.argmax(R.forward(token, pos)))
        stream.append(token)
    R.close()
    return np.array(stream, np.int32)


def flip_survey(path: str, steps: int, config=synth.TINY_CONFIG, device=None):
    """Teacher-force runq.c's greedy stream through runq.c, the kernel-order
    oracle and (optionally) a device model side by side.  Returns a dict:
      stream          runq.c's greedy stream
      first_flip      first position whose int8 activations differ between
                      runq.c and the kernel-order oracle (steps if none)
      rel_before      largest relative logits difference, oracle vs runq.c,
                      before first_flip
      rel_corrected   largest relative logits difference over every position
                      when the oracle uses runq.c's int8 activations
      device_bitwise  the device logits equal the oracle's bit for bit at
                      every position (None without a device model)
      device_rel_before  largest relative difference, device vs runq.c,
                      before first_flip (None without a device model)"""
    stream = runq_greedy_stream(path, steps)
    R, M, M2 = O.RefRunq(path), O.OracleModel(path), O.OracleModel(path)
    out = {"stream": stream, "first_flip": None, "rel_before": 0.0, "rel_corrected": 0.0,
           "device_bitwise": None if device is None else True,
           "device_rel_before": None if device is None else 0.0}
    token = 1
    for pos in range(steps):
        lr, rq, rs = R.forward_traced(token, pos, config)
        lo, oq = M.forward_kernel_order_traced(token, pos)
        lw = M2.forward_kernel_order_with(token, pos, rq, rs)
        out["rel_corrected"] = max(out["rel_corrected"], rel(lw, lr))
        if out["first_flip"] is None and not np.array_equal(rq, oq):
            out["first_flip"] = pos
        if device is not None:
            lg = device.forward(token, pos)
            if not np.array_equal(lg.view(np.uint32), lo.view(np.uint32)):
                out["device_bitwise"] = False
            if out["first_flip"] is None:
                out["device_rel_before"] = max(out["device_rel_before"], rel(lg, lr))
        if out["first_flip"] is None:
            out["rel_before"] = max(out["rel_before"], rel(lo, lr))
        token = int(stream[pos])
    for m in (R, M, M2):
        m.close()
    if out["first_flip"] is None:
        out["first_flip"] = steps
    return out


def matched_prefix(a, b) -> int:
    n = 0
    while n < min(len(a), len(b)) and int(a[n]) == int(b[n]):
        n += 1
    return n


GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def _pieces(tokenizer_path: str, vocab: int):
    import struct

    with open(tokenizer_path, "rb") as f:
        f.read(4)
        out = []
        for _ in range(vocab):
            _, n = struct.unpack("<fi", f.read(8))
            out.append(f.read(n))
    return out


def runq_piece(pieces, prev: int, tok: int) -> bytes:
    """runq.c's decode + safe_printf (runq.c:474-498): the bytes printed for
    token `tok` after `prev`."""
    p = pieces[tok]
    if prev == 1 and p[:1] == b" ":
        p = p[1:]
    if len(p) == 6 and p.startswith(b"<0x") and p.endswith(b">"):
        p = bytes([int(p[3:5], 16)])
    if len(p) == 1 and not (0x20 <= p[0] <= 0x7E or p[0] in (9, 10, 11, 12, 13)):  # C-locale isprint / isspace
        return b""
    return p


def runq_generate_greedy(path: str, tokenizer_path: str, prompt: str, steps: int):
    """runq.c's generate() with -t 0, replayed through its own forward and
    encoder (the build shim): the token fed at every position, and the bytes
    printed after each position (runq.c:681-716)."""
    vocab = synth.TINY_CONFIG[5]
    ids = O.ref_encode(tokenizer_path, vocab, prompt)
    pieces = _pieces(tokenizer_path, vocab)
    R = O.RefRunq(path)
    fed, printed = [], []
    token = int(ids[0])
    for pos in range(steps):
        lg = R.forward(token, pos)
        nxt = int(ids[pos + 1]) if pos < len(ids) - 1 else int(np.argmax(lg))
        fed.append(token)
        if nxt == 1:
            break
        printed.append(runq_piece(pieces, token, nxt))
        token = nxt
    R.close()
    return fed, printed


def first_flip_along(path: str, fed, config=synth.TINY_CONFIG) -> int:
    """First position whose int8 activations differ between runq.c and the
    kernel-order oracle (the device's arithmetic) when both are fed `fed`
    (len(fed) if none)."""
    R, M = O.RefRunq(path), O.OracleModel(path)
    first = len(fed)
    for pos, tok in enumerate(fed):
        _, rq, _ = R.forward_traced(int(tok), pos, config)
        _, oq = M.forward_kernel_order_traced(int(tok), pos)
        if not np.array_equal(rq, oq):
            first = pos
            break
    R.close()
    M.close()
    return first
