"""The runner CLI (llama2-min-inference_b200/bin/run, the reference runners'
command line over the C ABI): greedy generation prints the pieces of the
same token stream the API produces, decoded as runq.c decodes them, reports
the "achieved tok/s" line on stderr, and starts like runq.c itself on the
same checkpoint and tokenizer."""
import os
import struct
import subprocess

import numpy as np
import pytest

import synth
from gpu_util import lq

pytestmark = pytest.mark.gpu

ROOT = os.path.abspath(os.path.join(os.path.dirname(__file__), ".."))
RUN = os.path.join(ROOT, "llama2-min-inference_b200", "bin", "run")
RUNQ = os.path.join(ROOT, "oracle", "_ref", "runq")


def _pieces(path, vocab):
    with open(path, "rb") as f:
        f.read(4)
        out = []
        for _ in range(vocab):
            _, n = struct.unpack("<fi", f.read(8))
            out.append(f.read(n))
    return out


def _decode(pieces, prev, tok):
    """runq.c's decode + safe print (runq.c:519-541)."""
    p = pieces[tok]
    if prev == 1 and p[:1] == b" ":
        p = p[1:]
    if len(p) == 6 and p.startswith(b"<0x") and p.endswith(b">"):
        p = bytes([int(p[3:5], 16)])
    if len(p) == 1 and not (0x20 <= p[0] <= 0x7E or p[0] in (9, 10, 11, 12, 13)):  # C-locale isprint / isspace
        return b""
    return p


def _expected(steps):
    t = lq.Transformer.from_file(synth.tiny_checkpoint(8, 32))
    pieces = _pieces(synth.tiny_tokenizer(), synth.TINY_CONFIG[5])
    out, token = b"", 1
    for pos in range(steps):
        nxt = t.forward_argmax(token, pos)
        if nxt == 1:
            break
        out += _decode(pieces, token, nxt)
        token = nxt
    t.close()
    return out + b"\n"


def test_runner_greedy_stream_equals_api(cuda):
    steps = 40
    r = subprocess.run([RUN, synth.tiny_checkpoint(8, 32), "-z", synth.tiny_tokenizer(), "-t", "0", "-n",
                        str(steps)], capture_output=True, timeout=300)
    assert r.returncode == 0, r.stderr.decode(errors="replace")
    assert r.stdout == _expected(steps)
    assert b"achieved tok/s:" in r.stderr


def test_runner_starts_like_runq(cuda):
    """runq.c and the B200 step agree token for token until an int8 rounding
    flip (documented in the parity notes); the first tokens' text matches."""
    if not os.path.exists(RUNQ):
        pytest.skip("runq.c was not built on this machine")
    args = [synth.tiny_checkpoint(8, 32), "-z", synth.tiny_tokenizer(), "-t", "0", "-n", "9"]
    ours = subprocess.run([RUN] + args, capture_output=True, timeout=300)
    ref = subprocess.run([RUNQ] + args, capture_output=True, timeout=300, env=dict(os.environ, OMP_NUM_THREADS="4"))
    if ref.returncode != 0:
        pytest.skip("runq.c does not run on this host: " + ref.stderr.decode(errors="replace")[:200])
    assert ours.returncode == 0
    assert ours.stdout == ref.stdout


RUNQ_CASES = {
    # chat template with a system prompt (runq.c:731-794), greedy
    "chat_greedy": ["-m", "chat", "-i", "What is a whale?", "-y", "You answer briefly.", "-t", "0", "-n", "64"],
    # seeded top-p sampling from BOS (runq.c:604-667: xorshift64*, temperature, nucleus)
    "sample_t0.8_s7": ["-t", "0.8", "-s", "7", "-n", "64"],
    # prompt encoding (runq.c:500-560) then seeded sampling
    "prompt_sample": ["-i", "Once upon a time", "-t", "0.8", "-p", "0.9", "-s", "11", "-n", "64"],
}


@pytest.mark.parametrize("case", sorted(RUNQ_CASES))
@pytest.mark.parametrize("seed", [42, 1234])
def test_runner_output_equals_runq(cuda, case, seed):
    """The runner and runq.c itself, same checkpoint, tokenizer and flags:
    byte-identical stdout (both computations are deterministic, and their
    logits agree to ~3e-7 relative until an int8 rounding flip, which these
    short runs do not turn into a different token)."""
    if not os.path.exists(RUNQ):
        pytest.skip("runq.c was not built on this machine")
    args = [synth.tiny_checkpoint(8, 32, seed=seed), "-z", synth.tiny_tokenizer()] + RUNQ_CASES[case]
    user_lines = b"Tell me more.\n" * 32  # later chat turns, if the model ends one (token 2)
    ref = subprocess.run([RUNQ] + args, capture_output=True, timeout=300, input=user_lines,
                         env=dict(os.environ, OMP_NUM_THREADS="4"))
    if ref.returncode != 0:
        pytest.skip("runq.c does not run on this host: " + ref.stderr.decode(errors="replace")[:200])
    ours = subprocess.run([RUN] + args, capture_output=True, timeout=300, input=user_lines)
    assert ours.returncode == 0, ours.stderr.decode(errors="replace")
    n = 0
    while n < min(len(ours.stdout), len(ref.stdout)) and ours.stdout[n] == ref.stdout[n]:
        n += 1
    print(f"{case} seed {seed}: {n} of {len(ref.stdout)} bytes identical")
    assert ours.stdout == ref.stdout
