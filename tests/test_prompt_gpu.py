"""Prompt prefill (forward_prompt): the prompt's tokens run through each step
as rows of one sequence, each row writing its own cache position and
attending causally over the cache up to it.

Per row the arithmetic is that of a decode step: below 16 rows the products
run on the GEMV, whose per-row order is the batch-1 forward's, so the prompt
logits equal feeding the tokens one at a time bit for bit; from 16 rows they
run on the tensor-core GEMM, and every row equals the kernel-order oracle's
restatement of that order.  A prompt of more than 64 tokens runs in steps of
64 rows (the last step may fall back to the GEMV)."""
import numpy as np
import pytest

import oracle as O
import synth
from gpu_util import lq

pytestmark = pytest.mark.gpu

CONF = synth.SMALL64_CONFIG  # head 64, 2:1 grouped-query attention, seq 128


def _prompt(n, seed=5):
    return np.random.default_rng(seed).integers(3, CONF[5], size=n).astype(np.int32)


def _bits(a):
    return np.ascontiguousarray(a, np.float32).view(np.uint32)


@pytest.mark.parametrize("kind", [8, 4])
def test_short_prompt_equals_token_by_token(cuda, kind):
    """9 prompt tokens (GEMV rows): the last token's logits, and the greedy
    continuation after the prompt, are bitwise those of feeding the prompt
    one token at a time."""
    path = synth.tiny_checkpoint(kind, 64, config=CONF)
    toks = _prompt(9)
    a = lq.Transformer.from_file(path)
    b = lq.Transformer.from_file(path)
    la = a.forward_prompt(toks).copy()
    for pos, tok in enumerate(toks):
        lb = b.forward(int(tok), pos).copy()
    assert np.array_equal(_bits(la), _bits(lb))
    ta = tb = int(np.argmax(la))
    for pos in range(len(toks), len(toks) + 8):
        na, nb = a.forward_argmax(ta, pos), b.forward_argmax(tb, pos)
        assert na == nb, pos
        ta, tb = na, nb
    a.close()
    b.close()


@pytest.mark.parametrize("kind,n", [(8, 40), (4, 40), (8, 100)])
def test_prompt_bit_exact_vs_kernel_order_oracle(cuda, kind, n):
    """Prompts of 40 tokens (one tensor-core step) and 100 tokens (a 64-row
    tensor-core step, then 36 rows): the last token's logits equal the oracle
    fed the prompt one token at a time in the device's order for each step's
    rows (the tensor-core GEMM's from 16 rows, the GEMV's below), bit for bit;
    the greedy decode after the prompt (batch-1 GEMV steps) stays bitwise
    equal to the oracle in the GEMV's order."""
    path = synth.tiny_checkpoint(kind, 64, config=CONF)
    toks = _prompt(n, seed=n)
    t = lq.Transformer.from_file(path)
    lg = t.forward_prompt(toks).copy()
    sms = cuda.cuda.get_device_properties(0).multi_processor_count
    M = O.OracleModel(path)
    for c0 in range(0, n, 64):
        rows = min(64, n - c0)
        M.set_mma_grid(sms if rows >= 16 else 0)
        for pos in range(c0, c0 + rows):
            lo = M.forward_kernel_order(int(toks[pos]), pos)
    assert np.array_equal(_bits(lg), _bits(lo)), float(np.abs(lg - lo).max())
    M.set_mma_grid(0)
    tok = int(np.argmax(lo))
    for pos in range(n, n + 6):
        lo = M.forward_kernel_order(tok, pos)
        lg = t.forward(tok, pos)
        assert np.array_equal(_bits(lg), _bits(lo)), pos
        tok = int(np.argmax(lo))
    t.close()
    M.close()


def test_prompt_continues_at_a_position(cuda):
    """A prompt split in two calls (the second at start_pos = length of the
    first) gives the same logits as one call of the whole prompt when both
    halves stay on the GEMV (below 16 rows per step)."""
    path = synth.tiny_checkpoint(8, 64, config=CONF)
    toks = _prompt(12, seed=9)
    a = lq.Transformer.from_file(path)
    b = lq.Transformer.from_file(path)
    la = a.forward_prompt(toks).copy()
    b.forward_prompt(toks[:5])
    lb = b.forward_prompt(toks[5:], 5).copy()
    assert np.array_equal(_bits(la), _bits(lb))
    a.close()
    b.close()


def test_prompt_errors(cuda):
    t = lq.Transformer.from_file(synth.tiny_checkpoint(8, 64, config=CONF))
    with pytest.raises(lq.LlamaQError):
        t.forward_prompt(np.zeros(0, np.int32))
    with pytest.raises(lq.LlamaQError):
        t.forward_prompt(_prompt(10), CONF[6] - 5)  # runs past the last position
    with pytest.raises(lq.LlamaQError):
        t.forward_prompt(np.array([1, CONF[5]], np.int32))  # token out of range
    assert t.forward_prompt(_prompt(3)).shape == (CONF[5],)  # still usable
    t.close()
