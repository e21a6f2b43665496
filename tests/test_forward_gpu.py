"""GPU decode step (forward) against runq.c and the oracle.

runq.c and any other correct implementation that sums in a different fp32
order agree to a few ulp until an fp32 value lands within an ulp of an int8
rounding boundary in one of the step's activation quantizations; from then
on the two runs see one different int8 value and the logits drift apart (a
property of the reference's own arithmetic: any re-association of its sums
flips a value within the first few to few dozen positions).  The parity
tests therefore check, for three config-1 seeds:
  * the device step equals the kernel-order oracle (runq.c's forward with the
    fp32 sums associated as the kernels do) bit for bit at every position;
  * before the first int8 flip the device logits are within 1e-3 relative of
    runq.c's (measured: ~3e-7);
  * over all 256 positions, the oracle fed runq.c's own int8 activations is
    within 1e-3 of runq.c (measured: ~3e-7), i.e. every larger difference is
    an int8 flip, not an arithmetic error;
  * the device's free-running greedy stream equals runq.c's at least up to
    the first flip.
and the kernel-order comparison runs on the shapes the benchmarks use (head
size 128, 8:1 grouped-query attention, contexts over 1100 positions)."""
import numpy as np
import pytest

import oracle as O
import synth
from gpu_util import lq
from runq_parity import flip_survey, matched_prefix, rel, runq_usable

pytestmark = pytest.mark.gpu


def _rel(a, b):
    return float(np.abs(a - b).max() / np.abs(b).max())


def test_tiny_int8_logits_match_runq(cuda, golden):
    """Golden runq.c logits (seed 1234): within 1e-3 relative at the golden
    positions before this checkpoint's first int8 flip; the later golden
    positions are past flips and only sanity-bounded."""
    g = golden("tiny_runq.npz")
    first = int(golden("runq_flips.npz")["first_flip_1234"])
    stream = g["stream"]
    t = lq.Transformer.from_file(synth.tiny_checkpoint(8, 32))
    token, errs = 1, {}
    for pos in range(len(stream)):
        lg = t.forward(token, pos)
        if f"logits_{pos}" in g.files:
            errs[pos] = rel(lg, g[f"logits_{pos}"])
        token = int(stream[pos])
    t.close()
    print(f"teacher-forced relative logits error vs runq.c (first int8 flip at {first}):", errs)
    assert any(pos < first for pos in errs)
    for pos, e in errs.items():
        assert e < (1e-3 if pos < first else 5e-2), (pos, e)


@pytest.mark.parametrize("seed", [1234, 42, 7])
def test_greedy_stream_vs_runq_fixture(cuda, golden, seed):
    """The device's free-running greedy stream (forward_argmax from BOS)
    equals runq.c's stream for this seed at least up to the first int8 flip
    recorded in the fixture; the matched length is printed."""
    f = golden("runq_flips.npz")
    want, first = f[f"stream_{seed}"], int(f[f"first_flip_{seed}"])
    t = lq.Transformer.from_file(synth.tiny_checkpoint(8, 32, seed=seed))
    token, got = 1, []
    for pos in range(len(want)):
        token = t.forward_argmax(token, pos)
        got.append(token)
    t.close()
    same = matched_prefix(got, want)
    print(f"seed {seed}: greedy stream identical to runq.c for {same} of {len(want)} steps "
          f"(first int8 flip at {first})")
    assert same >= first


@pytest.mark.parametrize("seed", [1234, 42, 7])
def test_flip_aware_parity_vs_runq(cuda, seed):
    """Live comparison with runq.c (built from the reference sources into
    oracle/_ref): teacher-forced with runq.c's greedy stream over 256
    positions, the device logits equal the kernel-order oracle's bitwise at
    every position, are within 1e-3 relative of runq.c's before the first
    int8 flip, and the oracle fed runq.c's int8 activations stays within
    1e-3 of runq.c at every position."""
    why = runq_usable()
    if why:
        pytest.skip(why)
    path = synth.tiny_checkpoint(8, 32, seed=seed)
    t = lq.Transformer.from_file(path)
    r = flip_survey(path, 256, device=t)
    t.close()
    print(f"seed {seed}: first int8 flip at {r['first_flip']}; device vs runq.c before it "
          f"{r['device_rel_before']:.2e}; flip-corrected oracle vs runq.c over 256 positions "
          f"{r['rel_corrected']:.2e}")
    assert r["device_bitwise"]
    assert r["first_flip"] > 0
    assert r["device_rel_before"] < 1e-3
    assert r["rel_corrected"] < 1e-3


def test_argmax_matches_host_argmax(cuda):
    t = lq.Transformer.from_file(synth.tiny_checkpoint(8, 32))
    token = 1
    for pos in range(16):
        lg = t.forward(token, pos).copy()
        nxt = t.forward_argmax(token, pos)  # same position again: same logits
        assert nxt == int(np.argmax(lg))
        token = nxt
    t.close()


KERNEL_ORDER_CASES = [
    (8, 32, synth.TINY_CONFIG, 72),     # config 1 shape: dim 288 / head 48, plain-load GEMV for n=288
    (4, 32, synth.TINY_CONFIG, 72),     # INT4, group 32
    (8, 64, synth.SMALL64_CONFIG, 72),  # GS 64, GQA (4 heads / 2 kv heads), bulk-copy GEMV
    (4, 64, synth.SMALL64_CONFIG, 72),
    (8, 64, synth.HEAD128_CONFIG, 1100),  # head 128, 1100 positions: the merge of 18 attention chunks
    (4, 64, synth.HEAD128_CONFIG, 1100),
    (8, 64, synth.GQA8_CONFIG, 1100),     # head 128, 8 query heads per kv head (the 70B layout)
    (4, 64, synth.GQA8_CONFIG, 1100),
]


@pytest.mark.parametrize("kind,gs,conf,steps", KERNEL_ORDER_CASES)
def test_forward_bit_exact_vs_kernel_order_oracle(cuda, kind, gs, conf, steps):
    """The decode step equals the oracle's kernel-order restatement of
    runq.c's forward bit for bit, free running (greedy, from BOS) over more
    than 64 positions, so both attention paths (one chunk, merged chunks)
    are covered; the head-128 cases run 1100 positions (18 chunks merged)
    with one and with eight query heads per kv head.  INT4 and GS 64 have no
    reference CPU runner; the oracle restates runq.c's forward with those
    parameters."""
    path = synth.tiny_checkpoint(kind, gs, config=conf)
    t = lq.Transformer.from_file(path)
    M = O.OracleModel(path)
    token = 1
    for pos in range(min(steps, conf[6])):
        lo = M.forward_kernel_order(token, pos)
        lg = t.forward(token, pos)
        assert np.array_equal(lg.view(np.uint32), lo.view(np.uint32)), (pos, _rel(lg, lo))
        token = int(np.argmax(lo))
    t.close()
    M.close()


@pytest.mark.parametrize("kind,gs", [(8, 64), (4, 64)])
def test_random_init_on_device_equals_file(cuda, kind, gs):
    """build_transformer_random generates the same weights on the device as
    the host generator + quantizer write to the file: identical logits."""
    conf = synth.SMALL64_CONFIG
    a = lq.Transformer.from_file(synth.tiny_checkpoint(kind, gs, config=conf))
    b = lq.Transformer.random(lq.Config.make(*conf), kind, gs, synth.TINY_SEED)
    token = 1
    for pos in range(8):
        la = a.forward(token, pos).copy()
        lb = b.forward(token, pos)
        assert np.array_equal(la, lb)
        token = int(np.argmax(la))
    a.close()
    b.close()


def test_bad_token_and_position_rejected(cuda):
    t = lq.Transformer.from_file(synth.tiny_checkpoint(8, 32))
    with pytest.raises(lq.LlamaQError):
        t.forward_argmax(32000, 0)
    with pytest.raises(lq.LlamaQError):
        t.forward_argmax(1, 256)
    assert t.forward_argmax(1, 0) >= 0  # still usable
    t.close()
