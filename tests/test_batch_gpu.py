"""Batched decode (forward_batch): B independent sequences advanced together.

Every row of a batched step must be bitwise the batch-1 forward of that
sequence (same tokens, same positions): the GEMV computes each activation row
with the same per-row reduction order whatever the batch, and attention, the
quantizers and the caches are per sequence.  The batch-1 forward itself is
bitwise the kernel-order oracle (test_forward_gpu.py), so this pins every
batched row to the oracle too."""
import numpy as np
import pytest

import synth
from gpu_util import lq

pytestmark = pytest.mark.gpu


def _model(kind, gs, max_seq=96, config=synth.SMALL64_CONFIG, seed=77):
    return lq.Transformer.random(lq.Config.make(*config), kind, gs, seed, max_seq)


def _histories(rng, batch, vocab, starts, steps):
    """Token history per sequence: sequence b joins the batch at step starts[b]."""
    return [list(rng.integers(0, vocab, size=steps - starts[b] + 1)) for b in range(batch)]


def _run_batched(t, hist, starts, steps):
    """Step s runs the sequences that have joined (a prefix of the rows)."""
    out = {}
    for s in range(steps):
        rows = [b for b in range(len(hist)) if starts[b] <= s]
        n = max(rows) + 1
        assert rows == list(range(n))
        tok = [hist[b][s - starts[b]] for b in range(n)]
        pos = [s - starts[b] for b in range(n)]
        lg = t.forward_batch(tok, pos)
        for b in range(n):
            out[(b, pos[b])] = lg[b].copy()
    return out


def _run_single(t, hist_b, npos):
    return [t.forward(int(hist_b[p]), p).copy() for p in range(npos)]


@pytest.mark.parametrize("kind,batch", [(8, 5), (4, 3), (8, 13)])
def test_batched_rows_equal_batch1_forward(cuda, kind, batch):
    """Rows join at different steps, so each step mixes positions and the
    batch size grows (new graph per size, padded GEMV chunks)."""
    rng = np.random.default_rng(batch * 10 + kind)
    vocab = synth.SMALL64_CONFIG[5]
    steps = 20
    starts = sorted(int(v) for v in rng.integers(0, 8, size=batch))
    starts[0] = 0
    hist = _histories(rng, batch, vocab, starts, steps)
    tb = _model(kind, 64)
    tb.reserve_batch(batch)
    got = _run_batched(tb, hist, starts, steps)
    tb.close()
    t1 = _model(kind, 64)
    for b in range(batch):
        ref = _run_single(t1, hist[b], steps - starts[b])
        for p, r in enumerate(ref):
            g = got[(b, p)]
            assert np.array_equal(g.view(np.uint32), r.view(np.uint32)), (b, p, float(np.abs(g - r).max()))
    t1.close()


def test_batched_argmax_matches_logits(cuda):
    t = _model(8, 64)
    t.reserve_batch(8)
    rng = np.random.default_rng(5)
    tok = rng.integers(0, synth.SMALL64_CONFIG[5], size=8)
    pos = np.zeros(8, np.int32)
    for step in range(4):
        lg = t.forward_batch(tok, pos).copy()
        # same step again on a fresh position via the argmax entry point
        nxt = t.forward_batch_argmax(tok, pos)
        assert np.array_equal(nxt, np.argmax(lg, axis=1).astype(np.int32))
        tok, pos = nxt, pos + 1
    t.close()


def test_batched_greedy_streams_are_independent(cuda):
    """Greedy decoding of 8 identical prompts gives 8 identical streams, and
    one different prompt does not disturb the others."""
    t = _model(4, 64)
    t.reserve_batch(8)
    tok = np.full(8, 1, np.int32)
    tok[5] = 17
    streams = []
    for p in range(24):
        tok = t.forward_batch_argmax(tok, np.full(8, p, np.int32))
        streams.append(tok.copy())
    t.close()
    s = np.stack(streams, 1)
    for b in range(8):
        if b != 5:
            assert np.array_equal(s[b], s[0])
    t1 = _model(4, 64)
    tk, ref = 1, []
    for p in range(24):
        tk = t1.forward_argmax(tk, p)
        ref.append(tk)
    t1.close()
    assert list(s[0]) == ref


def test_batch_errors(cuda):
    t = _model(8, 64)
    with pytest.raises(lq.LlamaQError):
        t.forward_batch([1, 2], [0, 0])  # max_batch is 1
    t.reserve_batch(4)
    with pytest.raises(lq.LlamaQError):
        t.forward_batch([1, 2, 3, 4, 5], [0] * 5)
    with pytest.raises(lq.LlamaQError):
        t.forward_batch([1, 10 ** 6], [0, 0])
    with pytest.raises(lq.LlamaQError):
        t.forward_batch([1, 2], [0, 96])
    with pytest.raises(lq.LlamaQError):
        t.reserve_batch(0)
    t.reserve_batch(2)
    assert t.forward_batch([1, 2], [0, 0]).shape == (2, synth.SMALL64_CONFIG[5])
    t.close()


@pytest.mark.parametrize("kind,batch", [(8, 16), (4, 20)])
def test_tensor_core_batch_bit_exact_vs_oracle(cuda, kind, batch):
    """From 16 sequences on, every product of the step runs on the tensor
    cores (tcgen05 kind::i8); each row equals the oracle's restatement of
    that order for its own sequence, bit for bit."""
    import oracle as O

    conf = synth.SMALL64_CONFIG
    path = synth.tiny_checkpoint(kind, 64, config=conf)
    t = lq.Transformer.from_file(path, 64)
    t.reserve_batch(batch)
    rng = np.random.default_rng(batch + kind)
    steps = 12
    hist = rng.integers(0, conf[5], size=(batch, steps))
    got = []
    for p in range(steps):
        got.append(t.forward_batch(hist[:, p], np.full(batch, p, np.int32)).copy())
    t.close()
    sms = cuda.cuda.get_device_properties(0).multi_processor_count
    M = O.OracleModel(path, 64)
    M.set_mma_grid(sms)
    for b in range(batch):
        for p in range(steps):
            lo = M.forward_kernel_order(int(hist[b, p]), p)
            g = got[p][b]
            assert np.array_equal(g.view(np.uint32), lo.view(np.uint32)), (b, p, float(np.abs(g - lo).max()))
    M.close()
