"""Tensor-parallel split of the decode step, on the CPU: the numpy
restatement (tests/tp_ref.py) unsplit agrees with the oracle's forward, and
split over two gloo ranks (partial wo / w2 products all-reduced) agrees with
the unsplit step.  The split is the one the library applies on the GPU
(build_transformer_tp): rows of wq, wk, wv, w1, w3; columns of wo, w2."""
import os
import socket

import numpy as np
import pytest

import oracle as O
import synth
import tp_ref

CONF = synth.SMALL64_CONFIG  # dim 256, hidden 768, 4 layers, 4 heads / 2 kv heads, vocab 4096
TOKENS = [1, 17, 423, 9, 3000, 55]


def _rel(a, b):
    return float(np.abs(a - b).max() / np.abs(b).max())


@pytest.mark.parametrize("kind", [8, 4])
def test_unsplit_restatement_tracks_oracle(kind):
    path = synth.tiny_checkpoint(kind, 64, config=CONF)
    ref = tp_ref.TPStep(path)
    M = O.OracleModel(path, 64)
    for pos, tok in enumerate(TOKENS):
        a, b = ref.forward(tok, pos), M.forward(tok, pos)
        assert _rel(a, b) < 2e-3, (pos, _rel(a, b))
    M.close()


def _rank(rank, world, port, path, q):
    import torch.distributed as dist
    import tp_ref as R

    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world)

    def allreduce(v):
        import torch

        t = torch.from_numpy(np.ascontiguousarray(v, dtype=np.float32))
        dist.all_reduce(t)
        return t.numpy()

    step = R.TPStep(path, rank, world, allreduce)
    out = [step.forward(tok, pos) for pos, tok in enumerate(TOKENS)]
    q.put((rank, np.stack(out)))
    dist.destroy_process_group()


@pytest.mark.parametrize("kind", [8, 4])
def test_two_gloo_ranks_equal_unsplit(kind):
    import multiprocessing as mp
    import sys

    path = synth.tiny_checkpoint(kind, 64, config=CONF)
    here = os.path.dirname(os.path.abspath(__file__))
    sys.path[:0] = [here, os.path.join(here, "..", "oracle")]
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_rank, args=(r, 2, port, path, q)) for r in range(2)]
    for p in procs:
        p.start()
    got = dict(q.get(timeout=300) for _ in procs)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    # both ranks hold the same all-reduced stream and the replicated classifier
    assert np.array_equal(got[0], got[1])
    ref = tp_ref.TPStep(path)
    for pos, tok in enumerate(TOKENS):
        want = ref.forward(tok, pos)
        assert _rel(got[0][pos], want) < 1e-4, (pos, _rel(got[0][pos], want))
