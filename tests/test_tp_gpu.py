"""Tensor parallelism on the GPU (build_transformer_random_tp).

One GPU: the tensor-parallel step structure at tp_size 1 (products into a
partial buffer, the residual add done by the next quantizer from a second
residual buffer) gives bitwise the plain step's logits, batch 1 and batched
(tensor-core) alike.  Two GPUs (skipped with fewer): both processes return
bitwise identical logits, and they track the one-GPU model; the all-reduce
changes only the fp32 summation order of the wo / w2 products."""
import os

import numpy as np
import pytest

import synth
from gpu_util import lq

pytestmark = pytest.mark.gpu

CONF = synth.SMALL64_CONFIG
SEED = 91
TOKENS = [1, 17, 423, 9, 3000, 55, 7, 77, 777, 2]


def _cfg():
    return lq.Config.make(*CONF)


@pytest.mark.parametrize("kind", [8, 4])
def test_tp_structure_on_one_gpu_equals_plain_step(cuda, kind):
    a = lq.Transformer.random(_cfg(), kind, 64, SEED, 64)
    b = lq.Transformer.random_tp(_cfg(), kind, 64, SEED, 0, 1, None, 64)
    for pos, tok in enumerate(TOKENS):
        la = a.forward(tok, pos).copy()
        lb = b.forward(tok, pos)
        assert np.array_equal(la.view(np.uint32), lb.view(np.uint32)), pos
    for t in (a, b):
        t.reserve_batch(16)
    rng = np.random.default_rng(3)
    for pos in range(4):
        tok = rng.integers(0, CONF[5], size=16)
        la = a.forward_batch(tok, np.full(16, pos, np.int32)).copy()
        lb = b.forward_batch(tok, np.full(16, pos, np.int32))
        assert np.array_equal(la.view(np.uint32), lb.view(np.uint32)), pos
    a.close()
    b.close()


def _tp_rank(rank, world, gid, kind, q, allreduce=None):
    import importlib
    import sys

    if allreduce:
        os.environ["LQ_TP_ALLREDUCE"] = allreduce
    sys.path.insert(0, os.getcwd())
    L = importlib.import_module("llama2-min-inference_b200")
    L.lib()
    L.check(L.lib().lq_select_device(rank))
    t = L.Transformer.random_tp(L.Config.make(*CONF), kind, 64, SEED, rank, world, gid, 64)
    out = np.stack([t.forward(tok, pos).copy() for pos, tok in enumerate(TOKENS)])
    t.reserve_batch(16)
    tokb = np.arange(16, dtype=np.int32) * 31 + 1
    outb = np.stack([t.forward_batch(tokb, np.full(16, p, np.int32)).copy() for p in range(3)])
    t.close()
    q.put((rank, out, outb))


def _run_pair(kind, allreduce=None):
    import multiprocessing as mp

    gid = lq.tp_unique_id()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_tp_rank, args=(r, 2, gid, kind, q, allreduce)) for r in range(2)]
    for p in procs:
        p.start()
    got = {}
    for _ in procs:
        r, out, outb = q.get(timeout=600)
        got[r] = (out, outb)
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    return got


@pytest.mark.parametrize("kind", [8, 4])
def test_tp_two_gpus_track_one_gpu(cuda, kind):
    if cuda.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    got = _run_pair(kind)
    assert np.array_equal(got[0][0], got[1][0]) and np.array_equal(got[0][1], got[1][1])
    ref = lq.Transformer.random(_cfg(), kind, 64, SEED, 64)
    agree = 0
    for pos, tok in enumerate(TOKENS):
        want = ref.forward(tok, pos)
        rel = float(np.abs(got[0][0][pos] - want).max() / np.abs(want).max())
        assert rel < 5e-2, (pos, rel)
        agree += int(np.argmax(want) == np.argmax(got[0][0][pos]))
    assert agree >= len(TOKENS) - 1
    ref.close()


@pytest.mark.parametrize("kind", [8, 4])
def test_tp_peer_allreduce_equals_nccl(cuda, kind):
    """Batch 1 (GEMV) and batch 16 (tensor-core GEMM) steps: the peer
    all-reduce fused into the quantizer equals the NCCL all-reduce bitwise."""
    if cuda.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    peer = _run_pair(kind)
    ref = _run_pair(kind, "nccl")
    for r in range(2):
        for a, b in zip(peer[r], ref[r]):
            assert np.array_equal(a.view(np.uint32), b.view(np.uint32)), (r, float(np.abs(a - b).max()))
