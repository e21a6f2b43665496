"""Tensor parallelism on the GPU (build_transformer_tp / build_transformer_random_tp).

One GPU: the tensor-parallel step structure at tp_size 1 (products into a
partial buffer, the residual add done by the next quantizer from a second
residual buffer) gives bitwise the plain step's logits, batch 1 and batched
(tensor-core) alike; the all-reduce's bounded wait gives up and reports
LQ_ETIMEOUT when no peer publishes.  2, 4 and 8 GPUs (each size skipped when
fewer GPUs are visible): every process returns the same logits, bit for bit
equal to the oracle's restatement of the tensor-parallel step (wo and w2 as
per-process column-slice products, summed in process order); the peer
all-reduce fused into the quantizer agrees with the NCCL all-reduce (bitwise
at 2 GPUs, where both sums are y_0 + y_1); and a process that stops taking
part between steps makes its peers' next step fail with LQ_ETIMEOUT instead
of hanging."""
import os

import numpy as np
import pytest

import oracle as O
import synth
from gpu_util import lq

pytestmark = pytest.mark.gpu

CONF = synth.SMALL64_CONFIG
SEED = 91
TOKENS = [1, 17, 423, 9, 3000, 55, 7, 77, 777, 2]
# 16 query heads / 8 kv heads (head 64): splits over 2, 4 and 8 processes
TP_CONF = (1024, 2048, 2, 16, 8, 512, 128)
TP_TOKENS = [1, 17, 423, 9, 300, 55, 7, 77]


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


def test_tp_wait_gives_up_with_timeout(cuda):
    """The all-reduce quantizer as rank 0 of a group whose peers never
    publish: the bounded wait gives up after its limit (50 ms here) and the
    status is LQ_ETIMEOUT; the next call of the same step does not wait
    again."""
    for size in (2, 8):
        rc, first_ms, second_ms = lq.tp_wait_selftest(size, 50_000)
        assert rc == lq.ETIMEOUT, (rc, lq.last_error())
        assert first_ms >= 45.0, first_ms
        assert second_ms < 10.0, second_ms


def _visible(cuda, world):
    if cuda.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")


def _tp_rank(rank, world, gid, kind, q, mode, env):
    import importlib
    import sys

    os.environ.update(env)
    sys.path.insert(0, os.getcwd())
    L = importlib.import_module("llama2-min-inference_b200")
    L.check(L.lib().lq_select_device(rank))
    try:
        if mode == "file":
            path = synth.tiny_checkpoint(kind, 64, config=TP_CONF, seed=SEED)
            t = L.Transformer.from_file_tp(path, rank, world, gid)
            out = np.stack([t.forward(tok, pos).copy() for pos, tok in enumerate(TP_TOKENS)])
            t.close()
            q.put((rank, out, None))
        elif mode == "batch":
            t = L.Transformer.random_tp(L.Config.make(*TP_CONF), kind, 64, SEED, rank, world, gid, 64)
            out = np.stack([t.forward(tok, pos).copy() for pos, tok in enumerate(TP_TOKENS)])
            # 80 rows: more than the 64 the exchange region was set up for (it is
            # set up again), two tensor-core chunks (slot rows 0-63, 64-79)
            t.reserve_batch(80)
            tokb = (np.arange(80, dtype=np.int32) * 31 + 1) % TP_CONF[5]
            outb = np.stack([t.forward_batch(tokb, np.full(80, p, np.int32)).copy() for p in range(3)])
            t.close()
            q.put((rank, out, outb))
        elif mode == "stop":
            # rank 1 skips the third step (it stays alive and keeps its memory
            # mapped); rank 0's third step must come back with LQ_ETIMEOUT
            t = L.Transformer.random_tp(L.Config.make(*TP_CONF), kind, 64, SEED, rank, world, gid, 64)
            for pos in range(2):
                t.forward_argmax(TP_TOKENS[pos], pos)
            code = 0
            if rank == 0:
                try:
                    t.forward_argmax(TP_TOKENS[2], 2)
                except L.LlamaQError as e:
                    code = e.code
            t.close()
            q.put((rank, code, None))
    except Exception as e:  # reported to the parent, which fails the test
        q.put((rank, None, repr(e)))


def _run_group(world, kind, mode, env=None):
    import multiprocessing as mp

    if mode == "file":
        synth.tiny_checkpoint(kind, 64, config=TP_CONF, seed=SEED)  # written once, before the processes read it
    gid = lq.tp_unique_id()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_tp_rank, args=(r, world, gid, kind, q, mode, env or {})) for r in range(world)]
    for p in procs:
        p.start()
    got = {}
    for _ in procs:
        r, a, b = q.get(timeout=600)
        assert a is not None, (r, b)
        got[r] = (a, b)
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    return got


@pytest.mark.parametrize("world", [2, 4, 8])
@pytest.mark.parametrize("kind", [8, 4])
def test_tp_equals_tp_oracle(cuda, world, kind):
    """Every process's batch-1 logits equal the kernel-order oracle of the
    tensor-parallel step bit for bit (teacher-forced, 8 positions), for a
    checkpoint loaded and split by the processes themselves."""
    _visible(cuda, world)
    got = _run_group(world, kind, "file")
    M = O.OracleModel(synth.tiny_checkpoint(kind, 64, config=TP_CONF, seed=SEED))
    M.set_tp(world)
    for pos, tok in enumerate(TP_TOKENS):
        want = M.forward_kernel_order(tok, pos)
        for r in range(world):
            lg = got[r][0][pos]
            assert np.array_equal(lg.view(np.uint32), want.view(np.uint32)), (r, pos, float(np.abs(lg - want).max()))
    M.close()


@pytest.mark.parametrize("world", [2, 4, 8])
@pytest.mark.parametrize("kind", [8, 4])
def test_tp_peer_allreduce_vs_nccl(cuda, world, kind):
    """Batch 1 (GEMV) and batch 80 (tensor-core GEMM in chunks of 64 and 16
    rows, after a batch reservation beyond the rows the exchange region was
    first set up for) steps: the peer all-reduce fused into the quantizer
    against the NCCL all-reduce.  With 2
    processes both sums are y_0 + y_1, so the logits are bitwise equal; with
    more, NCCL may associate the sum differently, so the logits agree to
    fp32 rounding until an int8 activation flips (argmax agreement checked)."""
    _visible(cuda, world)
    peer = _run_group(world, kind, "batch")
    ref = _run_group(world, kind, "batch", {"LQ_TP_ALLREDUCE": "nccl"})
    for r in range(world):
        assert np.array_equal(peer[r][0], peer[0][0]) and np.array_equal(peer[r][1], peer[0][1]), r
        for a, b in zip(peer[r], ref[r]):
            if world == 2:
                assert np.array_equal(a.view(np.uint32), b.view(np.uint32)), (r, float(np.abs(a - b).max()))
            else:
                agree = np.mean(np.argmax(a, -1) == np.argmax(b, -1))
                rel = float(np.abs(a - b).max() / np.abs(b).max())
                print(f"world {world} rank {r}: peer vs NCCL max rel {rel:.2e}, argmax agreement {agree:.2f}")
                assert agree >= 0.75 and rel < 5e-2


def test_tp_peer_stops_between_steps(cuda):
    """A process that stops taking part between steps (alive, memory still
    mapped) makes its peer's next decode step return LQ_ETIMEOUT after the
    wait limit (LQ_TP_WAIT_MS = 200) instead of hanging."""
    _visible(cuda, 2)
    got = _run_group(2, 8, "stop", {"LQ_TP_WAIT_MS": "200"})
    assert got[0][0] == lq.ETIMEOUT
