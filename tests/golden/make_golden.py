"""Generate the golden fixtures in tests/golden/ by RUNNING the reference.

The reference has no tests or golden vectors of its own, so parity is pinned
against outputs of the reference code itself, produced here:
  * tools/quantize_int8.py quantize() / tools/quantize_int4.py quantize_q4()
    (imported from the reference tree) on seeded fp32 matrices;
  * v1-int8-vnni/runq.c, compiled from its sources into oracle/_ref/librunq.so
    by oracle/Makefile: quantize_act, matmul_q8 (and its VNNI group dots,
    read out through one-group rows), and build_transformer/forward on the
    tiny config-1 checkpoint;
  * the runq binary's stdout on that checkpoint with a synthetic tokenizer.
  * runq.c's greedy streams on config-1 checkpoints of three seeds, with the
    position of the first int8 activation that differs from the kernel-order
    oracle's (the product's arithmetic) and the largest relative logits
    difference seen when the oracle is fed runq.c's own int8 activations.
Usage (needs the reference tree, so it runs only on the build machine):
    python tests/golden/make_golden.py /path/to/reference
(or set LLAMA2Q_REF to the reference project root).
"""
from __future__ import annotations

import hashlib
import importlib
import os
import subprocess
import sys
import tempfile

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.abspath(os.path.join(HERE, "..", ".."))
sys.path.insert(0, ROOT)
sys.path.insert(0, os.path.join(ROOT, "oracle"))
sys.path.insert(0, os.path.join(ROOT, "tests"))

import oracle as O  # noqa: E402
import synth  # noqa: E402
from runq_parity import flip_survey  # noqa: E402

TINY = synth.TINY_CONFIG
TINY_SEED = synth.TINY_SEED
LOGIT_POSITIONS = (0, 1, 2, 16, 63, 255)
FLIP_SEEDS = (1234, 42, 7)


def main(ref_root: str) -> None:
    sys.path.insert(0, os.path.join(ref_root, "tools"))
    q8 = importlib.import_module("quantize_int8")
    q4 = importlib.import_module("quantize_int4")
    lq = importlib.import_module("llama2-min-inference_b200")
    rng = np.random.default_rng(20261201)

    # 1. weight quantizers (GS 32 only: the reference hard-codes BLOCK = 32)
    w = (rng.standard_normal((48, 288)) * 0.02).astype(np.float32)
    w[5, 32:64] = 0.0                       # an all-zero group (scale -> 1e-8)
    w[7, 0:32] = np.linspace(-1, 1, 32)     # exact .5 ties after division
    w[9, 64:96] = 0.03                      # positive absmax saturates INT4 at 7
    q8q, q8s = q8.quantize(w)
    q4q, q4s = q4.quantize_q4(w)
    np.savez_compressed(os.path.join(HERE, "quant_ref.npz"), w=w, q8=q8q, s8=q8s, q4=q4q, s4=q4s)

    # 2. runq.c quantize_act / matmul_q8 / VNNI group dots
    xs_in = [(rng.standard_normal(288) * 0.7).astype(np.float32),
             np.zeros(288, np.float32),
             (rng.standard_normal(768) * 3).astype(np.float32)]
    xs_in[1][40] = 1e-3
    acts = {}
    for i, x in enumerate(xs_in):
        a, s, t = O.ref_quantize_act(x)
        acts[f"x{i}"], acts[f"q{i}"], acts[f"s{i}"], acts[f"t{i}"] = x, a, s, t
    np.savez_compressed(os.path.join(HERE, "act_ref.npz"), **acts)

    x = xs_in[0]
    xq, xsc, xt = O.ref_quantize_act(x)
    rows, cols = w.shape
    ng = cols // 32
    qg = q8q.reshape(rows * ng, 32).copy()
    ones = np.ones((rows * ng, 1), np.float32)
    dprime = np.empty((rows, ng), np.int64)
    for g in range(ng):
        o = O.ref_matmul_q8(xq[g * 32:(g + 1) * 32].copy(), np.ones(1, np.float32), np.zeros(1, np.float32),
                            qg, ones, rows * ng, 32)
        dprime[:, g] = o.reshape(rows, ng)[:, g].astype(np.int64)
    sums = xq.reshape(ng, 32).astype(np.int64).sum(1)
    dots = (dprime - 128 * sums[None, :]).astype(np.int32)
    y = O.ref_matmul_q8(xq, xsc, xt, q8q, q8s, rows, cols)
    np.savez_compressed(os.path.join(HERE, "gemv_ref.npz"), x=x, xq=xq, xs=xsc, dots=dots, y=y)

    # 3. tiny checkpoint through the reference quantizer and runq.c
    with tempfile.TemporaryDirectory() as d:
        f32 = os.path.join(d, "tiny_f32.bin")
        ref8 = os.path.join(d, "tiny_q8_ref.bin")
        tok = os.path.join(d, "tokenizer.bin")
        lq.write_checkpoint_fp32(f32, lq.Config.make(*TINY), TINY_SEED, 0.02, False)
        subprocess.run([sys.executable, os.path.join(ref_root, "tools", "quantize_int8.py"), f32, ref8],
                       check=True, capture_output=True)
        ref4 = os.path.join(d, "tiny_q4_ref.bin")
        subprocess.run([sys.executable, os.path.join(ref_root, "tools", "quantize_int4.py"), f32, ref4],
                       check=True, capture_output=True)
        sha8 = hashlib.sha256(open(ref8, "rb").read()).hexdigest()
        sha4 = hashlib.sha256(open(ref4, "rb").read()).hexdigest()
        R = O.RefRunq(ref8)
        # free-running greedy stream from BOS (runq.c generate, -t 0)
        stream, gaps = [], []
        token = 1
        for pos in range(TINY[6]):
            lg = R.forward(token, pos)
            nxt = int(np.argmax(lg))
            srt = np.sort(lg)
            gaps.append(float(srt[-1] - srt[-2]))
            stream.append(nxt)
            if nxt == 1:
                break
            token = nxt
        R.close()
        # teacher-forced logits at a few positions (fresh model, same tokens)
        R = O.RefRunq(ref8)
        logits = {}
        token = 1
        for pos in range(len(stream)):
            lg = R.forward(token, pos)
            if pos in LOGIT_POSITIONS:
                logits[f"logits_{pos}"] = lg
            token = stream[pos]
        R.close()
        # the runq binary's text output with the synthetic tokenizer
        synth.write_tokenizer(tok, TINY[5])
        out = subprocess.run([O.REF_RUNQ, ref8, "-z", tok, "-t", "0", "-n", str(TINY[6]), "-s", "1"],
                             check=True, capture_output=True).stdout
    np.savez_compressed(os.path.join(HERE, "tiny_runq.npz"), config=np.array(TINY, np.int32),
                        seed=np.array(TINY_SEED, np.uint64), sha256_q8=np.array(sha8), sha256_q4=np.array(sha4),
                        stream=np.array(stream, np.int32), gaps=np.array(gaps, np.float32),
                        stdout=np.frombuffer(out, np.uint8), **logits)

    # 4. int8 flip survey over three seeds (the checkpoint bytes are pinned to
    #    tools/quantize_int8.py's output for each seed)
    flips = {}
    with tempfile.TemporaryDirectory() as d:
        for seed in FLIP_SEEDS:
            f32 = os.path.join(d, f"f32_{seed}.bin")
            ref8 = os.path.join(d, f"q8_{seed}.bin")
            lq.write_checkpoint_fp32(f32, lq.Config.make(*TINY), seed, 0.02, False)
            subprocess.run([sys.executable, os.path.join(ref_root, "tools", "quantize_int8.py"), f32, ref8],
                           check=True, capture_output=True)
            ours = synth.tiny_checkpoint(8, 32, seed=seed)
            assert open(ours, "rb").read() == open(ref8, "rb").read(), seed
            f = flip_survey(ref8, TINY[6])
            stream, first, before, corrected = f["stream"], f["first_flip"], f["rel_before"], f["rel_corrected"]
            flips[f"stream_{seed}"] = stream
            flips[f"first_flip_{seed}"] = np.array(first, np.int32)
            flips[f"rel_before_{seed}"] = np.array(before, np.float64)
            flips[f"rel_corrected_{seed}"] = np.array(corrected, np.float64)
            flips[f"sha256_{seed}"] = np.array(hashlib.sha256(open(ref8, "rb").read()).hexdigest())
            print(f"seed {seed}: first int8 flip at position {first}, max rel before {before:.2e}, "
                  f"flip-corrected max rel over {TINY[6]} positions {corrected:.2e}")
    np.savez_compressed(os.path.join(HERE, "runq_flips.npz"), seeds=np.array(FLIP_SEEDS, np.int64), **flips)
    print("golden fixtures written to", HERE)


if __name__ == "__main__":
    ref = sys.argv[1] if len(sys.argv) > 1 else os.environ.get("LLAMA2Q_REF")
    if not ref:
        sys.exit("usage: make_golden.py /path/to/reference (or set LLAMA2Q_REF)")
    main(ref)
