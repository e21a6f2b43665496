"""Benchmark of the decode hot path: batch-1 group-quantized GEMV.

Workload: INT8 weights, group size 64, symmetric fp32
group scales, from N(0, 0.02)-like synthetic values; activations fp32
~N(0,1) quantized per 64-group inside the GEMV; Llama-2-7B layer shapes
(n, d) = (4096, 4096) x4 [wq wk wv wo], (4096, 11008) x2 [w1 w3],
(11008, 4096) [w2], (4096, 32000) [classifier].  One step = one pass over
the eight products (eight kernel launches), captured in a CUDA graph with
programmatic dependent launch; two copies of every matrix (0.71 GB in all,
over 5x the 126 MB L2) alternate between steps so every weight byte comes
from HBM.

Metric: GB/s of algorithmic bytes (weights + scales + fp32 x in + fp32 y
out, each byte once) over the timed steps, summed over ranks.  One process
per GPU (torchrun for N > 1); every rank runs the same sweep on its own GPU
(replicas: a batch-1 GEMV does not shard), timing = max over ranks.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl reference]

--impl reference times the reference's own CPU path (runq.c matmul_q8,
compiled from its sources into oracle/_ref/librunq.so; group size 32, the
only one it supports) on the same shapes with all host threads.
"""
from __future__ import annotations

import argparse
import importlib
import json
import os
import statistics
import subprocess
import sys
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)
sys.path.insert(0, os.path.join(ROOT, "oracle"))

SHAPES = [(4096, 4096)] * 4 + [(4096, 11008)] * 2 + [(11008, 4096), (4096, 32000)]  # (n, d)
GS = 64
KIND = 8
COPIES = 2
METRIC = "quantized-GEMV HBM GB/s (INT8 GS64 batch-1 sweep over Llama-2-7B layer shapes)"
WORKLOAD = "config2: int8 gs64 batch-1 GEMV sweep, llama-2-7b shapes (wq,wk,wv,wo,w1,w3,w2,wcls)"


def gemv_bytes(n: int, d: int, gs: int, kind: int, act_bytes_per_elem: float = 4.0) -> int:
    wb = d * n if kind == 8 else d * n // 2
    return int(wb + d * (n // gs) * 4 + n * act_bytes_per_elem + 4 * d)


def step_bytes() -> int:
    return sum(gemv_bytes(n, d, GS, KIND) for n, d in SHAPES)


def peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(p) as f:
            j = json.load(f)
        return float(j["hbm_gbs"]), "measured"
    except Exception:
        return 6650.0, "fallback"


def traffic_per_launch():
    """DRAM bytes per GEMV launch from the committed ncu summary, if any."""
    p = os.path.join(ROOT, "profiles", "gemv_traffic.json")
    try:
        with open(p) as f:
            return json.load(f)
    except Exception:
        return None


# ---------------------------------------------------------------------------
# clocks during the timed region

class ClockSampler:
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None
        self.path = os.path.join("/tmp", f"lq_clocks_{os.getpid()}.csv")

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits", "-lms", "100",
                 "-i", str(self.gpu)], stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
            time.sleep(0.3)
        except Exception:
            self.proc = None

    def stop(self):
        if not self.proc:
            return None
        time.sleep(0.2)
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        rows = []
        for line in open(self.path):
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                rows.append((float(parts[1]), float(parts[2]), float(parts[3]), parts[5:9]))
            except ValueError:
                continue
        os.remove(self.path)
        if not rows:
            return None
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows for i, v in enumerate(r[3]) if v.lower() == "active"})
        loaded = [r for r in rows if r[2] > 200.0] or rows
        return {"sm_mhz": statistics.median(r[0] for r in loaded), "sm_max_mhz": max(r[1] for r in rows),
                "reasons": reasons, "samples": len(rows)}


# ---------------------------------------------------------------------------
# CPU baseline: the reference's runq.c matmul_q8 (or the scalar oracle)

def cpu_has_vnni() -> bool:
    try:
        flags = open("/proc/cpuinfo").read()
    except Exception:
        return False
    return all(f in flags for f in ("avx512_vnni", "avx512vl", "avx512bw", "avx512f"))


def cpu_baseline(seconds: float = 10.0, steps: int | None = None, warmup: int = 0):
    """Returns (GB/s, kind, cores, sample description, per-step seconds)."""
    import oracle as O

    rng = np.random.default_rng(0)
    use_ref = O.ref_available() and cpu_has_vnni()
    cores = os.cpu_count() or 1
    if use_ref:
        O.ref().ref_set_threads(cores)
        mats = []
        for n, d in SHAPES:
            q = rng.integers(0, 256, size=(d, n), dtype=np.uint8)
            s = (rng.random((d, n // 32), dtype=np.float32) * 1e-3).astype(np.float32)
            x = rng.standard_normal(n).astype(np.float32)
            xq, xs, xt = O.ref_quantize_act(x)
            mats.append((n, d, q, s, xq, xs, xt))
        per = sum(gemv_bytes(n, d, 32, 8, 1 + 8 / 32) for n, d in SHAPES)

        def one():
            for n, d, q, s, xq, xs, xt in mats:
                O.ref_matmul_q8(xq, xs, xt, q, s, d, n)
        kind, desc = "reference", "runq.c matmul_q8 (AVX-512 VNNI + OpenMP, group size 32) over the 8 shapes"
    else:
        cores = 1
        n, d = SHAPES[0]
        w = (rng.standard_normal((d, n)) * 0.02).astype(np.float32)
        q, s = O.quantize_weight(w, GS, KIND)
        x = rng.standard_normal(n).astype(np.float32)
        xq, xs, _ = O.quantize_act(x, GS)
        per = gemv_bytes(n, d, GS, KIND, 1 + 4 / GS)

        def one():
            O.gemv(xq, xs, q, s, n, GS, KIND)
        kind, desc = "port", "scalar C oracle GEMV, one 4096x4096 INT8 GS64 matrix per step (1 thread)"
    for _ in range(max(1, warmup)):
        one()
    times = []
    t_end = time.perf_counter() + seconds
    while (steps is None and (time.perf_counter() < t_end or not times)) or (steps is not None and len(times) < steps):
        t0 = time.perf_counter()
        one()
        times.append(time.perf_counter() - t0)
    gbs = per * len(times) / sum(times) / 1e9
    return gbs, kind, cores, desc + f"; {len(times)} passes", times


def cpu_model() -> str:
    try:
        for line in open("/proc/cpuinfo"):
            if line.startswith("model name"):
                return line.split(":", 1)[1].strip()
    except OSError:
        pass
    return "unknown"


def _run_timed(cmd, env):
    """Run a reference runner; (achieved tok/s from its own stderr line, wall s)."""
    import re

    t0 = time.perf_counter()
    r = subprocess.run(cmd, capture_output=True, text=True, env=env, timeout=900)
    wall = time.perf_counter() - t0
    m = re.search(r"achieved tok/s: ([0-9.]+)", r.stderr)
    if r.returncode != 0 or not m:
        return None, wall, (r.stderr or r.stdout)[-300:]
    return float(m.group(1)), wall, None


def cpu_decode_baselines(with_7b: bool):
    """The reference's CPU runners end to end, on this host's cores, each with
    its own `achieved tok/s` line (v1-int8-vnni/runq.c:710-716,
    v0-fp32/run.c:776-779, which leave out the first token), built from the
    reference sources into oracle/_ref:
      * runq.c (INT8 GS32, AVX-512 VNNI + OpenMP) on the config-1 checkpoint,
        greedy from BOS, 256 steps;
      * run.c (fp32 + OpenMP) on the same model's fp32 export;
      * runq.c on a Llama-2-7B-shape INT8 GS32 file (7.96 GB, written here
        with seeded weights), 32 steps — with_7b only, when host memory allows.
    Seeded synthetic models (no public checkpoint is involved)."""
    import tempfile

    ref_dir = os.path.join(ROOT, "oracle", "_ref")
    runq, run32 = os.path.join(ref_dir, "runq"), os.path.join(ref_dir, "run_fp32")
    cores = os.cpu_count() or 1
    out = {"cores": cores, "cpu": cpu_model(), "threads": "OMP_NUM_THREADS=%d" % cores,
           "kind": "reference", "timing": "each runner's own achieved tok/s line (first token excluded)"}
    if not (os.access(runq, os.X_OK) and os.access(run32, os.X_OK)):
        out["unavailable"] = "oracle/_ref runners not built (reference sources absent at build time)"
        return out
    if not cpu_has_vnni():
        out["unavailable"] = "host CPU lacks AVX-512 VNNI, which runq.c needs"
        return out
    sys.path.insert(0, os.path.join(ROOT, "tests"))
    import synth

    lq = importlib.import_module("llama2-min-inference_b200")
    env = dict(os.environ, OMP_NUM_THREADS=str(cores))
    with tempfile.TemporaryDirectory() as d:
        cfg = lq.Config.make(*synth.TINY_CONFIG)
        f32, q8, tok = os.path.join(d, "c1_f32.bin"), os.path.join(d, "c1_q8.bin"), os.path.join(d, "tok.bin")
        lq.write_checkpoint_fp32(f32, cfg, synth.TINY_SEED, 0.02, False)
        lq.quantize_checkpoint(f32, q8, lq.KIND_INT8, 32)
        synth.write_tokenizer(tok, cfg.vocab_size)
        for name, cmd in (("runq_config1_int8_gs32", [runq, q8]), ("run_fp32_config1", [run32, f32])):
            v, wall, err = _run_timed(cmd + ["-z", tok, "-t", "0", "-n", "256", "-s", "1"], env)
            out[name] = {"tok_s": v, "wall_s": round(wall, 3), "steps": 256} if v else {"error": err}
        if with_7b:
            try:
                mem = os.sysconf("SC_PAGE_SIZE") * os.sysconf("SC_AVPHYS_PAGES")
            except (ValueError, OSError):
                mem = 0
            c7 = lq.Config.make(4096, 11008, 32, 32, 32, 32000, 2048)
            if mem < 24 * 2**30:
                out["runq_7b_int8_gs32"] = {"unavailable": "less than 24 GB of free host memory"}
            else:
                p7 = os.path.join(d, "7b_q8.bin")
                t0 = time.perf_counter()
                lq.write_checkpoint_random(p7, c7, lq.KIND_INT8, 32, 7, 0.02)
                gen = time.perf_counter() - t0
                lq_tok = os.path.join(d, "tok7.bin")
                synth.write_tokenizer(lq_tok, 32000)
                v, wall, err = _run_timed([runq, p7, "-z", lq_tok, "-t", "0", "-n", "32", "-s", "1"], env)
                out["runq_7b_int8_gs32"] = ({"tok_s": v, "wall_s": round(wall, 2), "steps": 32,
                                             "file_bytes": os.path.getsize(p7), "file_write_s": round(gen, 1)}
                                            if v else {"error": err})
    return out


# ---------------------------------------------------------------------------

def setup_dist(n_gpus: int):
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    dist = None
    if world > 1:
        import datetime

        import torch.distributed as dist

        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=600))
    return rank, world, local, dist


def run_reference(args):
    rank, world, local, dist = setup_dist(args.gpus)
    if rank != 0:
        if dist:
            dist.destroy_process_group()
        return
    gbs, kind, cores, desc, times = cpu_baseline(steps=args.steps, warmup=args.warmup)
    ms = 1e3 * sum(times) / len(times)
    try:
        decode = cpu_decode_baselines(with_7b=not args.no_decode)
    except Exception as e:  # reported, never hides the GEMV line
        decode = {"error": str(e)[:300]}
    line = {"metric": METRIC, "value": round(gbs, 3), "unit": "GB/s", "n_gpus": args.gpus, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(ms, 4), "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "u8/s8 (int32 group dot, fp32 scales)", "data": "synthetic",
            "impl": "reference",
            "config": {"workload": WORKLOAD, "group_size_reference": 32,
                       "note": "reference runq.c supports only group size 32 (QBLOCK, runq.c:26)"},
            "cpu_baseline": {"value": round(gbs, 3), "unit": "GB/s", "cores": cores, "kind": kind, "sample": desc,
                             "cpu": cpu_model()},
            "e2e": {"value": round(gbs, 3), "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
            "reference_decode_cpu": decode}
    print(json.dumps(line), flush=True)
    if dist:
        dist.destroy_process_group()


def step_breakdown(lq, t, tokens, pos):
    """One traced decode step (device clock stamps of every kernel, see
    transformer_trace): the step's device time and, per kernel kind, the
    launch count, the time on the step's critical path (end of the kernel
    minus end of the one before it, in launch order) and the time from its
    dependency release to its end; and the first 24 kernels one by one.
    Tracing is switched off again after."""
    import numpy as np

    t.trace(True)
    B = len(tokens)
    for _ in range(2):  # the first step captures the traced graph
        t.forward_batch_argmax(np.asarray(tokens, np.int32), np.full(B, pos, np.int32))
    kinds, st = t.trace_read()
    t.trace(False)
    valid = (st < np.uint64(1) << np.uint64(63)).all(1)
    out = {"kernels": int(len(kinds))}
    if not valid.any():
        return out
    st = st.astype(np.float64)
    t0 = st[valid, 0].min()
    t_end = st[valid, 2].max()
    out["step_us"] = round((t_end - t0) / 1e3, 2)
    by = {}
    prev_end = t0
    for i, k in enumerate(kinds):
        name = lq.TRACE_KINDS.get(int(k), str(k))
        d = by.setdefault(name, {"count": 0, "critical_us": 0.0, "busy_us": 0.0})
        d["count"] += 1
        if valid[i]:
            d["critical_us"] += max(0.0, st[i, 2] - prev_end) / 1e3
            d["busy_us"] += max(0.0, st[i, 2] - st[i, 1]) / 1e3
            prev_end = max(prev_end, st[i, 2])
    for d in by.values():
        d["critical_us"] = round(d["critical_us"], 2)
        d["busy_us"] = round(d["busy_us"], 2)
    out["by_kind"] = by
    # the first kernels one by one: [kind, first CTA start, first CTA past its
    # dependency wait, last CTA end], in us after the previous kernel's end
    first, prev = [], t0
    for i in range(min(24, len(kinds))):
        if not valid[i]:
            continue
        name = lq.TRACE_KINDS.get(int(kinds[i]), str(kinds[i]))
        first.append([name] + [round((st[i, j] - prev) / 1e3, 2) for j in range(3)])
        prev = max(prev, st[i, 2])
    out["first_kernels_us"] = first
    return out


def decode_bench(lq, torch, positions: int = 2048):
    """Config 3: Llama-2-7B-shape INT4 GS64 greedy decode from BOS over
    positions 0..positions-1, random-init weights generated on the device."""
    cfg = lq.Config.make(4096, 11008, 32, 32, 32, 32000, 2048)
    t0 = time.perf_counter()
    t = lq.Transformer.random(cfg, lq.KIND_INT4, 64, 7, positions)
    init_s = time.perf_counter() - t0
    token = 1
    for pos in range(3):  # warm-up (graph capture) at the first positions
        token = t.forward_argmax(token, pos)
    token = 1
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    for pos in range(positions):
        token = t.forward_argmax(token, pos)
    dt = time.perf_counter() - t0
    breakdown = step_breakdown(lq, t, [token], positions - 1)
    t.close()
    wbytes = (4096 * 4096 * 4 + 4096 * 11008 * 3) * 32 + 32000 * 4096
    wbytes = wbytes // 2 + wbytes // 64 * 4
    kv_avg = 2 * 32 * 4096 * 4 * (positions + 1) / 2
    return {"config": "config3: llama-2-7b shape, int4 gs64, fp32 KV, greedy from BOS, batch 1",
            "positions": positions, "tok_s": round(positions / dt, 2), "ms_per_token": round(1e3 * dt / positions, 4),
            "weight_bytes_per_token": wbytes, "avg_kv_bytes_per_token": int(kv_avg),
            "hbm_gbs_effective": round((wbytes + kv_avg) * positions / dt / 1e9, 1),
            "roofline_frac": round((wbytes + kv_avg) * positions / dt / 1e9 / peaks()[0], 4),
            "roofline": "(weight + average KV bytes per token) x tok/s / measured HBM peak",
            "timing": "host wall clock around forward_argmax calls (H2D token/pos, graph, D2H 4 bytes each)",
            "init_s": round(init_s, 2),
            "step_breakdown_last_position": breakdown}


def batch_bench(lq, torch, batches=(1, 8, 16, 32, 64), ctx: int = 1024, steps: int = 8):
    """Config 4: Llama-2-13B-shape batched decode, INT8 and INT4 GS64, B
    independent sequences at context length ctx.  From 16 sequences on the
    products run on the tensor cores (tcgen05 kind::i8); the dp4a GEMV is
    also timed at 16 and 64 sequences for the crossover.  The KV cache
    positions 0..ctx-1 are zero-filled instead of decoded (attention reads
    every cached position whatever its value, so the step's work is that of
    a real step at that context); every timed step is a full
    forward_batch_argmax call."""
    D, H, L, V = 5120, 13824, 40, 32000
    cfg = lq.Config.make(D, H, L, 40, 40, V, 4096)
    nmat = L * (4 * D * D + 3 * D * H) + V * D
    out = {"config": "config4: llama-2-13b shape, gs64, fp32 KV at context %d" % ctx,
           "timing": "host wall clock around %d forward_batch_argmax calls per batch size" % steps,
           "kv_note": "cache positions below the context are zero-filled, not decoded", "runs": []}
    plans = [(8, None, batches), (4, None, batches), (8, "1000", (16, 64)), (4, "1000", (16, 64))]
    for kind, mma_env, bs in plans:
        old = os.environ.get("LQ_MMA_MIN_ROWS")
        if mma_env is not None:
            os.environ["LQ_MMA_MIN_ROWS"] = mma_env
        try:
            t = lq.Transformer.random(cfg, kind, 64, 11, ctx + steps + 8)
        finally:
            if mma_env is not None:
                if old is None:
                    os.environ.pop("LQ_MMA_MIN_ROWS", None)
                else:
                    os.environ["LQ_MMA_MIN_ROWS"] = old
        t.reserve_batch(max(bs))
        wbytes = nmat * (1 if kind == 8 else 0.5) + nmat // 64 * 4
        for B in bs:
            tok = np.ones(B, np.int32)
            for w in range(3):
                tok = t.forward_batch_argmax(tok, np.full(B, ctx - 3 + w, np.int32))
            torch.cuda.synchronize()
            t0 = time.perf_counter()
            for s_ in range(steps):
                tok = t.forward_batch_argmax(tok, np.full(B, ctx + s_, np.int32))
            dt = (time.perf_counter() - t0) / steps
            kv = B * 2 * L * D * 4 * (ctx + steps / 2)
            gbs = (wbytes + kv) / dt / 1e9
            path = "tcgen05 kind::i8" if (B >= 16 and mma_env is None) else "dp4a GEMV"
            out["runs"].append({"weight_kind": "int%d" % kind, "batch": B, "path": path, "tok_s": round(B / dt, 1),
                                "ms_per_step": round(1e3 * dt, 3), "weight_bytes": int(wbytes),
                                "kv_bytes_per_step": int(kv), "hbm_gbs_effective": round(gbs, 1),
                                "roofline_frac": round(gbs / peaks()[0], 4)})
        t.close()
    return out


def _group_id(lq, torch, rank, world, dist):
    if world == 1:
        return None
    buf = torch.zeros(128, dtype=torch.uint8, device="cuda")
    if rank == 0:
        buf.copy_(torch.frombuffer(bytearray(lq.tp_unique_id()), dtype=torch.uint8))
    dist.broadcast(buf, 0)
    return bytes(buf.cpu().numpy().tobytes())


def tp_check(lq, torch, rank, world, dist, layers: int = 2, tokens=(1, 3000, 17, 9)):
    """Correctness of the tensor-parallel step inside the benchmark run: the
    70B layer shape with `layers` layers, 4 teacher-forced positions, on every
    process with the peer all-reduce and with NCCL; rank 0 also runs the
    unsplit model on its GPU.  Reports whether every process returned the
    same logits, whether the peer and NCCL all-reduces agree bit for bit
    (they must with 2 processes, where both sums are y_0 + y_1; with more,
    NCCL may associate the sum differently) and the largest relative logits
    difference against the one-GPU model (the split only re-associates the
    wo / w2 sums, so the difference is fp32 rounding until an int8
    activation flips)."""
    cfg = lq.Config.make(8192, 28672, layers, 64, 8, 32000, 64)
    outs = {}
    for mode in ("peer", "nccl"):
        if mode == "nccl" and world == 1:
            break
        gid = _group_id(lq, torch, rank, world, dist)
        if mode == "nccl":
            os.environ["LQ_TP_ALLREDUCE"] = "nccl"
        try:
            t = lq.Transformer.random_tp(cfg, lq.KIND_INT4, 64, 29, rank, world, gid, 64)
        finally:
            os.environ.pop("LQ_TP_ALLREDUCE", None)
        outs[mode] = np.stack([t.forward(tok, pos).copy() for pos, tok in enumerate(tokens)])
        t.close()
    res = {"layers": layers, "positions": len(tokens)}
    mine = torch.from_numpy(outs["peer"]).cuda()
    if dist:
        allp = [torch.empty_like(mine) for _ in range(world)]
        dist.all_gather(allp, mine)
        res["all_ranks_identical"] = all(bool(torch.equal(allp[0], x)) for x in allp)
    else:
        res["all_ranks_identical"] = True
    if "nccl" in outs:
        a, b = outs["peer"], outs["nccl"]
        eq = torch.tensor([int(np.array_equal(a.view(np.uint32), b.view(np.uint32)))], device="cuda")
        if dist:
            dist.all_reduce(eq, op=dist.ReduceOp.MIN)
        res["peer_equals_nccl"] = bool(eq.item())
        res["peer_vs_nccl_max_rel"] = float(np.abs(a - b).max() / np.abs(b).max())
    if rank == 0:
        ref = lq.Transformer.random(cfg, lq.KIND_INT4, 64, 29, 64)
        want = np.stack([ref.forward(tok, pos).copy() for pos, tok in enumerate(tokens)])
        ref.close()
        a = outs["peer"]
        res["max_rel_vs_1gpu"] = float(np.abs(a - want).max() / np.abs(want).max())
        res["argmax_agree_vs_1gpu"] = float(np.mean(np.argmax(a, -1) == np.argmax(want, -1)))
        res["bitwise_equal_1gpu"] = bool(np.array_equal(a.view(np.uint32), want.view(np.uint32)))
    if dist:
        dist.barrier()
    return res


def tp_bench(lq, torch, rank, world, dist, ctx: int = 2048, steps1: int = 16, steps16: int = 8):
    """Config 5: Llama-2-70B-shape INT4 GS64 decode, tensor-parallel over the
    job's GPUs (one process per GPU), batch 1 and batch 16 at context ctx
    (cache positions below ctx zero-filled, not decoded).  The wo / w2
    partials are all-reduced by the quantizer that follows them, over peer
    memory (NVLink); with more than one GPU the NCCL all-reduce
    (LQ_TP_ALLREDUCE=nccl) is timed too, as the baseline.  Every process runs
    the same steps; the time is the slowest process's wall clock around the
    timed steps.  With more than one GPU, rank 0 first times the same model on
    its GPU alone, for the speed-up and efficiency of the split."""
    D, H, L, V = 8192, 28672, 80, 32000
    cfg = lq.Config.make(D, H, L, 64, 8, V, 4096)
    nmat = L * (2 * D * D + 2 * D * 1024 + 3 * D * H)
    peak, _ = peaks()

    def measure(allreduce, size, trace=False):
        wbytes = (nmat * 0.5 + nmat // 64 * 4) / size + V * D * (0.5 + 4 / 64)
        grp = dist if size > 1 else None
        gid = _group_id(lq, torch, rank if size > 1 else 0, size, grp)
        if allreduce:
            os.environ["LQ_TP_ALLREDUCE"] = allreduce
        t0 = time.perf_counter()
        try:
            t = lq.Transformer.random_tp(cfg, lq.KIND_INT4, 64, 23, rank if size > 1 else 0, size, gid,
                                         ctx + steps1 + 16)
        finally:
            os.environ.pop("LQ_TP_ALLREDUCE", None)
        init_s = time.perf_counter() - t0
        runs, breakdown = [], None
        for B in (1, 16):
            steps = steps1 if B == 1 else steps16
            if B > 1:
                t.reserve_batch(B)
            tok = np.ones(B, np.int32)
            for w in range(3):
                tok = t.forward_batch_argmax(tok, np.full(B, ctx - 3 + w, np.int32))
            if grp:
                grp.barrier()
            torch.cuda.synchronize()
            t1 = time.perf_counter()
            for s_ in range(steps):
                tok = t.forward_batch_argmax(tok, np.full(B, ctx + s_, np.int32))
            dt = (time.perf_counter() - t1) / steps
            if grp:
                m = torch.tensor([dt], device="cuda")
                grp.all_reduce(m, op=grp.ReduceOp.MAX)
                dt = float(m.item())
            kv = B * 2 * L * (1024 / size) * 4 * (ctx + steps / 2)
            gbs = (wbytes + kv) / dt / 1e9
            runs.append({"batch": B, "tok_s": round(B / dt, 1), "ms_per_step": round(1e3 * dt, 3),
                         "weight_bytes_per_gpu": int(wbytes), "kv_bytes_per_gpu_per_step": int(kv),
                         "hbm_gbs_per_gpu": round(gbs, 1), "roofline_frac": round(gbs / peak, 4),
                         "path": "tcgen05 kind::i8" if B >= 16 else "dp4a GEMV"})
            if trace and B == 1:
                breakdown = step_breakdown(lq, t, [int(tok[0])], ctx + steps)
        t.close()
        return runs, init_s, breakdown

    out = {"config": "config5: llama-2-70b shape, int4 gs64, tensor parallel x%d, context %d" % (world, ctx),
           "split": "wq/wk/wv/w1/w3 rows, wo/w2 columns; the wo / w2 partials are summed over the processes "
                    "by the next quantizer, reading the peers' partials over NVLink (in the decode graph)",
           "timing": "max over processes of the wall clock around the timed forward_batch_argmax calls",
           "kv_note": "cache positions below the context are zero-filled, not decoded",
           "roofline": "roofline_frac = (this GPU's weight + KV bytes per step / step time) / measured HBM peak"}
    if world > 1:
        one = None
        if rank == 0:
            one, _, _ = measure(None, 1)
        if dist:
            dist.barrier()
        if rank == 0:
            out["one_gpu_runs"] = [{"batch": r["batch"], "tok_s": r["tok_s"], "ms_per_step": r["ms_per_step"]}
                                   for r in one]
    runs, init_s, breakdown = measure(None, world, trace=True)
    out["init_s"] = round(init_s, 1)
    out["runs"] = runs
    out["step_breakdown_batch1_rank%d" % rank] = breakdown
    if world > 1 and rank == 0:
        out["speedup_vs_1gpu"] = {str(r["batch"]): round(r["tok_s"] / o["tok_s"], 3)
                                  for r, o in zip(runs, out["one_gpu_runs"])}
        out["efficiency"] = {k: round(v / world, 3) for k, v in out["speedup_vs_1gpu"].items()}
    if world > 1:
        nccl_runs, _, _ = measure("nccl", world)
        out["nccl_allreduce_runs"] = [{"batch": r["batch"], "tok_s": r["tok_s"], "ms_per_step": r["ms_per_step"]}
                                      for r in nccl_runs]
    try:
        out["tp_check"] = tp_check(lq, torch, rank, world, dist)
    except Exception as e:
        out["tp_check"] = {"error": str(e)[:300]}
    return out


PROBE_SHAPES = {  # dim, hidden, heads, kv heads of the Llama-2 layer shapes
    "13b": (5120, 13824, 40, 40),
    "70b": (8192, 28672, 64, 8),
    "7b": (4096, 11008, 32, 32),
}


def probe(spec: str):
    """One small decode case for profilers: "LAYERS:BATCH:KIND:CTX[:SHAPE]"
    on a Llama-2 layer shape (13b by default, or 70b / 7b); 3 warm steps, 1
    timed step, printed in ms."""
    import torch

    f = spec.split(":")
    L, B, kind, ctx = (int(v) for v in f[:4])
    D, H, NH, NKV = PROBE_SHAPES[f[4] if len(f) > 4 else "13b"]
    lq = importlib.import_module("llama2-min-inference_b200")
    t = lq.Transformer.random(lq.Config.make(D, H, L, NH, NKV, 32000, 4096), kind, 64, 11, ctx + 16)
    t.reserve_batch(B)
    tok = np.ones(B, np.int32)
    for w in range(3):
        tok = t.forward_batch_argmax(tok, np.full(B, ctx - 3 + w, np.int32))
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    t.forward_batch_argmax(tok, np.full(B, ctx, np.int32))
    print(f"probe {spec}: {1e3 * (time.perf_counter() - t0):.3f} ms", flush=True)
    t.close()


def run_gpu(args):
    import torch

    rank, world, local, dist = setup_dist(args.gpus)
    torch.cuda.set_device(local)
    lq = importlib.import_module("llama2-min-inference_b200")
    lq.lib()
    stream = torch.cuda.Stream()
    lq.set_stream(stream.cuda_stream)

    keep = []
    weights = [[None] * len(SHAPES) for _ in range(COPIES)]
    with torch.cuda.stream(stream):
        for c in range(COPIES):
            for i, (n, d) in enumerate(SHAPES):
                q = torch.empty((d, n if KIND == 8 else n // 2), dtype=torch.uint8, device="cuda")
                s = torch.empty((d, n // GS), dtype=torch.float32, device="cuda")
                w = lq.QuantizedTensor(q=q.data_ptr(), s=s.data_ptr(), rows=d, cols=n, group_size=GS, kind=KIND)
                lq.synth_tensor(w, 1000 + rank, 100 * c + i, 0.02)
                weights[c][i] = w
                keep += [q, s]
        gen = torch.Generator(device="cuda").manual_seed(5)
        xs = [torch.randn(n, device="cuda", generator=gen) for n, d in SHAPES]
        ys = [torch.empty(d, device="cuda") for n, d in SHAPES]
    stream.synchronize()

    # one plain call first: the library allocates its scratch outside graph capture
    for i, (n, d) in enumerate(SHAPES):
        lq.matmul_f32(ys[i].data_ptr(), xs[i].data_ptr(), weights[0][i], n, d)
    stream.synchronize()
    lq.set_launch_flags(lq.LAUNCH_PDL)
    graphs = []
    for c in range(COPIES):
        lq.graph_begin()
        for i, (n, d) in enumerate(SHAPES):
            lq.matmul_f32(ys[i].data_ptr(), xs[i].data_ptr(), weights[c][i], n, d)
        graphs.append(lq.graph_end())
    lq.set_launch_flags(0)

    for s_ in range(args.warmup):
        lq.graph_launch(graphs[s_ % COPIES])
    stream.synchronize()
    lq.sync()

    clocks = ClockSampler(local) if rank == 0 else None
    if clocks:
        clocks.start()
    if dist:
        dist.barrier()
    torch.cuda.synchronize()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    ev0.record(stream)
    for s_ in range(args.steps):
        lq.graph_launch(graphs[s_ % COPIES])
    ev1.record(stream)
    ev1.synchronize()
    torch.cuda.synchronize()
    ms = ev0.elapsed_time(ev1)
    if dist:
        dist.barrier()
    clk = clocks.stop() if clocks else None
    lq.sync()
    if dist:
        t = torch.tensor([ms], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())

    sb = step_bytes()
    per_gpu_gbs = sb * args.steps / (ms / 1e3) / 1e9
    value = per_gpu_gbs * world

    # end to end through the public C ABI with pinned host buffers
    hx = [torch.randn(n).pin_memory() for n, d in SHAPES]
    hy = [torch.empty(d).pin_memory() for n, d in SHAPES]
    calls = [[(hy[i].data_ptr(), hx[i].data_ptr(), weights[c][i], n, d) for i, (n, d) in enumerate(SHAPES)]
             for c in range(COPIES)]
    e2e_steps = max(3, min(args.steps, 200))
    for s_ in range(3):
        for call in calls[s_ % COPIES]:
            lq.matmul_f32(*call)
    if dist:
        dist.barrier()
    t0 = time.perf_counter()
    for s_ in range(e2e_steps):
        for call in calls[s_ % COPIES]:
            lq.matmul_f32(*call)
    e2e_s = time.perf_counter() - t0
    if dist:
        t = torch.tensor([e2e_s], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        e2e_s = float(t.item())
    e2e_gbs = sb * e2e_steps / e2e_s / 1e9 * world

    for g in graphs:
        lq.graph_destroy(g)

    # per-shape device time: for each shape, a graph of back-to-back products
    # of that shape cycling through enough copies of the matrix that they
    # exceed 4x L2 (126 MB), so every product streams from HBM
    per_shape = {}
    if not args.no_per_shape:
        ps_keep = []
        with torch.cuda.stream(stream):
            for i, (n, d) in enumerate(SHAPES):
                key = f"{n}x{d}"
                if key in per_shape:
                    continue
                nb = gemv_bytes(n, d, GS, KIND)
                ncopy = max(4, -(-4 * 126 * 2**20 // nb))
                ws_ = []
                for c in range(ncopy):
                    q = torch.empty((d, n), dtype=torch.uint8, device="cuda")
                    sc = torch.empty((d, n // GS), dtype=torch.float32, device="cuda")
                    w = lq.QuantizedTensor(q=q.data_ptr(), s=sc.data_ptr(), rows=d, cols=n, group_size=GS, kind=KIND)
                    lq.synth_tensor(w, 2000 + rank, 10 * i + c, 0.02)
                    ws_.append(w)
                    ps_keep += [q, sc]
                reps = max(ncopy, 16)
                lq.set_launch_flags(lq.LAUNCH_PDL)
                lq.graph_begin()
                for r_ in range(reps):
                    lq.matmul_f32(ys[i].data_ptr(), xs[i].data_ptr(), ws_[r_ % ncopy], n, d)
                g = lq.graph_end()
                lq.set_launch_flags(0)
                for _ in range(3):
                    lq.graph_launch(g)
                e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                e0.record(stream)
                for _ in range(5):
                    lq.graph_launch(g)
                e1.record(stream)
                e1.synchronize()
                us = e0.elapsed_time(e1) * 1e3 / (5 * reps)
                lq.graph_destroy(g)
                per_shape[key] = {"us": round(us, 3), "bytes": nb, "gbs": round(nb / us / 1e3, 1),
                                  "copies": ncopy}
        del ps_keep
        stream.synchronize()

    extra = {}
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu:
        gbs, kind, cores, desc, _ = cpu_baseline(seconds=args.cpu_seconds)
        cpu = {"value": round(gbs, 3), "unit": "GB/s", "cores": cores, "kind": kind, "sample": desc,
               "cpu": cpu_model()}
        try:
            extra["reference_decode_cpu"] = cpu_decode_baselines(with_7b=False)
        except Exception as e:
            extra["reference_decode_cpu"] = {"error": str(e)[:300]}
    if rank == 0 and world == 1 and not args.no_decode:
        try:
            extra["decode"] = decode_bench(lq, torch, args.decode_positions)
        except Exception as e:  # reported, never hides the GEMV line
            extra["decode"] = {"error": str(e)[:300]}
    if not args.no_tp:
        # every process takes part (tensor parallel over the job's GPUs)
        try:
            extra["tp_decode"] = tp_bench(lq, torch, rank, world, dist)
        except Exception as e:
            extra["tp_decode"] = {"error": str(e)[:300]}
    if rank == 0 and world == 1 and not args.no_batch:
        try:
            extra["batched"] = batch_bench(lq, torch)
        except Exception as e:
            extra["batched"] = {"error": str(e)[:300]}

    if rank == 0:
        peak, peak_kind = peaks()
        for v in per_shape.values():
            v["frac"] = round(v["gbs"] / peak, 4)
        tr = traffic_per_launch()
        line = {
            "metric": METRIC, "value": round(value, 2), "unit": "GB/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(ms / args.steps, 5), "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "u8 x s8 -> int32 group dot, fp32 scales",
            "data": "synthetic",
            "config": {"workload": WORKLOAD, "group_size": GS, "weight_kind": "int8", "batch": 1,
                       "bytes_per_step": sb, "l2": f"{COPIES} weight copies ({COPIES * sb / 1e9:.2f} GB) alternate; "
                       "inputs larger than L2", "parallelism": f"replicas x{world}",
                       "launch": "CUDA graph per step: 8 x (activation quantizer + GEMV), programmatic dependent "
                                 "launch",
                       "per_shape_us": per_shape},
            "roofline": {"bound": "hbm", "achieved": round(per_gpu_gbs, 1), "peak": peak, "unit": "GB/s",
                         "frac": round(per_gpu_gbs / peak, 4), "peak_source": peak_kind,
                         "kernel": "lq::gemv_tma_kernel<8,1>",
                         "traffic": (tr or {}).get("dram_bytes_per_step_scaled"),
                         "traffic_source": ("copied from profiles/gemv_traffic.json (ncu dram__bytes_read.sum + "
                                            "dram__bytes_write.sum of the sweep's launches), not measured in this run")
                         if tr else None},
            "cpu_baseline": cpu,
            "e2e": {"value": round(e2e_gbs, 2), "unit": "GB/s", "steps": e2e_steps,
                    "h2d_bytes_per_step": sum(4 * n for n, d in SHAPES),
                    "d2h_bytes_per_step": sum(4 * d for n, d in SHAPES),
                    "path": "matmul_f32 C ABI, pinned host x and y, copies + sync inside each call"},
            "gpu_launches": args.steps * 2 * len(SHAPES),
            "clocks": clk,
        }
        line.update(extra)
        print(json.dumps(line), flush=True)
    if dist:
        dist.barrier()
        dist.destroy_process_group()


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=1000)
    ap.add_argument("--warmup", type=int, default=20)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--cpu-seconds", type=float, default=10.0)
    ap.add_argument("--decode-positions", type=int, default=2048)
    ap.add_argument("--no-cpu", action="store_true")
    ap.add_argument("--no-decode", action="store_true")
    ap.add_argument("--no-batch", action="store_true")
    ap.add_argument("--no-tp", action="store_true")
    ap.add_argument("--no-per-shape", action="store_true")
    ap.add_argument("--probe", default=None, help="LAYERS:BATCH:KIND:CTX[:13b|70b|7b]: one small decode step for profilers")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    if args.probe:
        probe(args.probe)
    elif args.impl == "reference":
        run_reference(args)
    else:
        run_gpu(args)


if __name__ == "__main__":
    main()
