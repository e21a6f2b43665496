"""Seeded synthetic inputs shared by the tests, the fixture generator and
bench.py: the config-1 tiny model shape, a tokenizer.bin writer, and cached
tiny checkpoints written through the library's own generator/quantizer.

No public dataset is involved: the reference quotes no benchmark data, and
every input here is seeded synthetic data of the reference's shapes.
"""
from __future__ import annotations

import importlib
import os
import struct
import tempfile

import numpy as np

ROOT = os.path.abspath(os.path.join(os.path.dirname(__file__), ".."))

# config 1: dim 288, hidden 768, 6 layers, 6/6 heads, vocab 32000, seq 256
TINY_CONFIG = (288, 768, 6, 6, 6, 32000, 256)
TINY_SEED = 1234
# group-size-64 and GQA coverage at a small shape: dim 256, hidden 768,
# 4 layers, 4 query heads / 2 kv heads (head 64), vocab 4096, seq 128
SMALL64_CONFIG = (256, 768, 4, 4, 2, 4096, 128)
# head size 128 (the 7B / 13B / 70B head), multi-head: dim 256, 2 heads, 2
# layers, long context (seq 1280) for the split-KV merge over 18+ chunks
HEAD128_CONFIG = (256, 768, 2, 2, 2, 512, 1280)
# head size 128 with 8:1 grouped-query attention (the 70B layout, one kv head
# serving 8 query heads): dim 1024, 1 layer, seq 1280
GQA8_CONFIG = (1024, 1024, 1, 8, 1, 512, 1280)


def lq():
    return importlib.import_module("llama2-min-inference_b200")


def write_tokenizer(path: str, vocab: int, seed: int = 7) -> None:
    """tokenizer.bin in the reference's format (runq.c:444-465): int32
    max_token_length, then per token float32 score, int32 len, bytes.
    Tokens 0-2 are <unk>/BOS/EOS, 3-258 the <0xXX> byte tokens, 259 a single
    space, the rest seeded printable strings."""
    rng = np.random.default_rng(seed)
    toks = [b"<unk>", b"\n<s>\n", b"\n</s>\n"] + [b"<0x%02X>" % i for i in range(256)] + [b" "]
    seen = set(toks)
    while len(toks) < vocab:
        n = int(rng.integers(1, 7))
        s = bytes(int(c) for c in rng.integers(32, 127, size=n))
        if rng.random() < 0.3:
            s = b" " + s
        if s not in seen:
            seen.add(s)
            toks.append(s)
    scores = rng.standard_normal(vocab).astype(np.float32)
    with open(path, "wb") as f:
        f.write(struct.pack("<i", max(len(t) for t in toks)))
        for t, sc in zip(toks, scores):
            f.write(struct.pack("<fi", float(sc), len(t)))
            f.write(t)


_CACHE = os.path.join(tempfile.gettempdir(), "llama2q_test_ckpt")


def tiny_checkpoint(kind: int = 8, gs: int = 32, shared: bool = False, config=TINY_CONFIG,
                    seed: int = TINY_SEED) -> str:
    """Quantized checkpoint of the synthetic model (cached in /tmp)."""
    os.makedirs(_CACHE, exist_ok=True)
    tag = "_".join(str(v) for v in config) + f"_s{seed}_{'sh' if shared else 'un'}"
    f32 = os.path.join(_CACHE, f"f32_{tag}.bin")
    out = os.path.join(_CACHE, f"q{kind}_g{gs}_{tag}.bin")
    L = lq()
    if not os.path.exists(f32):
        L.write_checkpoint_fp32(f32 + ".tmp", L.Config.make(*config), seed, 0.02, shared)
        os.replace(f32 + ".tmp", f32)
    if not os.path.exists(out):
        L.quantize_checkpoint(f32, out + ".tmp", kind, gs)
        os.replace(out + ".tmp", out)
    return out


def tiny_tokenizer(vocab: int = TINY_CONFIG[5]) -> str:
    os.makedirs(_CACHE, exist_ok=True)
    p = os.path.join(_CACHE, f"tokenizer_{vocab}.bin")
    if not os.path.exists(p):
        write_tokenizer(p + ".tmp", vocab)
        os.replace(p + ".tmp", p)
    return p
