"""Checkpoint formats and the synthetic generator (CPU only)."""
import hashlib
import os
import struct

import numpy as np
import pytest

import oracle as O
import synth


def _sha(p):
    return hashlib.sha256(open(p, "rb").read()).hexdigest()


def test_quantized_checkpoint_is_byte_identical_to_reference_tools(golden):
    """The library's streaming quantizer writes the same bytes as the
    reference's tools/quantize_int8.py and quantize_int4.py (fixture hashes)."""
    g = golden("tiny_runq.npz")
    assert _sha(synth.tiny_checkpoint(8, 32)) == str(g["sha256_q8"])
    assert _sha(synth.tiny_checkpoint(4, 32)) == str(g["sha256_q4"])
    assert os.path.getsize(synth.tiny_checkpoint(8, 32)) == 53965476


def test_header_roundtrip(lq):
    for kind, gs, version, conf in [(8, 32, 1, synth.TINY_CONFIG), (4, 32, 2, synth.TINY_CONFIG),
                                    (8, 64, 3, synth.SMALL64_CONFIG), (4, 64, 3, synth.SMALL64_CONFIG)]:
        p = synth.tiny_checkpoint(kind, gs, config=conf)
        raw = open(p, "rb").read(12)
        magic, ver = struct.unpack("<II", raw[:8])
        assert magic == (0x384C4C51 if kind == 8 else 0x344C4C51)
        assert ver == version
        cfg, k, g, shared = lq.read_header(p)
        assert cfg.as_tuple() == conf and k == kind and g == gs and not shared


def test_gs64_file_matches_oracle_quantizer(lq):
    """Version-3 (GS-carrying) file: every quantized tensor equals the oracle
    quantizer applied to the fp32 weights."""
    p = synth.tiny_checkpoint(4, 64, config=synth.SMALL64_CONFIG)
    data = open(p, "rb").read()
    dim, hid, L, nh, nkv, V, seq = synth.SMALL64_CONFIG
    off = 40 + V * dim * 4 + L * dim * 4
    # first tensor: wq [L*dim, dim]
    rows, cols, gs = L * dim, dim, 64
    q = np.frombuffer(data, np.uint8, rows * cols // 2, off).reshape(rows, cols // 2)
    s = np.frombuffer(data, np.float32, rows * cols // gs, off + rows * cols // 2).reshape(rows, cols // gs)
    w = np.array([lq.synth_value(synth.TINY_SEED, lq.T_WQ, i) for i in range(8 * cols)], np.float32).reshape(8, cols)
    oq, os_ = O.quantize_weight(w, gs, 4)
    assert np.array_equal(q[:8], oq) and np.array_equal(s[:8], os_)


def test_synth_values_are_deterministic_and_normal_like(lq):
    v = np.array([lq.synth_value(99, 3, i, 1.0) for i in range(20000)], np.float32)
    assert v.tolist()[:5] == [lq.synth_value(99, 3, i, 1.0) for i in range(5)]
    assert abs(v.mean()) < 0.03 and abs(v.std() - 1.0) < 0.03
    assert lq.synth_value(99, 3, 0, 1.0) != lq.synth_value(99, 4, 0, 1.0)


def test_bad_magic_and_version_rejected(lq, tmp_path):
    p = tmp_path / "bad.bin"
    p.write_bytes(struct.pack("<II7i", 0x12345678, 1, 288, 768, 6, 6, 6, -32000, 256))
    with pytest.raises(lq.LlamaQError) as e:
        lq.read_header(str(p))
    assert e.value.code == lq.EFORMAT
    p.write_bytes(struct.pack("<II7i", 0x384C4C51, 2, 288, 768, 6, 6, 6, -32000, 256))
    with pytest.raises(lq.LlamaQError) as e:
        lq.read_header(str(p))
    assert e.value.code == lq.EFORMAT


def test_truncated_checkpoint_rejected_before_any_gpu_work(lq, tmp_path):
    """The reference mmaps without a size check (runq.c:269-277); the
    library reports LQ_EFORMAT (checked before any CUDA call)."""
    src = synth.tiny_checkpoint(8, 32)
    p = tmp_path / "trunc.bin"
    p.write_bytes(open(src, "rb").read()[: 10_000_000])
    with pytest.raises(lq.LlamaQError) as e:
        lq.Transformer.from_file(str(p))
    assert e.value.code == lq.EFORMAT


def test_missing_file(lq):
    with pytest.raises(lq.LlamaQError) as e:
        lq.Transformer.from_file("/nonexistent/model.bin")
    assert e.value.code == lq.EIO


def test_tokenizer_format(tmp_path):
    p = tmp_path / "tok.bin"
    synth.write_tokenizer(str(p), 300)
    data = p.read_bytes()
    (maxlen,) = struct.unpack_from("<i", data, 0)
    off, n = 4, 0
    while off < len(data):
        sc, ln = struct.unpack_from("<fi", data, off)
        off += 8 + ln
        n += 1
    assert n == 300 and maxlen >= 6


@pytest.mark.parametrize("kind,gs", [(8, 32), (4, 32), (8, 64), (4, 128)])
def test_direct_random_writer_equals_fp32_then_quantize(lq, tmp_path, kind, gs):
    """lq_write_checkpoint_random writes the bytes of the fp32 export followed
    by the quantizer (the reference's tools/quantize_int8.py / quantize_int4.py
    pipeline), without the fp32 intermediate."""
    import synth

    cfg = lq.Config.make(*synth.SMALL64_CONFIG)
    f32, a, b = (str(tmp_path / n) for n in ("f.bin", "a.bin", "b.bin"))
    lq.write_checkpoint_fp32(f32, cfg, 11, 0.02, False)
    lq.quantize_checkpoint(f32, a, kind, gs)
    lq.write_checkpoint_random(b, cfg, kind, gs, 11, 0.02)
    assert open(a, "rb").read() == open(b, "rb").read()
