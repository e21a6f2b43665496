"""numpy restatement of the decode step (runq.c:320-421) split by tensor
parallelism: process `rank` of `world` holds the output rows of wq, wk, wv,
w1, w3 of its heads / hidden rows and the matching input columns of wo and
w2; the wo and w2 products are partial sums completed by `allreduce`.

TEST INFRASTRUCTURE ONLY: the quantized products use the oracle
(oracle.gemv, oracle.quantize_act); everything else is plain numpy fp32."""
from __future__ import annotations

import numpy as np

import oracle as O

ORDER = [("emb", 0), ("rms_att", 0), ("wq", 1), ("wk", 1), ("wv", 1), ("wo", 1), ("rms_ffn", 0), ("w1", 1),
         ("w2", 1), ("w3", 1), ("rms_final", 0), ("wcls", 1)]


def load(path: str):
    """Tensors of an unshared-classifier QLL8 / QLL4 checkpoint (versions 1-3)."""
    raw = open(path, "rb").read()
    magic, ver = (int(v) for v in np.frombuffer(raw[:8], np.uint32))
    dim, hid, L, nh, nkv, V, seq = (int(v) for v in np.frombuffer(raw[8:36], np.int32))
    kind = 8 if magic == 0x384C4C51 else 4
    gs, off = 32, 36
    if ver == 3:
        gs, off = int(np.frombuffer(raw[36:40], np.int32)[0]), 40
    assert V < 0, "shared classifier not supported here"
    V = -V
    kvd = dim * nkv // nh
    shapes = {"emb": (V, dim), "rms_att": (L, dim), "wq": (L * dim, dim), "wk": (L * kvd, dim),
              "wv": (L * kvd, dim), "wo": (L * dim, dim), "rms_ffn": (L, dim), "w1": (L * hid, dim),
              "w2": (L * dim, hid), "w3": (L * hid, dim), "rms_final": (1, dim), "wcls": (V, dim)}
    T = {}
    for name, quantized in ORDER:
        r, c = shapes[name]
        if quantized:
            rb = c if kind == 8 else c // 2
            q = np.frombuffer(raw, np.uint8, r * rb, off).reshape(r, rb)
            off += r * rb
            s = np.frombuffer(raw, np.float32, r * (c // gs), off).reshape(r, c // gs)
            off += r * (c // gs) * 4
            T[name] = (q, s)
        else:
            T[name] = np.frombuffer(raw, np.float32, r * c, off).reshape(r, c)
            off += r * c * 4
    cfg = dict(dim=dim, hidden=hid, layers=L, heads=nh, kv_heads=nkv, vocab=V, seq=seq, kind=kind, gs=gs)
    return cfg, T


def _rows(t, l, rows_per_layer, r0, nr):
    q, s = t
    a = l * rows_per_layer + r0
    return q[a:a + nr], s[a:a + nr]


def _cols(t, l, rows_per_layer, c0, nc, gs, kind):
    q, s = t
    a = l * rows_per_layer
    b0, nb = (c0, nc) if kind == 8 else (c0 // 2, nc // 2)
    return (np.ascontiguousarray(q[a:a + rows_per_layer, b0:b0 + nb]),
            np.ascontiguousarray(s[a:a + rows_per_layer, c0 // gs:(c0 + nc) // gs]))


def _rmsnorm(x, w):
    ss = np.float32(np.dot(x.astype(np.float32), x.astype(np.float32)) / np.float32(x.size) + np.float32(1e-5))
    return (w * (np.float32(1.0) / np.sqrt(ss)) * x).astype(np.float32)


class TPStep:
    def __init__(self, path: str, rank: int = 0, world: int = 1, allreduce=None, max_seq: int = 64):
        self.c, self.T = load(path)
        c = self.c
        self.rank, self.world = rank, world
        self.allreduce = allreduce or (lambda v: v)
        self.hs = c["dim"] // c["heads"]
        self.kv_mul = c["heads"] // c["kv_heads"]
        self.nh = c["heads"] // world
        self.nkv = c["kv_heads"] // world
        self.dq = self.nh * self.hs
        self.kvl = self.nkv * self.hs
        self.hid = c["hidden"] // world
        L, S = c["layers"], max_seq
        self.kc = np.zeros((L, S, self.kvl), np.float32)
        self.vc = np.zeros((L, S, self.kvl), np.float32)

    def _mv(self, x, w, n):
        c = self.c
        xq, xs, _ = O.quantize_act(x.astype(np.float32), c["gs"])
        return O.gemv(xq, xs, w[0], w[1], n, c["gs"], c["kind"])[0]

    def forward(self, token: int, pos: int) -> np.ndarray:
        c, T, r = self.c, self.T, self.rank
        D, gs, kind, hs = c["dim"], c["gs"], c["kind"], self.hs
        kvd = D * c["kv_heads"] // c["heads"]
        x = T["emb"][token].astype(np.float32).copy()
        for l in range(c["layers"]):
            xb = _rmsnorm(x, T["rms_att"][l])
            q = self._mv(xb, _rows(T["wq"], l, D, r * self.dq, self.dq), D)
            k = self._mv(xb, _rows(T["wk"], l, kvd, r * self.kvl, self.kvl), D)
            v = self._mv(xb, _rows(T["wv"], l, kvd, r * self.kvl, self.kvl), D)
            for vec in (q, k):  # RoPE (runq.c:351-365): the index within the head is the same locally
                for i in range(0, vec.size, 2):
                    hd = i % hs
                    freq = np.float32(1.0) / np.float32(10000.0) ** np.float32(hd / hs)
                    val = np.float32(pos) * freq
                    cr, ci = np.float32(np.cos(val)), np.float32(np.sin(val))
                    v0, v1 = vec[i], vec[i + 1]
                    vec[i], vec[i + 1] = v0 * cr - v1 * ci, v0 * ci + v1 * cr
            self.kc[l, pos], self.vc[l, pos] = k, v
            att = np.zeros(self.dq, np.float32)
            for h in range(self.nh):
                kh = h // self.kv_mul
                qh = q[h * hs:(h + 1) * hs]
                K = self.kc[l, :pos + 1, kh * hs:(kh + 1) * hs]
                V = self.vc[l, :pos + 1, kh * hs:(kh + 1) * hs]
                sc = (K @ qh) / np.float32(np.sqrt(hs))
                p = np.exp(sc - sc.max())
                att[h * hs:(h + 1) * hs] = (p / p.sum()) @ V
            part = self._mv(att, _cols(T["wo"], l, D, r * self.dq, self.dq, gs, kind), self.dq)
            x = (x + self.allreduce(part)).astype(np.float32)
            xb = _rmsnorm(x, T["rms_ffn"][l])
            h1 = self._mv(xb, _rows(T["w1"], l, c["hidden"], r * self.hid, self.hid), D)
            h3 = self._mv(xb, _rows(T["w3"], l, c["hidden"], r * self.hid, self.hid), D)
            hh = (h1 / (1.0 + np.exp(-h1)) * h3).astype(np.float32)
            part = self._mv(hh, _cols(T["w2"], l, D, r * self.hid, self.hid, gs, kind), self.hid)
            x = (x + self.allreduce(part)).astype(np.float32)
        xb = _rmsnorm(x, T["rms_final"][0])
        return self._mv(xb, T["wcls"], D)
