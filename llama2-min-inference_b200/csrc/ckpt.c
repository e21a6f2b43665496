/*
 * Checkpoint files and the synthetic weight generator (host only).
 *
 * Formats (little-endian), as written by the reference's quantizers:
 *   fp32 llama2.c file: int32 cfg[7], then fp32 tensors in the order of
 *     tools/quantize_int8.py:81-96 (two freq_cis blocks of seq*head/2 floats
 *     before the optional classifier).
 *   QLL8 v1 (tools/quantize_int8.py:11-37) and QLL4 v2
 *     (tools/quantize_int4.py:9-26): uint32 magic, uint32 version, int32
 *     cfg[7], then emb, rms_att, wq, wk, wv, wo, rms_ffn, w1, w2, w3,
 *     rms_final, [wcls]; each quantized tensor is all of its packed values
 *     followed by all of its fp32 group scales.  Group size 32 is implied.
 *   Version 3 (this library's extension, either magic): the same, with an
 *     int32 group size right after cfg.
 */
#include "lq_host.h"

#include <fcntl.h>
#include <math.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

/* ---- synthetic generator ------------------------------------------------
 * splitmix64 (S. Vigna's published finalizer) over a counter; a normal-like
 * value is the Irwin-Hall sum of twelve 24-bit uniforms, formed in exact
 * integer arithmetic and converted with one rounding, so the host and the
 * device produce identical fp32 values. */
static inline uint64_t mix64(uint64_t z) {
    z += 0x9E3779B97F4A7C15ull;
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}

float lq_synth_value(uint64_t seed, int tensor_id, uint64_t index, float std) {
    uint64_t base = mix64(seed) + ((uint64_t)tensor_id << 48) + index * 6ull;
    int32_t s = 0;
    for (int j = 0; j < 6; j++) {
        uint64_t h = mix64(base + (uint64_t)j);
        s += (int32_t)(h & 0xFFFFFFu) + (int32_t)((h >> 32) & 0xFFFFFFu);
    }
    s -= 6 << 24;
    return (float)s * (std * 5.9604644775390625e-8f);
}

/* ---- shapes ------------------------------------------------------------- */

int lq_tensor_table(const Config* c, LqTensorDesc out[LQ_NT]) {
    if (c->dim <= 0 || c->hidden_dim <= 0 || c->n_layers <= 0 || c->n_heads <= 0 ||
        c->n_kv_heads <= 0 || c->vocab_size <= 0 || c->seq_len <= 0)
        return LQ_EINVAL;
    if (c->dim % c->n_heads != 0 || c->n_heads % c->n_kv_heads != 0) return LQ_EINVAL;
    int64_t L = c->n_layers, D = c->dim, H = c->hidden_dim, V = c->vocab_size;
    int64_t KV = (int64_t)c->dim * c->n_kv_heads / c->n_heads;
    LqTensorDesc t[LQ_NT] = {
        {LQ_T_EMB, V, D, 0},     {LQ_T_RMS_ATT, L, D, 0}, {LQ_T_WQ, L * D, D, 1},
        {LQ_T_WK, L * KV, D, 1}, {LQ_T_WV, L * KV, D, 1}, {LQ_T_WO, L * D, D, 1},
        {LQ_T_RMS_FFN, L, D, 0}, {LQ_T_W1, L * H, D, 1},  {LQ_T_W2, L * D, H, 1},
        {LQ_T_W3, L * H, D, 1},  {LQ_T_RMS_FINAL, 1, D, 0}, {LQ_T_WCLS, V, D, 1},
    };
    memcpy(out, t, sizeof(t));
    return LQ_OK;
}

/* ---- fp32 writer -------------------------------------------------------- */

static int write_synth(FILE* f, uint64_t seed, int tid, int64_t n, float std, int ones) {
    enum { CH = 1 << 16 };
    static float buf[CH];
    for (int64_t i = 0; i < n; i += CH) {
        int64_t m = n - i < CH ? n - i : CH;
        for (int64_t j = 0; j < m; j++)
            buf[j] = ones ? 1.0f : lq_synth_value(seed, tid, (uint64_t)(i + j), std);
        if (fwrite(buf, 4, (size_t)m, f) != (size_t)m) return LQ_EIO;
    }
    return LQ_OK;
}

int lq_write_checkpoint_fp32(const char* path, const Config* cfg, uint64_t seed, float std,
                             int shared) {
    LqTensorDesc t[LQ_NT];
    if (!path || !cfg || lq_tensor_table(cfg, t) != LQ_OK)
        return lq_fail(LQ_EINVAL, "lq_write_checkpoint_fp32: bad config");
    FILE* f = fopen(path, "wb");
    if (!f) return lq_fail(LQ_EIO, "cannot open %s for writing", path);
    int32_t hdr[7] = {cfg->dim, cfg->hidden_dim, cfg->n_layers, cfg->n_heads,
                      cfg->n_kv_heads, shared ? cfg->vocab_size : -cfg->vocab_size, cfg->seq_len};
    int rc = fwrite(hdr, 4, 7, f) == 7 ? LQ_OK : LQ_EIO;
    for (int i = 0; i < LQ_NT && rc == LQ_OK; i++) {
        if (t[i].id == LQ_T_WCLS) {
            /* freq_cis_real / freq_cis_imag: unused by every reader; zeros */
            int64_t n = (int64_t)cfg->seq_len * (cfg->dim / cfg->n_heads);
            float z = 0.0f;
            for (int64_t j = 0; j < n && rc == LQ_OK; j++)
                if (fwrite(&z, 4, 1, f) != 1) rc = LQ_EIO;
            if (shared) break;
        }
        int ones = t[i].id == LQ_T_RMS_ATT || t[i].id == LQ_T_RMS_FFN || t[i].id == LQ_T_RMS_FINAL;
        rc = write_synth(f, seed, t[i].id, t[i].rows * t[i].cols, std, ones);
    }
    if (fclose(f) != 0 && rc == LQ_OK) rc = LQ_EIO;
    if (rc != LQ_OK) return lq_fail(rc, "write failed: %s", path);
    return LQ_OK;
}

/* ---- weight quantizers (tools/quantize_int8.py:52-63, quantize_int4.py:38-51)
 * float32 arithmetic throughout: scale = amax / 127 (or / 8), 0 -> 1e-8,
 * q = rint(w / scale) (half to even), clipped. */

void lq_quantize_rows_host(const float* w, int64_t rows, int64_t cols, int gs, int kind,
                           uint8_t* q, float* s) {
    int64_t ng = cols / gs;
    float qmax = kind == LQ_KIND_INT8 ? 127.0f : 8.0f;
    for (int64_t r = 0; r < rows; r++) {
        for (int64_t g = 0; g < ng; g++) {
            const float* wg = w + r * cols + g * gs;
            float amax = 0.0f;
            for (int j = 0; j < gs; j++) {
                float a = fabsf(wg[j]);
                if (a > amax) amax = a;
            }
            float sc = amax / qmax;
            if (sc == 0.0f) sc = 1e-8f;
            s[r * ng + g] = sc;
            if (kind == LQ_KIND_INT8) {
                for (int j = 0; j < gs; j++) {
                    float v = rintf(wg[j] / sc);
                    v = v > 127.0f ? 127.0f : (v < -127.0f ? -127.0f : v);
                    q[r * cols + g * gs + j] = (uint8_t)(int)(v + 128.0f);
                }
            } else {
                for (int j = 0; j < gs; j += 2) {
                    float a = rintf(wg[j] / sc), b = rintf(wg[j + 1] / sc);
                    a = a > 7.0f ? 7.0f : (a < -8.0f ? -8.0f : a);
                    b = b > 7.0f ? 7.0f : (b < -8.0f ? -8.0f : b);
                    q[r * (cols / 2) + (g * gs + j) / 2] =
                        (uint8_t)(((unsigned)(int)a & 0xFu) | (((unsigned)(int)b & 0xFu) << 4));
                }
            }
        }
    }
}

static int put_q(FILE* f, const float* w, int64_t rows, int64_t cols, int gs, int kind) {
    /* all packed values, then all scales (quantize_int8.py:102-107) */
    int64_t rb = kind == LQ_KIND_INT8 ? cols : cols / 2;
    int64_t blk = 64;
    uint8_t* q = (uint8_t*)malloc((size_t)(blk * rb));
    float* s = (float*)malloc((size_t)(rows * (cols / gs) * 4));
    if (!q || !s) { free(q); free(s); return LQ_ENOMEM; }
    int rc = LQ_OK;
    for (int64_t r = 0; r < rows && rc == LQ_OK; r += blk) {
        int64_t m = rows - r < blk ? rows - r : blk;
        lq_quantize_rows_host(w + r * cols, m, cols, gs, kind, q, s + r * (cols / gs));
        if (fwrite(q, 1, (size_t)(m * rb), f) != (size_t)(m * rb)) rc = LQ_EIO;
    }
    size_t ns = (size_t)(rows * (cols / gs));
    if (rc == LQ_OK && fwrite(s, 4, ns, f) != ns) rc = LQ_EIO;
    free(q);
    free(s);
    return rc;
}

int lq_quantize_checkpoint(const char* src, const char* dst, int kind, int gs) {
    if (kind != LQ_KIND_INT8 && kind != LQ_KIND_INT4)
        return lq_fail(LQ_EINVAL, "lq_quantize_checkpoint: kind must be INT8 or INT4");
    if (gs <= 0 || gs % 32 != 0 || gs > 256)
        return lq_fail(LQ_EINVAL, "group size must be a multiple of 32, at most 256");
    int fd = open(src, O_RDONLY);
    if (fd < 0) return lq_fail(LQ_EIO, "cannot open %s", src);
    struct stat st;
    fstat(fd, &st);
    if (st.st_size < 28) { close(fd); return lq_fail(LQ_EFORMAT, "%s: too short", src); }
    const uint8_t* base = (const uint8_t*)mmap(NULL, (size_t)st.st_size, PROT_READ, MAP_PRIVATE, fd, 0);
    close(fd);
    if (base == MAP_FAILED) return lq_fail(LQ_EIO, "mmap failed: %s", src);
    int32_t hdr[7];
    memcpy(hdr, base, 28);
    Config c = {hdr[0], hdr[1], hdr[2], hdr[3], hdr[4], abs(hdr[5]), hdr[6]};
    int shared = hdr[5] > 0;
    LqTensorDesc t[LQ_NT];
    int rc = lq_tensor_table(&c, t);
    if (rc == LQ_OK && (c.dim % gs || c.hidden_dim % gs)) rc = LQ_EINVAL;
    /* expected size */
    int64_t need = 28;
    for (int i = 0; i < LQ_NT && rc == LQ_OK; i++) {
        if (t[i].id == LQ_T_WCLS) {
            need += 4 * (int64_t)c.seq_len * (c.dim / c.n_heads);
            if (shared) break;
        }
        need += 4 * t[i].rows * t[i].cols;
    }
    if (rc == LQ_OK && need > st.st_size) rc = LQ_EFORMAT;
    FILE* f = NULL;
    if (rc == LQ_OK) {
        f = fopen(dst, "wb");
        if (!f) rc = LQ_EIO;
    }
    if (rc == LQ_OK) {
        uint32_t magic = kind == LQ_KIND_INT8 ? LQ_MAGIC_Q8 : LQ_MAGIC_Q4;
        uint32_t version = gs == 32 ? (kind == LQ_KIND_INT8 ? 1u : 2u) : 3u;
        int32_t g = gs;
        if (fwrite(&magic, 4, 1, f) != 1 || fwrite(&version, 4, 1, f) != 1 ||
            fwrite(hdr, 4, 7, f) != 7 || (version == 3 && fwrite(&g, 4, 1, f) != 1))
            rc = LQ_EIO;
    }
    const float* p = (const float*)(base + 28);
    for (int i = 0; i < LQ_NT && rc == LQ_OK; i++) {
        if (t[i].id == LQ_T_WCLS) {
            p += (int64_t)c.seq_len * (c.dim / c.n_heads);
            if (shared) break;
        }
        int64_t n = t[i].rows * t[i].cols;
        if (t[i].quantized) rc = put_q(f, p, t[i].rows, t[i].cols, gs, kind);
        else if (fwrite(p, 4, (size_t)n, f) != (size_t)n) rc = LQ_EIO;
        p += n;
    }
    if (f && fclose(f) != 0 && rc == LQ_OK) rc = LQ_EIO;
    munmap((void*)base, (size_t)st.st_size);
    if (rc != LQ_OK) return lq_fail(rc, "lq_quantize_checkpoint(%s -> %s) failed", src, dst);
    return LQ_OK;
}

/* ---- seeded quantized writer ---------------------------------------------
 * The same bytes lq_write_checkpoint_fp32 followed by lq_quantize_checkpoint
 * would produce (same generator, same quantizer), written block by block
 * without the fp32 intermediate; rows are generated and quantized in
 * parallel (OpenMP). */

static int put_synth_q(FILE* f, uint64_t seed, int tid, int64_t rows, int64_t cols, int gs, int kind, float std) {
    const int64_t rb = kind == LQ_KIND_INT8 ? cols : cols / 2, ng = cols / gs;
    const int64_t blk = 256;
    float* w = (float*)malloc((size_t)(blk * cols) * 4);
    uint8_t* q = (uint8_t*)malloc((size_t)(blk * rb));
    float* s = (float*)malloc((size_t)(rows * ng) * 4);
    if (!w || !q || !s) {
        free(w);
        free(q);
        free(s);
        return LQ_ENOMEM;
    }
    int rc = LQ_OK;
    for (int64_t r0 = 0; r0 < rows && rc == LQ_OK; r0 += blk) {
        const int64_t m = rows - r0 < blk ? rows - r0 : blk;
#pragma omp parallel for schedule(static)
        for (int64_t r = 0; r < m; r++) {
            for (int64_t c = 0; c < cols; c++)
                w[r * cols + c] = lq_synth_value(seed, tid, (uint64_t)((r0 + r) * cols + c), std);
            lq_quantize_rows_host(w + r * cols, 1, cols, gs, kind, q + r * rb, s + (r0 + r) * ng);
        }
        if (fwrite(q, 1, (size_t)(m * rb), f) != (size_t)(m * rb)) rc = LQ_EIO;
    }
    if (rc == LQ_OK && fwrite(s, 4, (size_t)(rows * ng), f) != (size_t)(rows * ng)) rc = LQ_EIO;
    free(w);
    free(q);
    free(s);
    return rc;
}

static int put_synth_f32(FILE* f, uint64_t seed, int tid, int64_t n, float std, int ones) {
    const int64_t blk = (int64_t)1 << 20;
    float* buf = (float*)malloc((size_t)blk * 4);
    if (!buf) return LQ_ENOMEM;
    int rc = LQ_OK;
    for (int64_t i = 0; i < n && rc == LQ_OK; i += blk) {
        const int64_t m = n - i < blk ? n - i : blk;
#pragma omp parallel for schedule(static)
        for (int64_t j = 0; j < m; j++) buf[j] = ones ? 1.0f : lq_synth_value(seed, tid, (uint64_t)(i + j), std);
        if (fwrite(buf, 4, (size_t)m, f) != (size_t)m) rc = LQ_EIO;
    }
    free(buf);
    return rc;
}

int lq_write_checkpoint_random(const char* path, const Config* cfg, int kind, int gs, uint64_t seed, float std) {
    LqTensorDesc t[LQ_NT];
    if (!path || !cfg || lq_tensor_table(cfg, t) != LQ_OK)
        return lq_fail(LQ_EINVAL, "lq_write_checkpoint_random: bad config");
    if (kind != LQ_KIND_INT8 && kind != LQ_KIND_INT4)
        return lq_fail(LQ_EINVAL, "lq_write_checkpoint_random: kind must be INT8 or INT4");
    if (gs <= 0 || gs % 32 != 0 || gs > 256 || cfg->dim % gs || cfg->hidden_dim % gs)
        return lq_fail(LQ_EINVAL, "lq_write_checkpoint_random: group size %d", gs);
    FILE* f = fopen(path, "wb");
    if (!f) return lq_fail(LQ_EIO, "cannot open %s for writing", path);
    const uint32_t magic = kind == LQ_KIND_INT8 ? LQ_MAGIC_Q8 : LQ_MAGIC_Q4;
    const uint32_t version = gs == 32 ? (kind == LQ_KIND_INT8 ? 1u : 2u) : 3u;
    const int32_t hdr[7] = {cfg->dim, cfg->hidden_dim, cfg->n_layers, cfg->n_heads,
                            cfg->n_kv_heads, -cfg->vocab_size, cfg->seq_len};
    const int32_t g = gs;
    int rc = (fwrite(&magic, 4, 1, f) == 1 && fwrite(&version, 4, 1, f) == 1 && fwrite(hdr, 4, 7, f) == 7 &&
              (version != 3 || fwrite(&g, 4, 1, f) == 1))
                 ? LQ_OK
                 : LQ_EIO;
    for (int i = 0; i < LQ_NT && rc == LQ_OK; i++) {
        const int ones = t[i].id == LQ_T_RMS_ATT || t[i].id == LQ_T_RMS_FFN || t[i].id == LQ_T_RMS_FINAL;
        rc = t[i].quantized ? put_synth_q(f, seed, t[i].id, t[i].rows, t[i].cols, gs, kind, std)
                            : put_synth_f32(f, seed, t[i].id, t[i].rows * t[i].cols, std, ones);
    }
    if (fclose(f) != 0 && rc == LQ_OK) rc = LQ_EIO;
    if (rc != LQ_OK) return lq_fail(rc, "write failed: %s", path);
    return LQ_OK;
}

/* ---- reader ------------------------------------------------------------- */

int lq_parse_header(const uint8_t* p, size_t size, Config* cfg, int* kind, int* gs, int* shared,
                    size_t* header_bytes) {
    if (size < 36) return lq_fail(LQ_EFORMAT, "checkpoint too short");
    uint32_t magic, version;
    memcpy(&magic, p, 4);
    memcpy(&version, p + 4, 4);
    int k;
    if (magic == LQ_MAGIC_Q8 && (version == 1 || version == 3)) k = LQ_KIND_INT8;
    else if (magic == LQ_MAGIC_Q4 && (version == 2 || version == 3)) k = LQ_KIND_INT4;
    else return lq_fail(LQ_EFORMAT, "bad magic/version (got %08x v%u)", magic, version);
    int32_t h[7];
    memcpy(h, p + 8, 28);
    int g = 32;
    size_t hb = 36;
    if (version == 3) {
        if (size < 40) return lq_fail(LQ_EFORMAT, "checkpoint too short");
        memcpy(&g, p + 36, 4);
        hb = 40;
    }
    Config c = {h[0], h[1], h[2], h[3], h[4], abs(h[5]), h[6]};
    LqTensorDesc t[LQ_NT];
    if (lq_tensor_table(&c, t) != LQ_OK || g <= 0 || g % 32 || g > 256 || c.dim % g ||
        c.hidden_dim % g)
        return lq_fail(LQ_EFORMAT, "bad config in checkpoint header");
    if (cfg) *cfg = c;
    if (kind) *kind = k;
    if (gs) *gs = g;
    if (shared) *shared = h[5] > 0;
    if (header_bytes) *header_bytes = hb;
    return LQ_OK;
}

int lq_read_header(const char* path, Config* cfg, int* kind, int* gs, int* shared) {
    uint8_t buf[40];
    FILE* f = fopen(path, "rb");
    if (!f) return lq_fail(LQ_EIO, "cannot open %s", path);
    size_t n = fread(buf, 1, sizeof(buf), f);
    fclose(f);
    return lq_parse_header(buf, n, cfg, kind, gs, shared, NULL);
}

int64_t lq_qtensor_bytes(int64_t rows, int64_t cols, int gs, int kind) {
    int64_t rb = kind == LQ_KIND_INT8 ? cols : cols / 2;
    return rows * rb + rows * (cols / gs) * 4;
}
