/*
 * Scalar CPU oracle for the group-quantized decode hot path.
 *
 * TEST INFRASTRUCTURE ONLY: loaded by tests/, __graft_entry__.smoke() and the
 * CPU-baseline leg of bench.py, never by the product library.
 *
 * Each function cites the reference lines it restates (paths relative to the
 * reference project root).  The group size is a parameter; at GS=32 the INT8
 * path is pinned against runq.c itself (tests/test_oracle_pin.py and the
 * fixtures in tests/golden/).
 */
#include "oracle.h"

#include <math.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

/* ------------------------------------------------------------------------ */
/* activation quantize: v1-int8-vnni/runq.c:117-139                         */

void orc_quantize_act(const float* x, int n, int gs, int8_t* xq, float* xs, float* xt) {
    int nb = n / gs;
    for (int b = 0; b < nb; b++) {
        const float* xb = x + (size_t)b * gs;
        float amax = 0.0f;
        for (int j = 0; j < gs; j++) {
            float a = fabsf(xb[j]);
            if (a > amax) amax = a;
        }
        float s = amax / 127.0f;
        if (s == 0.0f) s = 1e-8f;
        int sum = 0;
        for (int j = 0; j < gs; j++) {
            int q = (int)lrintf(xb[j] / s);
            if (q > 127) q = 127;
            if (q < -127) q = -127;
            xq[(size_t)b * gs + j] = (int8_t)q;
            sum += q;
        }
        xs[b] = s;
        if (xt) xt[b] = s * 128.0f * (float)sum;
    }
}

/* ------------------------------------------------------------------------ */
/* weight quantizers: tools/quantize_int8.py:52-63, tools/quantize_int4.py:38-51
 * numpy float32 arithmetic: amax / 127.0 stays float32 (NEP 50), the division
 * w / scale is float32, np.rint rounds half to even (rintf in the default
 * rounding mode).                                                           */

static float group_scale(const float* w, int gs, float qmax) {
    float amax = 0.0f;
    for (int j = 0; j < gs; j++) {
        float a = fabsf(w[j]);
        if (a > amax) amax = a;
    }
    float s = amax / qmax;
    if (s == 0.0f) s = 1e-8f;
    return s;
}

void orc_quantize_w8(const float* w, int64_t rows, int64_t cols, int gs, uint8_t* q, float* s) {
    int64_t ng = cols / gs;
    for (int64_t r = 0; r < rows; r++) {
        for (int64_t g = 0; g < ng; g++) {
            const float* wg = w + r * cols + g * gs;
            float sc = group_scale(wg, gs, 127.0f);
            s[r * ng + g] = sc;
            for (int j = 0; j < gs; j++) {
                float v = rintf(wg[j] / sc);
                if (v > 127.0f) v = 127.0f;
                if (v < -127.0f) v = -127.0f;
                q[r * cols + g * gs + j] = (uint8_t)(int)(v + 128.0f);
            }
        }
    }
}

void orc_quantize_w4(const float* w, int64_t rows, int64_t cols, int gs, uint8_t* q, float* s) {
    int64_t ng = cols / gs;
    for (int64_t r = 0; r < rows; r++) {
        for (int64_t g = 0; g < ng; g++) {
            const float* wg = w + r * cols + g * gs;
            float sc = group_scale(wg, gs, 8.0f);
            s[r * ng + g] = sc;
            for (int j = 0; j < gs; j += 2) {
                float v0 = rintf(wg[j] / sc), v1 = rintf(wg[j + 1] / sc);
                if (v0 > 7.0f) v0 = 7.0f;
                if (v0 < -8.0f) v0 = -8.0f;
                if (v1 > 7.0f) v1 = 7.0f;
                if (v1 < -8.0f) v1 = -8.0f;
                unsigned lo = (unsigned)((int)v0 & 0xF), hi = (unsigned)((int)v1 & 0xF);
                q[r * (cols / 2) + (g * gs + j) / 2] = (uint8_t)(lo | (hi << 4));
            }
        }
    }
}

/* ------------------------------------------------------------------------ */
/* integer group dots                                                        */

/* weight element k of a row, as a signed integer */
static inline int wval(const uint8_t* row, int64_t k, int kind) {
    if (kind == 8) return (int)row[k] - 128;                 /* quantize_int8.py:62 bias */
    unsigned byte = row[k >> 1];                             /* quantize_int4.py:47-50  */
    unsigned nib = (k & 1) ? (byte >> 4) : (byte & 0xF);
    return ((int)(nib ^ 8u)) - 8;                            /* v5 run.cu:253 sign extend */
}

static inline size_t row_bytes(int64_t cols, int kind) {
    return kind == 8 ? (size_t)cols : (size_t)cols / 2;
}

void orc_group_dots(int32_t* D, const uint8_t* wq, const int8_t* xq,
                    int64_t rows, int64_t cols, int gs, int kind) {
    int64_t ng = cols / gs;
    size_t rb = row_bytes(cols, kind);
    for (int64_t r = 0; r < rows; r++) {
        const uint8_t* row = wq + (size_t)r * rb;
        for (int64_t g = 0; g < ng; g++) {
            int32_t d = 0;
            for (int j = 0; j < gs; j++) {
                int64_t k = g * gs + j;
                d += wval(row, k, kind) * (int32_t)xq[k];
            }
            D[r * ng + g] = d;
        }
    }
}

void orc_gemv(float* out, const int8_t* xq, const float* xs, const uint8_t* wq,
              const float* ws, int64_t rows, int64_t cols, int gs, int kind) {
    int64_t ng = cols / gs;
    size_t rb = row_bytes(cols, kind);
    for (int64_t r = 0; r < rows; r++) {
        const uint8_t* row = wq + (size_t)r * rb;
        float acc = 0.0f;
        for (int64_t g = 0; g < ng; g++) {
            int32_t d = 0;
            for (int j = 0; j < gs; j++) {
                int64_t k = g * gs + j;
                d += wval(row, k, kind) * (int32_t)xq[k];
            }
            acc += (ws[r * ng + g] * xs[g]) * (float)d;
        }
        out[r] = acc;
    }
}

void orc_gemm(float* out, const int8_t* xq, const float* xs, const uint8_t* wq,
              const float* ws, int B, int64_t rows, int64_t cols, int gs, int kind) {
    int64_t ng = cols / gs;
    for (int b = 0; b < B; b++)
        orc_gemv(out + (size_t)b * rows, xq + (size_t)b * cols, xs + (size_t)b * ng,
                 wq, ws, rows, cols, gs, kind);
}

/* ------------------------------------------------------------------------ */
/* model: checkpoint reader (runq.c:230-278, v5 run.cu:534-551, plus the     */
/* GS-carrying version-3 header of the product library) and forward        */

typedef struct {
    uint8_t* q;
    float* s;
    int64_t rows, cols;
} OrcQ;

struct OrcModel {
    OrcConfig c;
    int kind, gs;
    int mma_grid; /* > 0: GEMVs in the tensor-core GEMM's order for this grid size */
    int tp;       /* > 1: the tensor-parallel step over tp processes (wo / w2 as per-process column slices) */
    float *emb, *rms_att, *rms_ffn, *rms_final;
    OrcQ wq, wk, wv, wo, w1, w2, w3, wcls;
    uint8_t* file;      /* whole file in memory */
    uint8_t* own_wcls_q;
    float* own_wcls_s;
    /* run state */
    int max_seq;
    float *x, *xb, *xb2, *hb, *hb2, *q, *att, *logits, *kc, *vc;
    int8_t* aq;
    float* as;
    /* optional trace of every int8 activation the forwards compute, in order */
    int8_t* trace;
    long trace_cap, trace_n;
    /* optional override: the next forward uses these int8 activations and
     * group scales in place of its own, value by value in call order */
    const int8_t* ovr_q;
    const float* ovr_s;
    long ovr_cap, ovr_n;
};

static void act_trace(OrcModel* m, int n) {
    if (m->ovr_q && m->ovr_n + n <= m->ovr_cap) {
        memcpy(m->aq, m->ovr_q + m->ovr_n, (size_t)n);
        memcpy(m->as, m->ovr_s + m->ovr_n / m->gs, (size_t)(n / m->gs) * sizeof(float));
    }
    m->ovr_n += n;
    for (int i = 0; i < n; i++) {
        if (m->trace && m->trace_n < m->trace_cap) m->trace[m->trace_n] = m->aq[i];
        m->trace_n++;
    }
}

long orc_act_override(OrcModel* m, const int8_t* xq, const float* xs, long n) {
    long used = m->ovr_n;
    m->ovr_q = xq;
    m->ovr_s = xs;
    m->ovr_cap = n;
    m->ovr_n = 0;
    return used;
}

long orc_act_trace(OrcModel* m, int8_t* buf, long cap) {
    long n = m->trace_n;
    m->trace = buf;
    m->trace_cap = cap;
    m->trace_n = 0;
    return n;
}

static int take(uint8_t** p, uint8_t* end, size_t n, void** out) {
    if ((size_t)(end - *p) < n) return -1;
    *out = *p;
    *p += n;
    return 0;
}

static int take_q(uint8_t** p, uint8_t* end, OrcQ* w, int64_t rows, int64_t cols, int gs, int kind) {
    w->rows = rows;
    w->cols = cols;
    if (take(p, end, (size_t)rows * row_bytes(cols, kind), (void**)&w->q)) return -1;
    if (take(p, end, (size_t)rows * (cols / gs) * sizeof(float), (void**)&w->s)) return -1;
    return 0;
}

OrcModel* orc_model_load(const char* path, int max_seq) {
    FILE* f = fopen(path, "rb");
    if (!f) { fprintf(stderr, "oracle: cannot open %s\n", path); return NULL; }
    fseek(f, 0, SEEK_END);
    long size = ftell(f);
    fseek(f, 0, SEEK_SET);
    OrcModel* m = (OrcModel*)calloc(1, sizeof(OrcModel));
    m->file = (uint8_t*)malloc((size_t)size);
    if (fread(m->file, 1, (size_t)size, f) != (size_t)size) {
        fclose(f);
        orc_model_free(m);
        return NULL;
    }
    fclose(f);
    uint8_t* p = m->file;
    uint8_t* end = m->file + size;
    uint32_t magic, version;
    memcpy(&magic, p, 4);
    memcpy(&version, p + 4, 4);
    p += 8;
    if (magic == 0x384C4C51u && (version == 1 || version == 3)) m->kind = 8;
    else if (magic == 0x344C4C51u && (version == 2 || version == 3)) m->kind = 4;
    else { fprintf(stderr, "oracle: bad magic/version\n"); orc_model_free(m); return NULL; }
    int32_t cfg[7];
    memcpy(cfg, p, 28);
    p += 28;
    m->gs = 32;
    if (version == 3) { int32_t g; memcpy(&g, p, 4); p += 4; m->gs = g; }
    int shared = cfg[5] > 0;
    m->c.dim = cfg[0]; m->c.hidden_dim = cfg[1]; m->c.n_layers = cfg[2];
    m->c.n_heads = cfg[3]; m->c.n_kv_heads = cfg[4];
    m->c.vocab_size = abs(cfg[5]); m->c.seq_len = cfg[6];
    OrcConfig* c = &m->c;
    int kv_dim = c->dim * c->n_kv_heads / c->n_heads;
    int64_t L = c->n_layers;
    int gs = m->gs, k = m->kind;
    int bad = 0;
    bad |= take(&p, end, (size_t)c->vocab_size * c->dim * 4, (void**)&m->emb);
    bad |= take(&p, end, (size_t)L * c->dim * 4, (void**)&m->rms_att);
    bad |= take_q(&p, end, &m->wq, L * c->dim, c->dim, gs, k);
    bad |= take_q(&p, end, &m->wk, L * kv_dim, c->dim, gs, k);
    bad |= take_q(&p, end, &m->wv, L * kv_dim, c->dim, gs, k);
    bad |= take_q(&p, end, &m->wo, L * c->dim, c->dim, gs, k);
    bad |= take(&p, end, (size_t)L * c->dim * 4, (void**)&m->rms_ffn);
    bad |= take_q(&p, end, &m->w1, L * c->hidden_dim, c->dim, gs, k);
    bad |= take_q(&p, end, &m->w2, L * c->dim, c->hidden_dim, gs, k);
    bad |= take_q(&p, end, &m->w3, L * c->hidden_dim, c->dim, gs, k);
    bad |= take(&p, end, (size_t)c->dim * 4, (void**)&m->rms_final);
    if (!shared) {
        bad |= take_q(&p, end, &m->wcls, c->vocab_size, c->dim, gs, k);
    } else {
        /* shared classifier: quantize the fp32 embedding with the same
         * weight quantizer (extension; the reference exits here, runq.c:247) */
        int64_t V = c->vocab_size, D = c->dim;
        m->own_wcls_q = (uint8_t*)malloc((size_t)V * row_bytes(D, k));
        m->own_wcls_s = (float*)malloc((size_t)V * (D / gs) * 4);
        if (k == 8) orc_quantize_w8(m->emb, V, D, gs, m->own_wcls_q, m->own_wcls_s);
        else orc_quantize_w4(m->emb, V, D, gs, m->own_wcls_q, m->own_wcls_s);
        m->wcls.q = m->own_wcls_q; m->wcls.s = m->own_wcls_s;
        m->wcls.rows = V; m->wcls.cols = D;
    }
    if (bad) { fprintf(stderr, "oracle: truncated checkpoint\n"); orc_model_free(m); return NULL; }
    m->max_seq = (max_seq > 0 && max_seq < c->seq_len) ? max_seq : c->seq_len;
    int maxn = c->hidden_dim > c->dim ? c->hidden_dim : c->dim;
    m->x = (float*)calloc(c->dim, 4);
    m->xb = (float*)calloc(c->dim, 4);
    m->xb2 = (float*)calloc(c->dim, 4);
    m->hb = (float*)calloc(c->hidden_dim, 4);
    m->hb2 = (float*)calloc(c->hidden_dim, 4);
    m->q = (float*)calloc(c->dim, 4);
    m->att = (float*)calloc((size_t)c->n_heads * m->max_seq, 4);
    m->logits = (float*)calloc(c->vocab_size, 4);
    m->kc = (float*)calloc((size_t)L * m->max_seq * kv_dim, 4);
    m->vc = (float*)calloc((size_t)L * m->max_seq * kv_dim, 4);
    m->aq = (int8_t*)calloc(maxn, 1);
    m->as = (float*)calloc(maxn / gs + 1, 4);
    return m;
}

void orc_model_free(OrcModel* m) {
    if (!m) return;
    free(m->file); free(m->own_wcls_q); free(m->own_wcls_s);
    free(m->x); free(m->xb); free(m->xb2); free(m->hb); free(m->hb2); free(m->q);
    free(m->att); free(m->logits); free(m->kc); free(m->vc); free(m->aq); free(m->as);
    free(m);
}

void orc_model_info(const OrcModel* m, OrcConfig* cfg, int* kind, int* gs) {
    if (cfg) *cfg = m->c;
    if (kind) *kind = m->kind;
    if (gs) *gs = m->gs;
}

/* rmsnorm, runq.c:294-305.  The reference sums squares in 16 fp32 lanes with
 * fused multiply-add and reduces them with _mm512_reduce_add_ps; the same
 * lane order is kept here (tree: lanes i and i+8, then i and i+4, then pairs)
 * so that the oracle tracks runq.c closely. */
static void rmsnorm(float* o, const float* x, const float* w, int n) {
    float lane[16] = {0};
    int j = 0;
    for (; j + 16 <= n; j += 16)
        for (int i = 0; i < 16; i++) lane[i] = fmaf(x[j + i], x[j + i], lane[i]);
    float t8[8], t4[4];
    for (int i = 0; i < 8; i++) t8[i] = lane[i] + lane[i + 8];
    for (int i = 0; i < 4; i++) t4[i] = t8[i] + t8[i + 4];
    float s = (t4[0] + t4[2]) + (t4[1] + t4[3]);
    for (; j < n; j++) s += x[j] * x[j];
    s = 1.0f / sqrtf(s / n + 1e-5f);
    for (int i = 0; i < n; i++) o[i] = w[i] * (s * x[i]);
}

static void softmax(float* x, int n) {   /* runq.c:307-318 */
    float mx = x[0];
    for (int i = 1; i < n; i++) if (x[i] > mx) mx = x[i];
    float sum = 0.0f;
    for (int i = 0; i < n; i++) { x[i] = expf(x[i] - mx); sum += x[i]; }
    for (int i = 0; i < n; i++) x[i] /= sum;
}

static void qmatmul(OrcModel* m, float* out, const OrcQ* w, int64_t l, int64_t layer_rows, int n) {
    size_t rb = row_bytes(w->cols, m->kind);
    const uint8_t* q = w->q + (size_t)l * layer_rows * rb;
    const float* s = w->s + (size_t)l * layer_rows * (w->cols / m->gs);
    orc_gemv(out, m->aq, m->as, q, s, layer_rows, n, m->gs, m->kind);
}

float* orc_forward(OrcModel* m, int token, int pos) {
    OrcConfig* p = &m->c;
    int dim = p->dim, hidden = p->hidden_dim, hs = dim / p->n_heads;
    int kv_dim = dim * p->n_kv_heads / p->n_heads, kv_mul = p->n_heads / p->n_kv_heads;
    int gs = m->gs;
    float* x = m->x;
    memcpy(x, m->emb + (size_t)token * dim, dim * 4);            /* runq.c:332-333 */
    for (int64_t l = 0; l < p->n_layers; l++) {
        rmsnorm(m->xb, x, m->rms_att + l * dim, dim);             /* :338 */
        size_t loff = (size_t)l * m->max_seq * kv_dim;
        float* k = m->kc + loff + (size_t)pos * kv_dim;
        float* v = m->vc + loff + (size_t)pos * kv_dim;
        orc_quantize_act(m->xb, dim, gs, m->aq, m->as, NULL);     /* :345 */
        act_trace(m, dim);
        qmatmul(m, m->q, &m->wq, l, dim, dim);                     /* :346-348 */
        qmatmul(m, k, &m->wk, l, kv_dim, dim);
        qmatmul(m, v, &m->wv, l, kv_dim, dim);
        for (int i = 0; i < dim; i += 2) {                         /* RoPE :351-365 */
            int hd = i % hs;
            float freq = 1.0f / powf(10000.0f, hd / (float)hs);
            float val = pos * freq;
            float fcr = cosf(val), fci = sinf(val);
            int rotn = i < kv_dim ? 2 : 1;
            for (int r = 0; r < rotn; r++) {
                float* vec = r == 0 ? m->q : k;
                float v0 = vec[i], v1 = vec[i + 1];
                vec[i] = v0 * fcr - v1 * fci;
                vec[i + 1] = v0 * fci + v1 * fcr;
            }
        }
        for (int h = 0; h < p->n_heads; h++) {                     /* attention :369-391 */
            float* qh = m->q + h * hs;
            float* att = m->att + (size_t)h * m->max_seq;
            for (int t = 0; t <= pos; t++) {
                float* kt = m->kc + loff + (size_t)t * kv_dim + (h / kv_mul) * hs;
                float sc = 0.0f;
                for (int i = 0; i < hs; i++) sc += qh[i] * kt[i];
                att[t] = sc / sqrtf(hs);
            }
            softmax(att, pos + 1);
            float* xb = m->xb + h * hs;
            memset(xb, 0, hs * 4);
            for (int t = 0; t <= pos; t++) {
                float* vt = m->vc + loff + (size_t)t * kv_dim + (h / kv_mul) * hs;
                float a = att[t];
                for (int i = 0; i < hs; i++) xb[i] += a * vt[i];
            }
        }
        orc_quantize_act(m->xb, dim, gs, m->aq, m->as, NULL);     /* :394-396 */
        act_trace(m, dim);
        qmatmul(m, m->xb2, &m->wo, l, dim, dim);
        for (int i = 0; i < dim; i++) x[i] += m->xb2[i];
        rmsnorm(m->xb, x, m->rms_ffn + l * dim, dim);              /* :399-402 */
        orc_quantize_act(m->xb, dim, gs, m->aq, m->as, NULL);
        act_trace(m, dim);
        qmatmul(m, m->hb, &m->w1, l, hidden, dim);
        qmatmul(m, m->hb2, &m->w3, l, hidden, dim);
        for (int i = 0; i < hidden; i++) {                         /* SwiGLU :405-410 */
            float val = m->hb[i];
            val *= (1.0f / (1.0f + expf(-val)));
            val *= m->hb2[i];
            m->hb[i] = val;
        }
        orc_quantize_act(m->hb, hidden, gs, m->aq, m->as, NULL);  /* :412-414 */
        act_trace(m, hidden);
        qmatmul(m, m->xb, &m->w2, l, dim, hidden);
        for (int i = 0; i < dim; i++) x[i] += m->xb[i];
    }
    rmsnorm(x, x, m->rms_final, dim);                              /* :417-419 */
    orc_quantize_act(x, dim, gs, m->aq, m->as, NULL);
    act_trace(m, dim);
    orc_gemv(m->logits, m->aq, m->as, m->wcls.q, m->wcls.s, p->vocab_size, dim, gs, m->kind);
    return m->logits;
}

int orc_argmax(const float* v, int n) {                            /* runq.c:578-585 */
    int mi = 0;
    float mv = v[0];
    for (int i = 1; i < n; i++) if (v[i] > mv) { mi = i; mv = v[i]; }
    return mi;
}


/* ======================================================================== */
/* Kernel-order forward                                                      */
/*                                                                           */
/* The same decode step as orc_forward, with every floating-point reduction  */
/* evaluated in the order the B200 kernels of the product use, so that the   */
/* product's logits can be compared bit for bit.  The math is runq.c's       */
/* (file:line cited at each step); only the association order of the fp32    */
/* sums differs from runq.c, as it must for any parallel implementation:     */
/*  - a 32-lane warp sum is the xor butterfly (lane l adds lane l^16, l^8,   */
/*    l^4, l^2, l^1 in turn);                                                */
/*  - GEMV rows: lane L accumulates fmaf((ws*xs), D, acc) over its groups;   */
/*    which groups a lane owns depends on the kernel that runs the shape;    */
/*  - rmsnorm: 256 threads, thread t sums float4 chunks t, t+256, ...;       */
/*  - attention in chunks of 64 positions merged with max / exp weights;     */
/*  - exp is the project's own Cody-Waite + degree-7 Taylor evaluation and   */
/*    RoPE cos/sin come from a table built with runq.c's formula.            */
/* ======================================================================== */

static float pow2i(int k) {
    unsigned u = (unsigned)(k + 127) << 23;
    float f;
    memcpy(&f, &u, 4);
    return f;
}

/* exp(x): x = k ln2 + r, |r| <= ln2/2, Taylor degree 7 (same constants and
 * operation order as the product's device code). */
float orc_expf(float x) {
    if (!(x > -104.0f)) return x != x ? x : 0.0f;
    if (x > 88.75f) return pow2i(127) * 2.0f;
    const float k = rintf(x * 1.44269502f);
    float r = fmaf(k, -0.693145751953125f, x);
    r = fmaf(k, -1.42860677e-06f, r);
    float p = 1.98412698e-04f;
    p = fmaf(p, r, 1.38888889e-03f);
    p = fmaf(p, r, 8.33333377e-03f);
    p = fmaf(p, r, 4.16666679e-02f);
    p = fmaf(p, r, 1.66666672e-01f);
    p = fmaf(p, r, 0.5f);
    p = fmaf(p, r, 1.0f);
    p = fmaf(p, r, 1.0f);
    int ki = (int)k;
    if (ki > 127) return p * pow2i(127) * pow2i(ki - 127);
    if (ki < -126) return p * pow2i(ki + 64) * pow2i(-64);
    return p * pow2i(ki);
}

static float warp_butterfly(float* v) { /* 32 values, returns lane 0's result */
    for (int o = 16; o > 0; o >>= 1) {
        float nv[32];
        for (int l = 0; l < 32; l++) nv[l] = v[l] + v[l ^ o];
        memcpy(v, nv, sizeof(nv));
    }
    return v[0];
}

/* rmsnorm + quantize as the product's activation quantizer */
static void mirror_act_quant(const float* x, const float* w, int n, int gs, int8_t* xq, float* xs, float* tmp) {
    if (w) {
        float red[8];
        for (int wi = 0; wi < 8; wi++) {
            float lanes[32];
            for (int l = 0; l < 32; l++) {
                int t = wi * 32 + l;
                float ss = 0.0f;
                for (int c = t; c < n / 4; c += 256)
                    for (int e = 0; e < 4; e++) ss = fmaf(x[4 * c + e], x[4 * c + e], ss);
                lanes[l] = ss;
            }
            red[wi] = warp_butterfly(lanes);
        }
        float t = 0.0f;
        for (int wi = 0; wi < 8; wi++) t += red[wi];
        float inv = 1.0f / sqrtf(t / (float)n + 1e-5f);
        for (int i = 0; i < n; i++) tmp[i] = w[i] * (inv * x[i]);
        x = tmp;
    }
    orc_quantize_act(x, n, gs, xq, xs, NULL);
}

/* kernel selection of the product's GEMV (bulk-copy kernel when every
 * segment has an even row count and the group count is a multiple of 4) */
typedef struct {
    int mode; /* 0: whole rows (bulk copy), 1: row slices (bulk copy), 2: plain-load kernel,
                 3: tensor-core GEMM (stream-K pieces) */
    int slice_groups;
    int lpg;  /* plain-load kernel: lanes per group */
    int tile0, tiles, grid; /* mode 3: first tile of this matrix, tiles in the launch, CTAs */
} RowOrder;

/* stream-K partition of the tensor-core GEMM: CTA i owns stages [i*W/G, (i+1)*W/G) */
static int64_t sk_start(int64_t i, int64_t W, int64_t G) { return i * W / G; }
static int64_t sk_owner(int64_t s, int64_t W, int64_t G) { return ((s + 1) * G + W - 1) / W - 1; }

static RowOrder mma_order(int tile0, int tiles, int grid) {
    RowOrder o = {3, 0, 1, tile0, tiles, grid};
    return o;
}

/* One output of the tensor-core GEMM: per piece of the row's tile, fmaf over
 * its groups in K order from 0; pieces summed left to right. */
static float mma_row(const int32_t* D, const float* srow, const float* xs, int n, int gs, int64_t r, RowOrder o) {
    const int K = n / 128, gst = 128 / gs;
    const int64_t W = (int64_t)o.tiles * K;
    const int64_t G = W < o.grid ? W : o.grid;
    const int64_t t = o.tile0 + r / 128, tk0 = t * K;
    const int64_t first = sk_owner(tk0, W, G), last = sk_owner(tk0 + K - 1, W, G);
    float y = 0.0f;
    for (int64_t i = first; i <= last; i++) {
        int64_t k0 = sk_start(i, W, G), k1 = sk_start(i + 1, W, G);
        if (k0 < tk0) k0 = tk0;
        if (k1 > tk0 + K) k1 = tk0 + K;
        float acc = 0.0f;
        for (int64_t g = (k0 - tk0) * gst; g < (k1 - tk0) * gst; g++) acc = fmaf(srow[g] * xs[g], (float)D[g], acc);
        y = i == first ? acc : y + acc;
    }
    return y;
}

void orc_gemm_mma(float* out, const int8_t* xq, const float* xs, const uint8_t* wq, const float* ws, int B,
                  int64_t rows, int64_t n, int gs, int kind, int tile0, int tiles, int grid) {
    const int ng = (int)(n / gs);
    const size_t rb = kind == 8 ? (size_t)n : (size_t)n / 2;
    int32_t* D = (int32_t*)malloc(sizeof(int32_t) * ng);
    RowOrder o = mma_order(tile0, tiles, grid);
    for (int b = 0; b < B; b++)
        for (int64_t r = 0; r < rows; r++) {
            for (int g = 0; g < ng; g++) {
                int32_t d = 0;
                for (int j = 0; j < gs; j++)
                    d += wval(wq + r * rb, (int64_t)g * gs + j, kind) * (int32_t)xq[(size_t)b * n + g * gs + j];
                D[g] = d;
            }
            out[(size_t)b * rows + r] = mma_row(D, ws + r * ng, xs + (size_t)b * ng, (int)n, gs, r, o);
        }
    free(D);
}

void orc_set_mma_grid(OrcModel* m, int grid) { m->mma_grid = grid; }

static RowOrder row_order(int n, int gs, int kind, int paired, int rows_even) {
    RowOrder o = {0, 0, 1};
    int ng = n / gs, rb = kind == 8 ? n : n / 2, gb = kind == 8 ? gs : gs / 2;
    if (ng % 4 == 0 && rows_even) {
        int tw = 8192 / (paired ? 2 : 1);
        if (2 * rb <= tw) o.mode = 0;
        else { o.mode = 1; o.slice_groups = (tw / 2) / gb; }
    } else {
        int cpg = gb / 16;
        o.mode = 2;
        o.lpg = cpg == 1 ? 1 : 2;
    }
    return o;
}

static float mirror_row(const uint8_t* wrow, const float* srow, const int8_t* xq, const float* xs, int n, int gs,
                        int kind, RowOrder o, int64_t r) {
    int ng = n / gs;
    if (o.mode == 3) {
        int32_t D[1024];
        for (int g = 0; g < ng; g++) {
            int32_t d = 0;
            for (int j = 0; j < gs; j++) d += wval(wrow, (int64_t)g * gs + j, kind) * (int32_t)xq[g * gs + j];
            D[g] = d;
        }
        return mma_row(D, srow, xs, n, gs, r, o);
    }
    float lanes[32] = {0};
    float tmp[32];
    for (int g = 0; g < ng; g++) {
        int32_t d = 0;
        for (int j = 0; j < gs; j++) d += wval(wrow, (int64_t)g * gs + j, kind) * (int32_t)xq[g * gs + j];
        float f = srow[g] * xs[g];
        if (o.mode == 0) {
            lanes[g % 32] = fmaf(f, (float)d, lanes[g % 32]);
        } else if (o.mode == 2) {
            int lane = o.lpg == 1 ? g % 32 : 2 * (g % 16);
            lanes[lane] = fmaf(f, (float)d, lanes[lane]);
        } else {
            int j = g / o.slice_groups, gl = g - j * o.slice_groups;
            if (gl == 0) memset(tmp, 0, sizeof(tmp));
            tmp[gl % 32] = fmaf(f, (float)d, tmp[gl % 32]);
            if (gl == o.slice_groups - 1 || g == ng - 1)
                for (int l = 0; l < 32; l++) lanes[l] = lanes[l] + tmp[l];
        }
    }
    return warp_butterfly(lanes);
}

static void mirror_gemv(float* out, const OrcQ* w, int64_t l, int64_t rows, const int8_t* xq, const float* xs, int n,
                        int gs, int kind, RowOrder o) {
    size_t rb = row_bytes(n, kind);
    const uint8_t* q = w->q + (size_t)l * rows * rb;
    const float* s = w->s + (size_t)l * rows * (n / gs);
    for (int64_t r = 0; r < rows; r++) out[r] = mirror_row(q + r * rb, s + r * (n / gs), xq, xs, n, gs, kind, o, r);
}

/* Tensor parallelism: a row-parallel product (wo, w2) as tp partial products
 * over consecutive column slices (each in the GEMV's order for its slice
 * length), summed in process order: ((y_0 + y_1) + y_2) + ... */
static void mirror_gemv_tp(float* out, const OrcQ* w, int64_t l, int64_t rows, const int8_t* xq, const float* xs, int n,
                           int gs, int kind, int tp) {
    int ns = n / tp, ng = n / gs, ngs = ns / gs;
    size_t rb = row_bytes(n, kind), rbs = row_bytes(ns, kind);
    RowOrder o = row_order(ns, gs, kind, 0, rows % 2 == 0);
    const uint8_t* q = w->q + (size_t)l * rows * rb;
    const float* s = w->s + (size_t)l * rows * ng;
    for (int64_t r = 0; r < rows; r++) {
        float y = 0.0f;
        for (int p = 0; p < tp; p++) {
            float v = mirror_row(q + r * rb + p * rbs, s + r * ng + p * ngs, xq + (size_t)p * ns, xs + (size_t)p * ngs,
                                 ns, gs, kind, o, r);
            y = p == 0 ? v : y + v;
        }
        out[r] = y;
    }
}

void orc_set_tp(OrcModel* m, int tp) { m->tp = tp; }

/* attention of one head over positions 0..pos in chunks of 64 (kernel order) */
static void mirror_attention(const float* q, const float* kc, const float* vc, size_t stride, int pos, int hs,
                             float* out) {
    enum { CH = 64 };
    int nsplit = pos / CH + 1;
    float* part_m = (float*)malloc(sizeof(float) * nsplit);
    float* part_l = (float*)malloc(sizeof(float) * nsplit);
    float* part_o = (float*)malloc(sizeof(float) * nsplit * hs);
    float rs = sqrtf((float)hs);
    float sc[CH];
    for (int s = 0; s < nsplit; s++) {
        int t0 = s * CH, nt = pos + 1 - t0 < CH ? pos + 1 - t0 : CH;
        for (int t = 0; t < nt; t++) {
            const float* k = kc + (size_t)(t0 + t) * stride;
            float lanes[32];
            for (int l = 0; l < 32; l++) {
                float p = 0.0f;
                for (int i = l; i < hs; i += 32) p = fmaf(q[i], k[i], p);
                lanes[l] = p;
            }
            sc[t] = warp_butterfly(lanes) / rs;
        }
        float m = -3.402823466e+38f;
        for (int t = 0; t < nt; t++) m = fmaxf(m, sc[t]);
        float lanes[32] = {0};
        for (int t = 0; t < nt; t++) {
            float e = orc_expf(sc[t] - m);
            sc[t] = e;
            lanes[t % 32] += e;
        }
        float lsum = warp_butterfly(lanes);
        for (int d = 0; d < hs; d++) {
            float o = 0.0f;
            for (int t = 0; t < nt; t++) o = fmaf(sc[t], vc[(size_t)(t0 + t) * stride + d], o);
            part_o[s * hs + d] = o;
        }
        part_m[s] = m;
        part_l[s] = lsum;
    }
    if (nsplit == 1) {
        for (int d = 0; d < hs; d++) out[d] = part_o[d] / part_l[0];
    } else {
        float M = -3.402823466e+38f;
        for (int s = 0; s < nsplit; s++) M = fmaxf(M, part_m[s]);
        for (int d = 0; d < hs; d++) {
            float L = 0.0f, o = 0.0f;
            for (int s = 0; s < nsplit; s++) {
                float w = orc_expf(part_m[s] - M);
                L = fmaf(part_l[s], w, L);
                o = fmaf(part_o[s * hs + d], w, o);
            }
            out[d] = o / L;
        }
    }
    free(part_m);
    free(part_l);
    free(part_o);
}

float* orc_forward_kernel_order(OrcModel* m, int token, int pos) {
    OrcConfig* p = &m->c;
    int dim = p->dim, hidden = p->hidden_dim, hs = dim / p->n_heads;
    int kv_dim = dim * p->n_kv_heads / p->n_heads, kv_mul = p->n_heads / p->n_kv_heads;
    int gs = m->gs, kind = m->kind;
    float* x = m->x;
    float* tmp = (float*)malloc(sizeof(float) * (hidden > dim ? hidden : dim));
    memcpy(x, m->emb + (size_t)token * dim, dim * 4);
    int qkv_even = dim % 2 == 0 && kv_dim % 2 == 0;
    RowOrder o_dim = row_order(dim, gs, kind, 0, qkv_even);
    RowOrder o_wo = row_order(dim, gs, kind, 0, dim % 2 == 0);
    RowOrder o_ffn = row_order(dim, gs, kind, 1, hidden % 2 == 0);
    RowOrder o_w2 = row_order(hidden, gs, kind, 0, dim % 2 == 0);
    RowOrder o_cls = row_order(dim, gs, kind, 0, p->vocab_size % 2 == 0);
    RowOrder o_q = o_dim, o_k = o_dim, o_v = o_dim;
    if (m->mma_grid > 0) {
        /* batched steps: every product on the tensor-core GEMM (qkv is one launch of three matrices) */
        int tq = dim / 128, tkv = kv_dim / 128, G = m->mma_grid;
        o_q = mma_order(0, tq + 2 * tkv, G);
        o_k = mma_order(tq, tq + 2 * tkv, G);
        o_v = mma_order(tq + tkv, tq + 2 * tkv, G);
        o_wo = mma_order(0, dim / 128, G);
        o_ffn = mma_order(0, hidden / 128, G);
        o_w2 = mma_order(0, dim / 128, G);
        o_cls = mma_order(0, p->vocab_size / 128, G);
    }
    for (int64_t l = 0; l < p->n_layers; l++) {
        size_t loff = (size_t)l * m->max_seq * kv_dim;
        float* k = m->kc + loff + (size_t)pos * kv_dim;
        float* v = m->vc + loff + (size_t)pos * kv_dim;
        mirror_act_quant(x, m->rms_att + l * dim, dim, gs, m->aq, m->as, tmp);    /* runq.c:338,345 */
        act_trace(m, dim);
        mirror_gemv(m->q, &m->wq, l, dim, m->aq, m->as, dim, gs, kind, o_q);        /* :346-348 */
        mirror_gemv(k, &m->wk, l, kv_dim, m->aq, m->as, dim, gs, kind, o_k);
        mirror_gemv(v, &m->wv, l, kv_dim, m->aq, m->as, dim, gs, kind, o_v);
        for (int i = 0; i < dim; i += 2) {                                          /* RoPE :351-365 */
            int hd = i % hs;
            float freq = 1.0f / powf(10000.0f, hd / (float)hs);
            float val = pos * freq;
            float fcr = cosf(val), fci = sinf(val);
            int rotn = i < kv_dim ? 2 : 1;
            for (int r = 0; r < rotn; r++) {
                float* vec = r == 0 ? m->q : k;
                float v0 = vec[i], v1 = vec[i + 1];
                vec[i] = v0 * fcr - v1 * fci;
                vec[i + 1] = v0 * fci + v1 * fcr;
            }
        }
        for (int h = 0; h < p->n_heads; h++)                                         /* :369-391 */
            mirror_attention(m->q + h * hs, m->kc + loff + (h / kv_mul) * hs, m->vc + loff + (h / kv_mul) * hs,
                             (size_t)kv_dim, pos, hs, m->xb + h * hs);
        mirror_act_quant(m->xb, NULL, dim, gs, m->aq, m->as, tmp);                   /* :394-396 */
        act_trace(m, dim);
        if (m->tp > 1)
            mirror_gemv_tp(m->xb2, &m->wo, l, dim, m->aq, m->as, dim, gs, kind, m->tp);
        else
            mirror_gemv(m->xb2, &m->wo, l, dim, m->aq, m->as, dim, gs, kind, o_wo);
        for (int i = 0; i < dim; i++) x[i] += m->xb2[i];
        mirror_act_quant(x, m->rms_ffn + l * dim, dim, gs, m->aq, m->as, tmp);      /* :399-402 */
        act_trace(m, dim);
        mirror_gemv(m->hb, &m->w1, l, hidden, m->aq, m->as, dim, gs, kind, o_ffn);
        mirror_gemv(m->hb2, &m->w3, l, hidden, m->aq, m->as, dim, gs, kind, o_ffn);
        for (int i = 0; i < hidden; i++) {                                           /* SwiGLU :405-410 */
            float val = m->hb[i];
            val = val * (1.0f / (1.0f + orc_expf(-val)));
            m->hb[i] = val * m->hb2[i];
        }
        mirror_act_quant(m->hb, NULL, hidden, gs, m->aq, m->as, tmp);                /* :412-414 */
        act_trace(m, hidden);
        if (m->tp > 1)
            mirror_gemv_tp(m->xb, &m->w2, l, dim, m->aq, m->as, hidden, gs, kind, m->tp);
        else
            mirror_gemv(m->xb, &m->w2, l, dim, m->aq, m->as, hidden, gs, kind, o_w2);
        for (int i = 0; i < dim; i++) x[i] += m->xb[i];
    }
    mirror_act_quant(x, m->rms_final, dim, gs, m->aq, m->as, tmp);                   /* :417-419 */
    act_trace(m, dim);
    mirror_gemv(m->logits, &m->wcls, 0, p->vocab_size, m->aq, m->as, dim, gs, kind, o_cls);
    free(tmp);
    return m->logits;
}
