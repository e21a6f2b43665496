/*
 * Build shim for the reference CPU runner (TEST INFRASTRUCTURE ONLY).
 *
 * Compiles the reference's own v1-int8-vnni/runq.c from where it lies (the
 * include path is given by oracle/Makefile; nothing is copied) into
 * oracle/_ref/librunq.so, with its main renamed, and exports thin wrappers
 * around its static functions so tests can pin the oracle against it:
 *   quantize_act  runq.c:117-139
 *   matmul_q8     runq.c:142-159
 *   build_transformer / forward / free_transformer  runq.c:280-421
 * plus a trace of the int8 activations forward() computes (for locating the
 * first position where a different fp32 summation order changes one int8
 * value), and bench.py --impl reference can time it on the host cores.
 */
#include <math.h>
#include <stdint.h>

/* Activation trace: runq.c calls fabsf and lrintf only inside quantize_act
 * (runq.c:123 and :130), each once per value in order, so wrapping them
 * records every activation quantize_act sees (|x|, from which the group
 * scale amax/127 follows) and every int8 value it produces (clamped as
 * quantize_act clamps it), without touching the reference source.  Off
 * unless buffers are set. */
static int8_t* g_act_q;
static float* g_act_abs;
static long g_act_cap, g_act_nq, g_act_nabs;

static long ref_lrintf_traced(float v) {
    long q = lrintf(v);
    if (g_act_q && g_act_nq < g_act_cap) g_act_q[g_act_nq] = (int8_t)(q > 127 ? 127 : (q < -127 ? -127 : q));
    g_act_nq++;
    return q;
}

static float ref_fabsf_traced(float v) {
    float a = fabsf(v);
    if (g_act_abs && g_act_nabs < g_act_cap) g_act_abs[g_act_nabs] = a;
    g_act_nabs++;
    return a;
}
#define lrintf(v) ref_lrintf_traced(v)
#define fabsf(v) ref_fabsf_traced(v)

#define main runq_main
#include "v1-int8-vnni/runq.c"
#undef main
#undef lrintf
#undef fabsf

/* Start recording into q (int8 values) and absx (|x|), cap values each (NULL
 * stops); returns the number of values quantized since the previous call. */
long ref_act_trace(int8_t* q, float* absx, long cap) {
    long n = g_act_nq;
    g_act_q = q;
    g_act_abs = absx;
    g_act_cap = cap;
    g_act_nq = g_act_nabs = 0;
    return n;
}

void ref_quantize_act(const float* x, int n, int8_t* xq, float* xs, float* xt) {
    quantize_act(x, n, xq, xs, xt);
}

void ref_matmul_q8(float* out, const int8_t* xq, const float* xs, const float* xt,
                   const uint8_t* q, const float* s, int rows, int cols) {
    QWeight w;
    w.q = (uint8_t*)q;
    w.s = (float*)s;
    w.rows = rows;
    w.cols = cols;
    w.nb = cols / QBLOCK;
    matmul_q8(out, xq, xs, xt, w);
}

void* ref_build(const char* path) {
    Transformer* t = (Transformer*)calloc(1, sizeof(Transformer));
    build_transformer(t, (char*)path);
    return t;
}

float* ref_forward(void* t, int token, int pos) { return forward((Transformer*)t, token, pos); }

int ref_vocab(void* t) { return ((Transformer*)t)->config.vocab_size; }

void ref_free(void* t) {
    free_transformer((Transformer*)t);
    free(t);
}

int ref_group_size(void) { return QBLOCK; }

/* runq.c's sampler (runq.c:587-667: temperature, softmax, xorshift64* coin,
 * multinomial or top-p) on the given logits (modified in place); *rng is the
 * sampler's state, advanced as runq.c advances it. */
int ref_sample(float* logits, int n, float temperature, float topp, unsigned long long* rng) {
    Sampler sp;
    build_sampler(&sp, n, temperature, topp, *rng);
    int next = sample(&sp, logits);
    *rng = sp.rng_state;
    free_sampler(&sp);
    return next;
}

/* runq.c's tokenizer (runq.c:444-560): load tokenizer.bin, encode text as
 * generate() does (BOS, no EOS), release. */
void* ref_tokenizer(const char* path, int vocab_size) {
    Tokenizer* t = (Tokenizer*)calloc(1, sizeof(Tokenizer));
    build_tokenizer(t, (char*)path, vocab_size);
    return t;
}

int ref_encode(void* t, const char* text, int* tokens) {
    int n = 0;
    encode((Tokenizer*)t, (char*)text, 1, 0, tokens, &n);
    return n;
}

void ref_tokenizer_free(void* t) {
    free_tokenizer((Tokenizer*)t);
    free(t);
}

void ref_set_threads(int n) { omp_set_num_threads(n); }
int ref_max_threads(void) { return omp_get_max_threads(); }
