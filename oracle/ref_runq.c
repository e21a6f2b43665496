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
 * and bench.py --impl reference can time it on the host cores.
 */
#define main runq_main
#include "v1-int8-vnni/runq.c"
#undef main

#include <omp.h>

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

void ref_set_threads(int n) { omp_set_num_threads(n); }
int ref_max_threads(void) { return omp_get_max_threads(); }
