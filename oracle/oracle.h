/*
 * Scalar CPU oracle for the group-quantized decode hot path.
 *
 * TEST INFRASTRUCTURE ONLY.  Nothing in the product library links or calls
 * this code; only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline
 * leg load it, and there only as the checker (or the timed CPU port).
 *
 * Every function restates the arithmetic of the reference with the group
 * size (GS) as a parameter.  At GS=32 / INT8 it is pinned bit-exact against
 * the reference's own runq.c (compiled from its sources into oracle/_ref by
 * oracle/Makefile) and byte-exact against tools/quantize_int8.py /
 * tools/quantize_int4.py (golden fixtures in tests/golden/).
 */
#ifndef LLAMA2Q_ORACLE_H
#define LLAMA2Q_ORACLE_H
#include <stdint.h>
#include <stddef.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Activation quantize, v1-int8-vnni/runq.c:117-139 with QBLOCK -> gs:
 * amax = max|x|, s = amax/127 (0 -> 1e-8), q = clamp(lrintf(x/s), +-127);
 * xt[b] = s*128*sum(q) (the reference's bias-correction term; may be NULL). */
void orc_quantize_act(const float* x, int n, int gs, int8_t* xq, float* xs, float* xt);

/* INT8 weight quantizer, tools/quantize_int8.py:52-63 (numpy float32
 * arithmetic, round-half-even): biased uint8 = q + 128 and fp32 scales. */
void orc_quantize_w8(const float* w, int64_t rows, int64_t cols, int gs, uint8_t* q, float* s);

/* INT4 weight quantizer, tools/quantize_int4.py:38-51: scale = amax/8,
 * q in [-8, 7], two's-complement nibbles, even element in the low nibble. */
void orc_quantize_w4(const float* w, int64_t rows, int64_t cols, int gs, uint8_t* q, float* s);

/* Exact int32 group dot products D[r, g] = sum_{k in g} qw[r,k] * xq[k].
 * kind 8: qw = biased byte - 128 (the integer identity behind
 * runq.c:150-156's VPDPBUSD + xt correction).  kind 4: qw = sign-extended
 * nibble (v5-cuda-fused/run.cu:252-269 decode, quantize_int4.py:47-50
 * order).  D is [rows, cols/gs]. */
void orc_group_dots(int32_t* D, const uint8_t* wq, const int8_t* xq,
                    int64_t rows, int64_t cols, int gs, int kind);

/* GEMV out[r] = sum_g (ws[r,g] * xs[g]) * (float)D[r,g], summed over g in
 * order (the scale epilogue of v5-cuda-fused/run.cu:305 / v3 run.cu:197). */
void orc_gemv(float* out, const int8_t* xq, const float* xs, const uint8_t* wq,
              const float* ws, int64_t rows, int64_t cols, int gs, int kind);

/* Batched form (v2-cuda/run.cu:131-162 semantics): B activation rows. */
void orc_gemm(float* out, const int8_t* xq, const float* xs, const uint8_t* wq,
              const float* ws, int B, int64_t rows, int64_t cols, int gs, int kind);

/* ---- full decode step (runq.c:320-421 with INT4 and GS as parameters) ---- */
typedef struct {
    int dim, hidden_dim, n_layers, n_heads, n_kv_heads, vocab_size, seq_len;
} OrcConfig;

typedef struct OrcModel OrcModel;

/* Reads a QLL8 v1 (INT8, GS 32), QLL4 v2 (INT4, GS 32) or the GS-carrying
 * v3 extension of either.  Returns NULL on error (message on stderr). */
OrcModel* orc_model_load(const char* path, int max_seq);
void orc_model_free(OrcModel* m);
void orc_model_info(const OrcModel* m, OrcConfig* cfg, int* kind, int* gs);
/* One token; returns the model-owned logits [vocab], overwritten by the
 * next call (runq.c:320 ownership). */
float* orc_forward(OrcModel* m, int token, int pos);
/* The same step evaluated in the B200 kernels' reduction order (fp32 sums
 * associated as the device code does), for bit-exact comparison with the
 * product.  Uses the model's own KV cache: do not mix with orc_forward on
 * one model. */
float* orc_forward_kernel_order(OrcModel* m, int token, int pos);
/* grid > 0: orc_forward_kernel_order mirrors the batched step, whose products
 * run on the tensor-core GEMM with `grid` CTAs (stream-K order); 0: batch-1 GEMV */
void orc_set_mma_grid(OrcModel* m, int grid);
/* tp > 1: orc_forward_kernel_order mirrors the tensor-parallel batch-1 step
 * over tp processes: wo and w2 as tp partial products over consecutive
 * column slices, summed in process order (the peer all-reduce's order) */
void orc_set_tp(OrcModel* m, int tp);
/* the tensor-core GEMM's fp32 order for one matrix of a launch: rows of tiles
 * tile0.. of a launch of `tiles` 128-row tiles over `grid` CTAs */
void orc_gemm_mma(float* out, const int8_t* xq, const float* xs, const uint8_t* wq, const float* ws, int B,
                  int64_t rows, int64_t n, int gs, int kind, int tile0, int tiles, int grid);
/* Record every int8 activation value the next forwards compute (in call
 * order: attention input, attention output, ffn input, ffn hidden per layer,
 * then the final norm) into buf, up to cap values; NULL stops.  Returns the
 * number of values computed since the previous call. */
long orc_act_trace(OrcModel* m, int8_t* buf, long cap);
/* Make the next forwards use the given int8 activations (n values, in the
 * trace's call order) and their group scales (n / gs values) in place of
 * their own quantizer outputs; NULL turns it off.  Returns the number of
 * values consumed since the previous call. */
long orc_act_override(OrcModel* m, const int8_t* xq, const float* xs, long n);
/* exp as evaluated by the product (Cody-Waite + Taylor degree 7). */
float orc_expf(float x);
/* sample_argmax, runq.c:578-585: first index of the maximum. */
int orc_argmax(const float* v, int n);

#ifdef __cplusplus
}
#endif
#endif
