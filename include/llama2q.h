/*
 * llama2q — B200 (sm_100a) decode hot path of llama2-min-inference:
 * group-quantized INT8 / INT4 weight x int8 activation GEMV with int32 group
 * accumulation and fp32 scale epilogue, plus the decode step around it.
 *
 * Plain C ABI: pointers, sizes and int status codes.  No torch or C++ types.
 * Every entry point names the reference interface it replaces (paths are
 * relative to the reference project root).
 *
 * Memory: unless a function says "host or device", pointers are device
 * pointers on the current CUDA device.  Work is issued on the stream set by
 * lq_set_stream (default: the legacy default stream).  Functions return
 * LQ_OK (0) or an LQ_E* code; lq_last_error() gives the message (per host
 * thread).  The reference exits the process on every error instead
 * (v1-int8-vnni/runq.c:258-275, v5-cuda-fused/run.cu:50-52).
 */
#ifndef LLAMA2Q_H
#define LLAMA2Q_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* status codes */
#define LQ_OK 0
#define LQ_EINVAL 1       /* bad argument / shape / alignment */
#define LQ_ECUDA 2        /* CUDA runtime error */
#define LQ_ENOMEM 3       /* allocation failed */
#define LQ_EIO 4          /* file open / read / write failed */
#define LQ_EFORMAT 5      /* bad magic, version or truncated checkpoint */
#define LQ_ETIMEOUT 6     /* a device-side wait ran out of its limit */
#define LQ_EUNSUPPORTED 7 /* valid input this build does not handle */

/* QuantizedTensor.kind */
#define LQ_KIND_INT8 8    /* weights: uint8 [rows, cols] = q + 128 (quantize_int8.py:62) */
#define LQ_KIND_INT4 4    /* weights: uint8 [rows, cols/2], two's-complement nibbles,
                             even column in the low nibble (quantize_int4.py:47-50) */
#define LQ_KIND_ACT8 1    /* activations: int8 [rows, cols] signed (runq.c:133) */

/* Group-quantized tensor (replaces QWeight, v1-int8-vnni/runq.c:43-49, and
 * DQWeight, v5-cuda-fused/run.cu:61-65; the activation form replaces the
 * actq/acts pair of runq.c:85-86).  Device encodings are the checkpoint's
 * own byte encodings, so loading a tensor is a plain copy. */
typedef struct QuantizedTensor {
    void* q;            /* device: quantized values (see kind) */
    float* s;           /* device: fp32 group scales [rows, cols / group_size] */
    int64_t rows;
    int64_t cols;       /* multiple of group_size */
    int32_t group_size; /* multiple of 32, <= 256 (reference: 32) */
    int32_t kind;       /* LQ_KIND_* */
} QuantizedTensor;

/* Model hyper-parameters, v1-int8-vnni/runq.c:33-41 (same field order as
 * the checkpoint header). vocab_size is positive here. */
typedef struct Config {
    int dim;
    int hidden_dim;
    int n_layers;
    int n_heads;
    int n_kv_heads;
    int vocab_size;
    int seq_len;
} Config;

typedef struct Transformer Transformer; /* opaque; runq.c:93-101 */

/* ---- context ----------------------------------------------------------- */
const char* lq_last_error(void);
/* Make `device` current for this host thread; -1 picks the device with the
 * most free memory, as the reference runners do (v2-cuda/run.cu:799-813,
 * v5-cuda-fused/run.cu:1109-1122), and reports the choice on stderr. */
int lq_select_device(int device);
int lq_set_stream(void* cuda_stream); /* cudaStream_t; NULL = legacy default */
void* lq_get_stream(void);
/* Synchronize the stream and report (then clear) the device-side error
 * words of the operator calls on the current device: the context's, and the
 * fixed scratch's when matmul_f32_noalloc has been used there.  A bounded
 * device wait that gave up in any earlier call makes this return
 * LQ_ETIMEOUT. */
int lq_sync(void);

/* Launch flags for the operator entry points.  LQ_LAUNCH_PDL lets each
 * operator kernel start (and start streaming its weights) while the previous
 * kernel on the stream is still finishing — programmatic dependent launch.
 * Activations are still read only after that kernel completes.  Set it only
 * when no kernel queued before an operator writes that operator's weights. */
#define LQ_LAUNCH_PDL 1
int lq_set_launch_flags(int flags);

/* Tracing: when set, every GEMV launched by quantize/matmul/matmul_f32
 * writes four globaltimer stamps (ns) per CTA into device_buffer
 * ([grid][4]: start, dependency satisfied, activation staged, end); NULL
 * turns it off.  The buffer must hold 4 x 148 x 8 bytes per launch and is
 * overwritten by each launch. */
int lq_set_trace(void* device_buffer);

/* Stream capture of operator calls into a CUDA graph on the library stream
 * (the reference captures its forward the same way,
 * v5-cuda-fused/run.cu:671-679).  lq_graph_end returns an executable graph
 * handle for lq_graph_launch / lq_graph_destroy. */
int lq_graph_begin(void);
int lq_graph_end(void** graph_exec);
int lq_graph_launch(void* graph_exec);
void lq_graph_destroy(void* graph_exec);

/* Fill a weight tensor (w->q, w->s allocated by the caller, rows/cols/
 * group_size/kind set) with seeded synthetic values ~ N(0, std) quantized
 * like tools/quantize_int8.py / quantize_int4.py, generated on the device;
 * identical to quantizing lq_synth_value(seed, tensor_id, r*cols+c, std). */
int lq_synth_tensor(QuantizedTensor* w, uint64_t seed, int tensor_id, float std);

/* ---- hot-path operators -------------------------------------------------- */

/* Activation quantize.  Replaces quantize_act, v1-int8-vnni/runq.c:117-139
 * (and quantize_act_kernel, v2-cuda/run.cu:102-127): per group of
 * out->group_size values, s = max|x|/127 (0 -> 1e-8), q = clamp(rint(x/s),
 * +-127).  x is fp32 [out->rows, n], host or device memory; out->q (int8)
 * and out->s must be device buffers of [rows, n] and [rows, n/gs].  Sets
 * out->cols = n and out->kind = LQ_KIND_ACT8.  The reference's xt term is
 * not produced: the kernels correct the weight bias from the group sums. */
int quantize(QuantizedTensor* out, const float* x, int n);

/* Quantized matrix-vector / matrix product.  Replaces matmul_q8,
 * v1-int8-vnni/runq.c:142-159 (INT8), matmul_q4_vec_kernel,
 * v5-cuda-fused/run.cu:276-330 (INT4) and matmul_q8_kernel,
 * v2-cuda/run.cu:131-162 (x->rows > 1), with the signature of the fp32
 * matmul(xout, x, w, n, d), v0-fp32/run.c:217: W (d x n) times x (n).
 * xout[b, i] = sum_g (w.s[i,g] * x.s[b,g]) * D[b,i,g], D the exact int32
 * group dot.  x: LQ_KIND_ACT8 [B, n]; w: LQ_KIND_INT8 / LQ_KIND_INT4 [d, n]
 * with the same group size; xout: fp32 [B, d].  All device memory. */
int matmul(float* xout, const QuantizedTensor* x, const QuantizedTensor* w, int n, int d);

/* fp32-input form: quantize x with the group size of w, then multiply, i.e.
 * runq.c's quantize_act followed by matmul_q8 (runq.c:345-348): two kernels,
 * the GEMV streaming its first weights while the quantizer runs.  x fp32 [n]
 * and xout fp32 [d] may be host or device memory; with host memory the copies
 * are part of the call, which then returns after the result is in xout. */
int matmul_f32(float* xout, const float* x, const QuantizedTensor* w, int n, int d);

/* Allocation-free form of matmul_f32, for callers that cannot allocate device
 * memory while they run (a host framework that owns all device memory and
 * forbids allocation while serving, or a latency-bound loop that cannot
 * afford a first-use cudaMalloc).  No counterpart in the reference.  Same
 * result as matmul_f32; x and xout must be device memory.  Its scratch is a
 * fixed 40 KB array in device memory held by every GPU that loads the
 * library until exit: n is limited to 32768 (larger n returns LQ_EINVAL),
 * every call on a device shares the array, and calls whose kernels overlap
 * on the GPU race on it.  The first call on a device looks up the array's
 * address; make that call before any stream capture.  A device-side error
 * of these calls (a bounded wait that gave up) is kept in the array until
 * the next lq_sync() reports it. */
int matmul_f32_noalloc(float* xout, const float* x, const QuantizedTensor* w, int n, int d);

/* ---- model ------------------------------------------------------------- */

/* Load a checkpoint: QLL8 version 1 (INT8, GS 32; tools/quantize_int8.py:11-37,
 * reader runq.c:230-278), QLL4 version 2 (INT4, GS 32; tools/quantize_int4.py:
 * 9-26, reader v5-cuda-fused/run.cu:534-551), or version 3 of either magic,
 * which adds an int32 group size after the config.  A positive vocab_size
 * (shared classifier) is accepted: the fp32 embedding is quantized at load
 * (the reference exits instead, runq.c:247-251).  max_seq_len bounds the KV
 * cache (0 = the header's seq_len).  Replaces build_transformer,
 * runq.c:280-283. */
int build_transformer(Transformer** t, const char* checkpoint_path, int max_seq_len);

/* Random-init model generated directly in device memory from a seed, with
 * the same values lq_write_checkpoint_random would write (no file I/O;
 * used for the 7B/13B/70B shapes).  kind LQ_KIND_INT8 or LQ_KIND_INT4. */
int build_transformer_random(Transformer** t, const Config* cfg, int kind, int group_size,
                             uint64_t seed, int max_seq_len);

/* One decode step: token at absolute position pos.  Returns host logits
 * [vocab] owned by t and overwritten by the next call, or NULL on error.
 * Replaces forward, v1-int8-vnni/runq.c:320-421 (GPU: run_token,
 * v5-cuda-fused/run.cu:682-695). */
float* forward(Transformer* t, int token, int pos);

/* Same step with the greedy choice made on the device: writes
 * argmax(logits) (first index of the maximum, sample_argmax runq.c:578-585)
 * to *next_token and copies 4 bytes instead of the logits. */
int forward_argmax(Transformer* t, int token, int pos, int* next_token);

/* Prompt prefill for sequence 0: tokens[0 .. n_tokens) at positions
 * start_pos .. start_pos + n_tokens - 1, written into the KV cache as if fed
 * one at a time.  The prompt runs in steps of up to 64 tokens whose rows go
 * through every product together (from 16 rows on, the tensor-core GEMM: the
 * weights are read once per step, not once per token), each row attending
 * causally over the cache up to its own position.  Returns host logits
 * [vocab] of the last prompt token (owned by t, valid until the next call),
 * or NULL on error.  Replaces the whole-sequence prompt forward of
 * v2-cuda/run.cu:347-394 (matmul_q8_kernel over T rows, :131-162, causal
 * attention :194-238) and the one-token-at-a-time prompt loop of runq.c's
 * generate (v1-int8-vnni/runq.c:691-703).  Rows below 16 use the GEMV, whose
 * per-row arithmetic is that of forward(); from 16 rows the per-row fp32
 * order is the tensor-core GEMM's. */
float* forward_prompt(Transformer* t, const int* tokens, int n_tokens, int start_pos);

/* ---- batched decode (B independent sequences, one token each per step) ---
 * The reference decodes one sequence; its batched kernel is the prompt-time
 * matmul_q8_kernel of v2-cuda/run.cu:131-162 (T rows against one weight
 * stream).  Here B sequences each hold their own KV cache and position and
 * advance together: every weight byte is streamed once per step for all B
 * rows.  Sequence b uses cache slot b; row b of the step is independent of
 * every other row (its logits are bitwise those of a batch-1 forward with the
 * same history). */

/* Size the model for up to max_batch sequences (default 1).  Releases and
 * re-creates the activations and KV caches: every sequence restarts. */
int transformer_reserve_batch(Transformer* t, int max_batch);

/* One decode step for sequences 0..batch-1: tokens[b] at positions pos[b].
 * Returns host logits [batch][vocab] owned by t and valid until the next call,
 * or NULL on error (lq_last_error()). */
float* forward_batch(Transformer* t, const int* tokens, const int* pos, int batch);

/* As forward_batch, writing only the greedy next token of every sequence. */
int forward_batch_argmax(Transformer* t, const int* tokens, const int* pos, int batch, int* next_tokens);

/* ---- tensor parallelism (the 70B shape over 2, 4 or 8 GPUs) -----------------
 * The reference runs on one device.  Here one process per GPU holds a
 * Megatron-style share of every layer: the output rows of wq, wk, wv, w1 and
 * w3 (its n_heads/tp_size query heads, n_kv_heads/tp_size kv heads and
 * hidden_dim/tp_size FFN rows) and the matching input columns of wo and w2.
 * Attention, RoPE, the KV cache and SwiGLU stay local; the wo and w2 products
 * are partial sums, completed by an all-reduce per product (two per layer)
 * inside the captured decode graph.  The all-reduce is fused into the next
 * activation quantizer: the wo / w2 products push their partial values into
 * every process's device memory over NVLink (CUDA IPC mappings set up when the
 * model is built) and the quantizer sums them once they have arrived.  Setting
 * LQ_TP_ALLREDUCE=nccl before building selects an ncclAllReduce instead.  At
 * most 8 processes, dim at most 8192, at most 1024 sequences a step.  The
 * embedding, the norms and the classifier are replicated, so every process
 * returns the full logits.  Every process calls forward / forward_argmax /
 * forward_batch / transformer_reserve_batch with the same arguments, and
 * free_transformer at the end: for tp_size > 1 it waits for the whole group
 * before the exchange memory is unmapped. */

/* Create the group id (128 bytes) on one process; the caller hands it to the
 * others (a file, a socket, torch.distributed, ...). */
int lq_tp_unique_id(void* id128);

/* As build_transformer / build_transformer_random, for process tp_rank of
 * tp_size (its GPU already selected).  All processes of the group call it;
 * it returns once every process has joined.  tp_size == 1 needs no id and runs
 * the tensor-parallel step structure on one GPU. */
int build_transformer_tp(Transformer** t, const char* checkpoint_path, int max_seq_len, int tp_rank, int tp_size,
                         const void* id128);
int build_transformer_random_tp(Transformer** t, const Config* cfg, int kind, int group_size, uint64_t seed,
                                int max_seq_len, int tp_rank, int tp_size, const void* id128);

/* Self-test of the failure path of the tensor-parallel all-reduce (no
 * counterpart in the reference, which has one device).  Runs the fused
 * all-reduce quantizer as rank 0 of a tp_size-process group (2..8) whose
 * other members never publish their partials, with a wait limit of wait_us
 * microseconds, twice in a row on the current device.  The first call's
 * bounded wait gives up and records the error; the second call sees the
 * recorded error and does not wait again.  Returns LQ_ETIMEOUT (the status a
 * decode step returns when a peer stops taking part) and the two calls'
 * device times in *first_ms / *second_ms (either may be NULL).  In a model
 * the limit is 2 s, or LQ_TP_WAIT_MS milliseconds when that is set before
 * the model is built. */
int lq_tp_wait_selftest(int tp_size, int wait_us, double* first_ms, double* second_ms);

/* Release a model (free_transformer, runq.c:285-289). */
void free_transformer(Transformer* t);

/* ---- step trace (profiling; no counterpart in the reference) -------------
 * With tracing on, every kernel of a decode step records three device-clock
 * stamps (globaltimer, ns): when its first CTA started, when its first CTA
 * got past the wait for the previous kernel (programmatic dependent launch),
 * and when its last warp finished.  Read them after a step to see where the
 * step's time goes (the reference times whole tokens only,
 * v1-int8-vnni/runq.c:710-716).  Turning tracing on or off re-captures the
 * step's graph at the next step. */
#define LQ_TRACE_QUANT 1      /* activation quantizer */
#define LQ_TRACE_GEMV 2       /* batch-1..8 GEMV */
#define LQ_TRACE_QGEMM 3      /* tensor-core GEMM */
#define LQ_TRACE_ATTENTION 4  /* split-KV attention */
#define LQ_TRACE_ALLREDUCE 5  /* tensor-parallel all-reduce fused into the quantizer */
#define LQ_TRACE_ARGMAX 6
#define LQ_TRACE_NCCL 7       /* NCCL all-reduce: a library kernel, no stamps (all bits set) */
int transformer_trace(Transformer* t, int enable);
/* After a step: *count = kernels in the step; for the first min(count,
 * max_kernels) kernels in launch order, kinds[i] (LQ_TRACE_*) and stamps[3i ..
 * 3i+2] = start, past-wait, end.  A stamp with all bits set was not recorded
 * (a kernel whose CTAs all exited before that point, or an NCCL kernel). */
int transformer_trace_read(Transformer* t, int max_kernels, int* kinds, uint64_t* stamps, int* count);

/* Copy out the model's shape, weight kind and group size. */
int transformer_config(const Transformer* t, Config* cfg, int* kind, int* group_size);

/* ---- checkpoint files (host only; no GPU needed) -------------------------- */

/* Write a llama2.c fp32 checkpoint (the input format of
 * tools/quantize_int8.py:71-96) with seeded synthetic weights: every matrix
 * and the embedding ~ N(0, std) via the project's counter-based generator,
 * RMSNorm weights = 1.  shared != 0 writes a positive vocab_size and no
 * classifier. */
int lq_write_checkpoint_fp32(const char* path, const Config* cfg, uint64_t seed, float std,
                             int shared);

/* Quantize a llama2.c fp32 checkpoint (tools/quantize_int8.py:66-126 /
 * tools/quantize_int4.py:54-115).  group_size 32 writes the reference's own
 * version 1 / 2 files; any other group size writes version 3. */
int lq_quantize_checkpoint(const char* src_fp32, const char* dst, int kind, int group_size);

/* Write a quantized checkpoint of seeded synthetic weights directly: the
 * bytes lq_write_checkpoint_fp32 (unshared classifier) followed by
 * lq_quantize_checkpoint would give, without the fp32 file (a 7B fp32
 * export is 27 GB).  Group size 32 writes the reference's version 1 (INT8) /
 * 2 (INT4) files; others version 3.  Uses all host threads (OpenMP). */
int lq_write_checkpoint_random(const char* path, const Config* cfg, int kind, int group_size, uint64_t seed,
                               float std);

/* Read only the header of a quantized checkpoint. */
int lq_read_header(const char* path, Config* cfg, int* kind, int* group_size, int* shared);

/* The synthetic generator used above (one value of tensor `tensor_id`,
 * element `index`), exposed so callers can rebuild any weight exactly. */
float lq_synth_value(uint64_t seed, int tensor_id, uint64_t index, float std);

#ifdef __cplusplus
}
#endif
#endif /* LLAMA2Q_H */
