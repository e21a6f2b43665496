// Transformer: checkpoint upload / on-device random init, and the decode
// step captured as one CUDA graph.
//
// Per layer the step is nine kernels (reference order, runq.c:335-415):
//   quantize(rmsnorm(x))  (layer 0: x = emb[token])
//   GEMV [wq|wk|wv]       epilogue RoPE(q) -> q, RoPE(k) -> K cache, v -> V cache
//   attention             split-KV over the cache, normalised fp32 output
//   quantize(att), GEMV wo            epilogue x += .
//   quantize(rmsnorm(x)), GEMV [w1|w3] epilogue h = silu(w1 x) * (w3 x)
//   quantize(h), GEMV w2              epilogue x += .
// then quantize(rmsnorm(x)), GEMV wcls and argmax.  The quantizers are
// wide one-pass kernels that also emit the int32 group sums the GEMV needs;
// every GEMV streams its weights from kernel start.  Every
// kernel is launched with programmatic dependent launch, so each GEMV's
// weight stream starts while its predecessor is finishing.  The graph reads
// token and position from device memory (the reference's d_meta idea,
// v5-cuda-fused/run.cu:671-695), so one graph serves every step.
#include <dlfcn.h>
#include <fcntl.h>
#include <nccl.h>  // types only: the library is opened at run time
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <cstdio>
#include <cstdlib>
#include <cmath>
#include <cstring>
#include <vector>

#include "lq_ctx.h"
#include "lq_device.cuh"  // kKtSlots (step-trace layout)
#include "lq_host.h"
#include "lq_kernels.h"
#include "lq_model.h"
#include "lq_ops.h"

using namespace lq;

namespace {

int64_t rbytes(int64_t cols, int kind) { return kind == LQ_KIND_INT8 ? cols : cols / 2; }


constexpr int kPromptRows = 64;  // prompt tokens per prefill step (forward_prompt)

// activation rows of the step buffers: max(max_batch, kPromptRows) (a
// prompt chunk is up to kPromptRows rows of one sequence)
int act_rows(const Transformer* t) { return t->max_batch > kPromptRows ? t->max_batch : kPromptRows; }

// one slot of the peer all-reduce exchange region: [tp][xr_rows][dim] 64-bit
// words, xr_rows = the activation rows when the region was set up
size_t xr_slot_bytes(const Transformer* t) {
    return (size_t)t->tp_size * t->xr_rows * t->c.dim * sizeof(uint64_t);
}
// slot k of the exchange region at `base` (this process's or a peer's mapping)
uint64_t* xr_slot(const Transformer* t, void* base, int k) {
    return reinterpret_cast<uint64_t*>(static_cast<char*>(base) + lq::kXrCountersBytes + k * xr_slot_bytes(t));
}

// NCCL, opened on first use: the copy a host framework already loaded
// (torch's) when there is one, else the system's libnccl.so.2
struct Nccl {
    ncclResult_t (*get_unique_id)(ncclUniqueId*);
    ncclResult_t (*comm_init_rank)(ncclComm_t*, int, ncclUniqueId, int);
    ncclResult_t (*all_reduce)(const void*, void*, size_t, ncclDataType_t, ncclRedOp_t, ncclComm_t, cudaStream_t);
    ncclResult_t (*all_gather)(const void*, void*, size_t, ncclDataType_t, ncclComm_t, cudaStream_t);
    ncclResult_t (*comm_destroy)(ncclComm_t);
    const char* (*error_string)(ncclResult_t);
};

const Nccl* nccl() {
    static Nccl f;
    static int state = 0;
    if (state == 0) {
        void* h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_NOLOAD);
        if (!h) h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
        state = -1;
        if (h) {
            f.get_unique_id = reinterpret_cast<decltype(f.get_unique_id)>(dlsym(h, "ncclGetUniqueId"));
            f.comm_init_rank = reinterpret_cast<decltype(f.comm_init_rank)>(dlsym(h, "ncclCommInitRank"));
            f.all_reduce = reinterpret_cast<decltype(f.all_reduce)>(dlsym(h, "ncclAllReduce"));
            f.all_gather = reinterpret_cast<decltype(f.all_gather)>(dlsym(h, "ncclAllGather"));
            f.comm_destroy = reinterpret_cast<decltype(f.comm_destroy)>(dlsym(h, "ncclCommDestroy"));
            f.error_string = reinterpret_cast<decltype(f.error_string)>(dlsym(h, "ncclGetErrorString"));
            if (f.get_unique_id && f.comm_init_rank && f.all_reduce && f.all_gather && f.comm_destroy && f.error_string)
                state = 1;
        }
    }
    return state == 1 ? &f : nullptr;
}

constexpr int kQgTiles = 8192;  // arrival counters: tiles of the largest launch (vocab / 128)

int alloc_q(QW& w, int64_t rows, int64_t cols, int gs, int kind) {
    w.rows = rows;
    w.cols = cols;
    cudaError_t e = cudaMalloc(&w.q, (size_t)(rows * rbytes(cols, kind)));
    if (e == cudaSuccess) e = cudaMalloc(&w.s, (size_t)(rows * (cols / gs) * 4));
    return e == cudaSuccess ? LQ_OK : cuda_fail(e, "weight allocation");
}

template <typename T>
int dalloc(T** p, size_t count) {
    cudaError_t e = cudaMalloc(reinterpret_cast<void**>(p), count * sizeof(T));
    if (e != cudaSuccess) return cuda_fail(e, "device allocation");
    return LQ_OK;
}

QW* weight_by_id(Transformer* t, int id) {
    switch (id) {
        case LQ_T_WQ: return &t->wq;
        case LQ_T_WK: return &t->wk;
        case LQ_T_WV: return &t->wv;
        case LQ_T_WO: return &t->wo;
        case LQ_T_W1: return &t->w1;
        case LQ_T_W2: return &t->w2;
        case LQ_T_W3: return &t->w3;
        case LQ_T_WCLS: return &t->wcls;
    }
    return nullptr;
}

float** f32_by_id(Transformer* t, int id) {
    switch (id) {
        case LQ_T_EMB: return &t->emb;
        case LQ_T_RMS_ATT: return &t->rms_att;
        case LQ_T_RMS_FFN: return &t->rms_ffn;
        case LQ_T_RMS_FINAL: return &t->rms_final;
    }
    return nullptr;
}

int check_config(const Config* c, int gs, int tp_size = 1) {
    LqTensorDesc t[LQ_NT];
    if (lq_tensor_table(c, t) != LQ_OK) return lq_fail(LQ_EINVAL, "bad model config");
    const int hs = c->dim / c->n_heads;
    if (hs % 2 || hs % 4) return lq_fail(LQ_EUNSUPPORTED, "head size %d must be a multiple of 4", hs);
    if (c->dim % gs || c->hidden_dim % gs) return lq_fail(LQ_EINVAL, "dim and hidden_dim must be multiples of gs");
    if (tp_size > 1) {
        if (c->n_kv_heads % tp_size || c->n_heads % tp_size)
            return lq_fail(LQ_EINVAL, "tensor parallelism: %d query / %d kv heads do not split over %d GPUs",
                           c->n_heads, c->n_kv_heads, tp_size);
        if (c->dim > 8192)
            return lq_fail(LQ_EUNSUPPORTED, "tensor parallelism: dim %d above 8192 (one quantizer CTA per row)", c->dim);
        if ((c->dim / tp_size) % gs || (c->hidden_dim / tp_size) % gs || c->hidden_dim % tp_size)
            return lq_fail(LQ_EINVAL, "tensor parallelism: dim/%d and hidden_dim/%d must be multiples of gs=%d",
                           tp_size, tp_size, gs);
    }
    return LQ_OK;
}

// device state: KV caches for max_batch sequences; activations for
// max(max_batch, kPromptRows) rows (a prompt chunk is up to kPromptRows rows
// of one sequence)
int alloc_state(Transformer* t) {
    const Config& c = t->c;
    const int B = act_rows(t);  // activation rows
    t->head_size = c.dim / c.n_heads;
    t->kv_mul = c.n_heads / c.n_kv_heads;
    t->nh_l = c.n_heads / t->tp_size;
    t->nkv_l = c.n_kv_heads / t->tp_size;
    t->dq_l = t->nh_l * t->head_size;
    t->kv_dim = t->nkv_l * t->head_size;  // this process's kv width
    t->hid_l = c.hidden_dim / t->tp_size;
    t->max_splits = (t->max_seq + kChunk - 1) / kChunk;
    const size_t kv = (size_t)t->max_batch * c.n_layers * t->kv_dim * t->max_seq;
    int rc = LQ_OK;
    rc = rc ? rc : dalloc(&t->x, (size_t)B * c.dim);
    rc = rc ? rc : dalloc(&t->q, (size_t)B * t->dq_l);
    rc = rc ? rc : dalloc(&t->att, (size_t)B * t->dq_l);
    rc = rc ? rc : dalloc(&t->h1, (size_t)B * t->hid_l);
    rc = rc ? rc : dalloc(&t->h3, (size_t)B * t->hid_l);
    if (t->tp) {
        rc = rc ? rc : dalloc(&t->x2, (size_t)B * c.dim);
        rc = rc ? rc : dalloc(&t->ybuf, (size_t)B * c.dim);
    }
    rc = rc ? rc : dalloc(&t->logits, (size_t)B * c.vocab_size);
    const int maxn = t->hid_l > c.dim ? t->hid_l : c.dim;
    // the quantized activation has padding rows up to a multiple of 8: a
    // GEMV launch reads 1, 2, 4 or 8 rows and stores only the valid ones
    const int BP = (B + 7) / 8 * 8;
    rc = rc ? rc : dalloc(&t->xq, (size_t)BP * maxn);
    rc = rc ? rc : dalloc(&t->xqs, (size_t)BP * (maxn / t->gs));
    rc = rc ? rc : dalloc(&t->xqsum, (size_t)BP * (maxn / t->gs));
    rc = rc ? rc : dalloc(&t->kc, kv);
    rc = rc ? rc : dalloc(&t->vc, kv);
    if (!rc && (kv / t->head_size >= (size_t)INT32_MAX ||
                !lq::kv_tensor_map(&t->kmap, t->kc, t->head_size, kv / t->head_size)))
        rc = lq_fail(LQ_EUNSUPPORTED, "K-cache tensor map (%zu rows of %d floats)", kv / t->head_size, t->head_size);
    rc = rc ? rc : dalloc(&t->part, (size_t)B * t->nh_l * t->max_splits * (t->head_size + 4));
    rc = rc ? rc : dalloc(&t->meta, (size_t)2 * B);
    rc = rc ? rc : dalloc(&t->next, (size_t)B);
    rc = rc ? rc : dalloc(&t->err, 1);
    rc = rc ? rc : dalloc(&t->rope, (size_t)t->max_seq * (t->head_size / 2));
    t->xs_ld = (B + 63) / 64 * 64;
    rc = rc ? rc : dalloc(&t->xs_t, (size_t)t->xs_ld * (maxn / t->gs));
    rc = rc ? rc : dalloc(&t->qg_part, qgemm_part_floats(t->num_sms));
    rc = rc ? rc : dalloc(&t->qg_cnt, (size_t)kQgTiles);
    if (rc) return rc;
    {
        // RoPE table with the reference's arithmetic (runq.c:352-356)
        const int hs = t->head_size;
        std::vector<float2> tab((size_t)t->max_seq * (hs / 2));
        for (int pos = 0; pos < t->max_seq; ++pos)
            for (int i = 0; i < hs / 2; ++i) {
                const float freq = 1.0f / powf(10000.0f, (2 * i) / (float)hs);
                const float val = pos * freq;
                tab[(size_t)pos * (hs / 2) + i] = make_float2(cosf(val), sinf(val));
            }
        cudaError_t e0 = cudaMemcpy(t->rope, tab.data(), tab.size() * sizeof(float2), cudaMemcpyHostToDevice);
        if (e0 != cudaSuccess) return cuda_fail(e0, "rope table");
    }
    cudaError_t e = cudaMemset(t->qg_cnt, 0, (size_t)kQgTiles * sizeof(int));
    if (e == cudaSuccess) e = cudaMemset(t->xs_t, 0, (size_t)t->xs_ld * (maxn / t->gs) * sizeof(float));
    if (e == cudaSuccess) e = cudaMemset(t->xq, 0, (size_t)BP * maxn);
    if (e == cudaSuccess) e = cudaMemset(t->xqs, 0, (size_t)BP * (maxn / t->gs) * sizeof(float));
    if (e == cudaSuccess) e = cudaMemset(t->xqsum, 0, (size_t)BP * (maxn / t->gs) * sizeof(int));
    if (e == cudaSuccess) e = cudaMemset(t->err, 0, sizeof(int));
    if (e == cudaSuccess) e = cudaMemset(t->meta, 0, 2 * B * sizeof(int));
    if (e == cudaSuccess) e = cudaMemset(t->kc, 0, kv * sizeof(float));
    if (e == cudaSuccess) e = cudaMemset(t->vc, 0, kv * sizeof(float));
    if (e == cudaSuccess) e = cudaMallocHost(&t->h_logits, (size_t)B * c.vocab_size * sizeof(float));
    if (e == cudaSuccess) e = cudaMallocHost(&t->h_meta, 2 * B * sizeof(int) + 64);
    if (e == cudaSuccess) e = cudaMallocHost(&t->h_next, B * sizeof(int) + 64);
    if (e == cudaSuccess) e = cudaMallocHost(&t->h_err, 64);
    if (e == cudaSuccess && !t->stream) e = cudaStreamCreateWithFlags(&t->stream, cudaStreamNonBlocking);
    if (e != cudaSuccess) return cuda_fail(e, "state allocation");
    return LQ_OK;
}

bool use_mma(const Transformer* t, int batch) { return batch >= t->mma_min; }

// release the per-sequence state (activations, caches, host mirrors, graph)
void free_state(Transformer* t) {
    if (t->stream) cudaStreamSynchronize(t->stream);
    if (t->exec) cudaGraphExecDestroy(t->exec);
    if (t->graph) cudaGraphDestroy(t->graph);
    t->exec = nullptr;
    t->graph = nullptr;
    t->graph_batch = 0;
    if (t->pexec) cudaGraphExecDestroy(t->pexec);
    if (t->pgraph) cudaGraphDestroy(t->pgraph);
    t->pexec = nullptr;
    t->pgraph = nullptr;
    t->pgraph_rows = 0;
    void* bufs[] = {t->x, t->q, t->att, t->h1, t->h3, t->xq, t->xqs, t->xqsum, t->logits, t->kc, t->vc,
                    t->part, t->meta, t->next, t->err, t->rope, t->xs_t, t->qg_part, t->qg_cnt,
                    t->x2, t->ybuf};
    for (void* b : bufs) cudaFree(b);
    t->xs_t = t->qg_part = t->x2 = t->ybuf = nullptr;
    t->qg_cnt = nullptr;
    t->x = t->q = t->att = t->h1 = t->h3 = t->logits = t->kc = t->vc = t->part = nullptr;
    t->xq = nullptr;
    t->xqs = nullptr;
    t->xqsum = t->meta = t->next = t->err = nullptr;
    t->rope = nullptr;
    cudaFreeHost(t->h_logits);
    cudaFreeHost(t->h_meta);
    cudaFreeHost(t->h_next);
    cudaFreeHost(t->h_err);
    t->h_logits = nullptr;
    t->h_meta = t->h_next = t->h_err = nullptr;
}

// rows per GEMV launch: the largest kernel row count (8, 4, 2, 1) whose int8
// activation rows fit the shared-memory budget of the bulk-copy kernel
int gemv_chunk(int cols) {
    for (int nb = 8; nb > 1; nb /= 2)
        if ((int64_t)nb * cols <= 112 * 1024) return nb;
    return 1;
}

// One GEMV over `batch` activation rows: launches of up to gemv_chunk rows,
// the last one rounded up to a kernel row count with the extra rows unstored.
cudaError_t gemv_rows(Transformer* t, const GemvArgs& a, int kind, int batch, cudaStream_t st);

// The product of one decode stage for `batch` activation rows: from
// t->mma_min rows on, on the tensor cores (up to 64 rows per launch), else
// the GEMV.
cudaError_t product_rows(Transformer* t, const GemvArgs& a, int batch, cudaStream_t st) {
    const int kind = t->kind;
    if (use_mma(t, batch) && qgemm_ok(a, kind, batch < 64 ? batch : 64) && qgemm_max_tiles(a) <= kQgTiles) {
        const int ng = a.cols / a.gs;
        for (int b0 = 0; b0 < batch; b0 += 64) {
            const int rows = batch - b0 < 64 ? batch - b0 : 64;
            GemvArgs c = a;
            c.nb = c.nvalid = rows;
            c.xq = a.xq + (size_t)b0 * a.cols;
            c.xs = a.xs + (size_t)b0 * ng;
            c.xsum_in = nullptr;
            c.meta = a.meta + 2 * b0;
            for (int i = 0; i < c.nseg; ++i)
                if (c.seg[i].y) c.seg[i].y += (size_t)b0 * a.y_stride;
            c.ll_row0 = a.ll_row0 + b0;
            if (c.kcache) c.kcache += (size_t)b0 * a.kv_seq_stride;
            if (c.vcache) c.vcache += (size_t)b0 * a.kv_seq_stride;
            // this chunk's scale table: [ng][npad] at chunk offset ng * 64
            c.kt = kt_next(t, LQ_TRACE_QGEMM);
            cudaError_t e = qgemm_launch(c, kind, t->xs_t + (size_t)(b0 / 64) * ng * 64, qgemm_npad(rows), t->qg_part,
                                         t->qg_cnt, st, true, t->num_sms);
            if (e != cudaSuccess) return e;
        }
        return cudaSuccess;
    }
    return gemv_rows(t, a, kind, batch, st);
}

cudaError_t gemv_rows(Transformer* t, const GemvArgs& a, int kind, int batch, cudaStream_t st) {
    const int chunk = gemv_chunk(a.cols);
    const int ng = a.cols / a.gs;
    for (int b0 = 0; b0 < batch; b0 += chunk) {
        const int left = batch - b0;
        int nb = 1;
        while (nb < left && nb < chunk) nb *= 2;
        GemvArgs c = a;
        c.nb = nb;
        c.nvalid = left < nb ? left : nb;
        c.xq = a.xq + (size_t)b0 * a.cols;
        c.xs = a.xs + (size_t)b0 * ng;
        c.xsum_in = a.xsum_in ? a.xsum_in + (size_t)b0 * ng : nullptr;
        if (c.xf) c.xf = a.xf + (size_t)b0 * a.cols;
        if (c.x_out) c.x_out = a.x_out + (size_t)b0 * a.cols;
        c.meta = a.meta + 2 * b0;
        for (int i = 0; i < c.nseg; ++i)
            if (c.seg[i].y) c.seg[i].y += (size_t)b0 * a.y_stride;
        c.ll_row0 = a.ll_row0 + b0;
        if (c.kcache) c.kcache += (size_t)b0 * a.kv_seq_stride;
        if (c.vcache) c.vcache += (size_t)b0 * a.kv_seq_stride;
        c.kt = kt_next(t, LQ_TRACE_GEMV);
        cudaError_t e = gemv_launch(c, kind, st, true, t->num_sms);
        if (e != cudaSuccess) return e;
    }
    return cudaSuccess;
}

Transformer* new_transformer(const Config* c, int kind, int gs, int max_seq, int max_batch) {
    Transformer* t = new Transformer();
    t->c = *c;
    t->kind = kind;
    t->gs = gs;
    t->max_seq = (max_seq > 0 && max_seq < c->seq_len) ? max_seq : c->seq_len;
    t->max_batch = max_batch;
    if (const char* e = getenv("LQ_MMA_MIN_ROWS")) {
        t->mma_min = atoi(e);
        if (t->mma_min < 1) t->mma_min = 1 << 30;  // 0 or negative: never
    }
    cudaGetDevice(&t->dev);
    cudaDeviceGetAttribute(&t->num_sms, cudaDevAttrMultiProcessorCount, t->dev);
    return t;
}

}  // namespace

namespace lq {

uint64_t* kt_next(Transformer* t, int kind) {
    if (!t->ktr || t->ktr_n >= t->ktr_cap) return nullptr;
    t->ktr_kind[t->ktr_n] = kind;
    return t->ktr + 3 * kKtSlots * (size_t)t->ktr_n++;
}

// Issue one decode step for `batch` sequences on t->stream (capturable).
int forward_launch(Transformer* t, int batch) {
    t->ktr_n = 0;
    const Config& c = t->c;
    const int kind = t->kind, gs = t->gs;
    // local widths: the whole model on one GPU, or this process's share under tensor parallelism
    const int D = c.dim, DQ = t->dq_l, H = t->hid_l, KV = t->kv_dim, hs = t->head_size;
    const int64_t rbD = rbytes(D, kind), rbQ = rbytes(DQ, kind), rbH = rbytes(H, kind);
    const int ngD = D / gs, ngQ = DQ / gs, ngH = H / gs;
    const int64_t kv_layer = (int64_t)t->nkv_l * t->max_seq * hs;
    // decode: row b is sequence b (its own cache); prompt: every row is a
    // position of sequence prompt_seq (one cache, no stride between rows)
    const int64_t kv_seq = t->prompt_seq >= 0 ? 0 : (int64_t)c.n_layers * kv_layer;
    float* const kc = t->kc + (t->prompt_seq >= 0 ? (int64_t)t->prompt_seq * c.n_layers * kv_layer : 0);
    float* const vc = t->vc + (t->prompt_seq >= 0 ? (int64_t)t->prompt_seq * c.n_layers * kv_layer : 0);
    cudaStream_t st = t->stream;
    auto base = [&](GemvArgs& a, int cols) {
        a = GemvArgs{};
        a.cols = cols;
        a.gs = gs;
        a.nb = batch;
        a.y_stride = D;
        a.meta = t->meta;
        a.rope = t->rope;
        a.head_size = hs;
        a.max_seq = t->max_seq;
        a.kv_seq_stride = kv_seq;
        a.err = t->err;
    };
    cudaError_t e;
    // activation quantizer in front of every GEMV (quantize_act, runq.c:345,394,400,412,418)
    auto qargs = [&](int mode, const float* x, int n, const float* rms_w, float* x_out = nullptr,
                     const float* y = nullptr) -> ActQuantArgs {
        ActQuantArgs q{};
        q.mode = mode;
        q.n = n;
        q.gs = gs;
        q.nb = batch;
        q.x = x;
        q.y = y;
        q.rms_w = rms_w;
        q.emb = t->emb;
        q.meta = t->meta;
        q.x_out = x_out ? x_out : t->x;
        q.xq = t->xq;
        q.xs = t->xqs;
        q.xsum = t->xqsum;
        if (use_mma(t, batch)) {
            q.xs_t = t->xs_t;
            q.xs_nfull = batch / 64;
            q.xs_npad_last = batch % 64 ? qgemm_npad(batch % 64) : 64;
            q.xs_t_mul = kind == LQ_KIND_INT4 ? 0.0625f : 1.0f;
        }
        q.kt = kt_next(t, LQ_TRACE_QUANT);
        return q;
    };
    auto quant = [&](int mode, const float* x, int n, const float* rms_w, float* x_out = nullptr,
                     const float* y = nullptr) -> cudaError_t {
        return act_quant_launch(qargs(mode, x, n, rms_w, x_out, y), st, true);
    };
    auto qin = [&](GemvArgs& a) {
        a.in_mode = IN_QUANT;
        a.xq = t->xq;
        a.xs = t->xqs;
        a.xsum_in = t->xqsum;
    };
    // tensor parallelism: wo and w2 give partial sums over this process's
    // columns; they are all-reduced and added to the residual stream by the
    // next quantizer, which reads one residual buffer and writes the other
    auto allreduce = [&]() -> int {
        if (t->tp_size == 1 || !t->tp_nccl) return LQ_OK;
        kt_next(t, LQ_TRACE_NCCL);  // a library kernel: kind recorded, no stamps
        const ncclResult_t r = nccl()->all_reduce(t->ybuf, t->ybuf, (size_t)batch * D, ncclFloat, ncclSum,
                                                  static_cast<ncclComm_t>(t->comm), st);
        return r == ncclSuccess ? LQ_OK : lq_fail(LQ_ECUDA, "all-reduce: %s", nccl()->error_string(r));
    };
    // peer all-reduce: wo writes its partial to slot 0 of this process's
    // exchange region, w2 to slot 1; the next quantizer reduces over the peers
    const bool peer = t->tp_size > 1 && !t->tp_nccl;
    auto add_quant = [&](const float* x, const float* rms_w, float* x_out, int k) -> cudaError_t {
        if (!peer) return quant(IN_ADD_RMSNORM, x, D, rms_w, x_out, t->ybuf);
        PeerAddArgs p{};
        // the quantizer fields as quant() fills them
        p.q.mode = IN_ADD_RMSNORM;
        p.q.n = D;
        p.q.gs = gs;
        p.q.nb = batch;
        p.q.x = x;
        p.q.rms_w = rms_w;
        p.q.x_out = x_out;
        p.q.xq = t->xq;
        p.q.xs = t->xqs;
        p.q.xsum = t->xqsum;
        if (use_mma(t, batch)) {
            p.q.xs_t = t->xs_t;
            p.q.xs_nfull = batch / 64;
            p.q.xs_npad_last = batch % 64 ? qgemm_npad(batch % 64) : 64;
            p.q.xs_t_mul = kind == LQ_KIND_INT4 ? 0.0625f : 1.0f;
        }
        p.slot = xr_slot(t, t->xr, k);
        p.ll_rows = t->xr_rows;
        p.counters = static_cast<uint32_t*>(t->xr);
        p.tp_rank = t->tp_rank;
        p.tp_size = t->tp_size;
        p.err = t->err;
        p.wait_ns = t->tp_wait_ns;
        p.q.kt = kt_next(t, LQ_TRACE_ALLREDUCE);
        return peer_add_quant_launch(p, st, true);
    };
    // the wo / w2 products under the peer all-reduce: partial values pushed to
    // slot k of every process's exchange region
    auto push_to = [&](GemvArgs& a, int k) {
        a.seg[0].epi = EPI_PUSH;
        a.seg[0].y = nullptr;
        for (int r = 0; r < t->tp_size; ++r) a.ll[r] = xr_slot(t, t->xr_peer[r], k);
        a.ll_call = static_cast<const uint32_t*>(t->xr);
        a.ll_tp = t->tp_size;
        a.ll_rank = t->tp_rank;
        a.ll_rows = t->xr_rows;
        a.ll_row0 = 0;
    };
    float* xa = t->x;              // residual stream after attention's add (and the embedding)
    float* xb = t->tp ? t->x2 : t->x;  // after the ffn's add
    int rc;
    for (int l = 0; l < c.n_layers; ++l) {
        GemvArgs a;
        // 1. q, k, v (attention rmsnorm + quantize first; layer 0 starts from emb[token])
        const float* rms_a = t->rms_att + (size_t)l * D;
        if (l == 0)
            e = quant(IN_RMSNORM_EMB, xa, D, rms_a, xa);
        else if (t->tp)
            e = add_quant(xb, rms_a, xa, 1);
        else
            e = quant(IN_RMSNORM, xa, D, rms_a);
        if (e != cudaSuccess) return cuda_fail(e, "attention rmsnorm");
        base(a, D);
        a.seg[0] = {t->wq.q + (size_t)l * DQ * rbD, t->wq.s + (size_t)l * DQ * ngD, t->q, DQ, EPI_ROPE_Q};
        a.seg[1] = {t->wk.q + (size_t)l * KV * rbD, t->wk.s + (size_t)l * KV * ngD, nullptr, KV, EPI_ROPE_KCACHE};
        a.seg[2] = {t->wv.q + (size_t)l * KV * rbD, t->wv.s + (size_t)l * KV * ngD, nullptr, KV, EPI_VCACHE};
        a.nseg = 3;
        a.y_stride = DQ;
        qin(a);
        a.kcache = kc + l * kv_layer;
        a.vcache = vc + l * kv_layer;
        if ((e = product_rows(t, a, batch, st)) != cudaSuccess) return cuda_fail(e, "qkv gemv");
        // 2. attention (this process's heads)
        AttnArgs at{};
        at.kmap = t->kmap;
        at.krow = (kc + l * kv_layer - t->kc) / hs;
        at.q = t->q;
        at.kcache = kc + l * kv_layer;
        at.vcache = vc + l * kv_layer;
        at.out = t->att;
        at.part = t->part;
        at.meta = t->meta;
        at.err = t->err;
        at.kv_seq_stride = kv_seq;
        at.q_stride = DQ;
        at.n_heads = t->nh_l;
        at.n_kv_heads = t->nkv_l;
        at.kv_mul = t->kv_mul;
        at.head_size = hs;
        at.max_seq = t->max_seq;
        at.max_splits = t->max_splits;
        at.kt = kt_next(t, LQ_TRACE_ATTENTION);
        if ((e = attention_launch(at, batch, st, true)) != cudaSuccess) return cuda_fail(e, "attention");
        // 3. wo + residual
        AttnQuantArgs aq{};
        aq.q = qargs(IN_F32, t->att, DQ, nullptr);
        aq.part = t->part;
        aq.head_size = hs;
        aq.max_splits = t->max_splits;
        if ((e = attn_quant_launch(aq, st, true)) != cudaSuccess) return cuda_fail(e, "attention merge + quantize");
        base(a, DQ);
        a.seg[0] = {t->wo.q + (size_t)l * D * rbQ, t->wo.s + (size_t)l * D * ngQ, t->tp ? t->ybuf : xa, D,
                    t->tp ? EPI_STORE : EPI_ADD};
        a.nseg = 1;
        if (peer) push_to(a, 0);
        qin(a);
        if ((e = product_rows(t, a, batch, st)) != cudaSuccess) return cuda_fail(e, "wo gemv");
        if ((rc = allreduce())) return rc;
        // 4. w1 | w3 paired, SwiGLU in the epilogue: h1 = silu(x.w1) * (x.w3)
        const float* rms_f = t->rms_ffn + (size_t)l * D;
        e = t->tp ? add_quant(xa, rms_f, xb, 0) : quant(IN_RMSNORM, xa, D, rms_f);
        if (e != cudaSuccess) return cuda_fail(e, "ffn rmsnorm");
        base(a, D);
        a.seg[0] = {t->w1.q + (size_t)l * H * rbD, t->w1.s + (size_t)l * H * ngD, t->h1, H, EPI_SWIGLU,
                    t->w3.q + (size_t)l * H * rbD, t->w3.s + (size_t)l * H * ngD};
        a.nseg = 1;
        a.paired = 1;
        a.y_stride = H;
        qin(a);
        if ((e = product_rows(t, a, batch, st)) != cudaSuccess) return cuda_fail(e, "w1/w3 gemv");
        // 5. w2 + residual
        if ((e = quant(IN_F32, t->h1, H, nullptr)) != cudaSuccess) return cuda_fail(e, "ffn quantize");
        base(a, H);
        a.seg[0] = {t->w2.q + (size_t)l * D * rbH, t->w2.s + (size_t)l * D * ngH, t->tp ? t->ybuf : xb, D,
                    t->tp ? EPI_STORE : EPI_ADD};
        a.nseg = 1;
        if (peer) push_to(a, 1);
        qin(a);
        if ((e = product_rows(t, a, batch, st)) != cudaSuccess) return cuda_fail(e, "w2 gemv");
        if ((rc = allreduce())) return rc;
    }
    GemvArgs a;
    e = t->tp ? add_quant(xb, t->rms_final, xa, 1) : quant(IN_RMSNORM, xa, D, t->rms_final);
    if (e != cudaSuccess) return cuda_fail(e, "final rmsnorm");
    base(a, D);
    a.seg[0] = {t->wcls.q, t->wcls.s, t->logits, c.vocab_size, EPI_STORE};
    a.nseg = 1;
    a.y_stride = c.vocab_size;
    qin(a);
    if ((e = product_rows(t, a, batch, st)) != cudaSuccess) return cuda_fail(e, "classifier gemv");
    if ((e = argmax_launch(t->logits, c.vocab_size, batch, c.vocab_size, t->next, st, true,
                           kt_next(t, LQ_TRACE_ARGMAX))) != cudaSuccess)
        return cuda_fail(e, "argmax");
    return LQ_OK;
}

int kernels_per_step(const Transformer* t, int batch) {
    if (use_mma(t, batch)) {
        const int g = (batch + 63) / 64;
        return t->c.n_layers * (5 + 4 * g) + 2 + g;
    }
    const int cd = gemv_chunk(t->c.dim), ch = gemv_chunk(t->hid_l), cq = gemv_chunk(t->dq_l);
    const int gd = (batch + cd - 1) / cd, gh = (batch + ch - 1) / ch, gq = (batch + cq - 1) / cq;
    // per layer: 4 quantizers, attention, GEMVs qkv / wo / w1|w3 / w2
    return t->c.n_layers * (5 + 2 * gd + gq + gh) + 2 + gd;
}

static int ensure_graph(Transformer* t, int batch) {
    if (t->exec && t->graph_batch == batch) return LQ_OK;
    if (t->exec) {
        cudaGraphExecDestroy(t->exec);
        t->exec = nullptr;
    }
    if (t->graph) {
        cudaGraphDestroy(t->graph);
        t->graph = nullptr;
    }
    cudaError_t e = cudaStreamBeginCapture(t->stream, cudaStreamCaptureModeThreadLocal);
    if (e != cudaSuccess) return cuda_fail(e, "begin capture");
    int rc = forward_launch(t, batch);
    cudaGraph_t g = nullptr;
    e = cudaStreamEndCapture(t->stream, &g);
    if (rc) {
        if (g) cudaGraphDestroy(g);
        return rc;
    }
    if (e != cudaSuccess) return cuda_fail(e, "end capture");
    t->graph = g;
    e = cudaGraphInstantiate(&t->exec, g, 0);
    if (e != cudaSuccess) return cuda_fail(e, "graph instantiate");
    t->graph_batch = batch;
    return LQ_OK;
}

// The prompt step's graph for `rows` rows (every row a position of sequence 0).
static int ensure_prompt_graph(Transformer* t, int rows) {
    if (t->pexec && t->pgraph_rows == rows) return LQ_OK;
    if (t->pexec) cudaGraphExecDestroy(t->pexec);
    if (t->pgraph) cudaGraphDestroy(t->pgraph);
    t->pexec = nullptr;
    t->pgraph = nullptr;
    t->pgraph_rows = 0;
    cudaError_t e = cudaStreamBeginCapture(t->stream, cudaStreamCaptureModeThreadLocal);
    if (e != cudaSuccess) return cuda_fail(e, "begin capture");
    t->prompt_seq = 0;
    int rc = forward_launch(t, rows);
    t->prompt_seq = -1;
    cudaGraph_t g = nullptr;
    e = cudaStreamEndCapture(t->stream, &g);
    if (rc) {
        if (g) cudaGraphDestroy(g);
        return rc;
    }
    if (e != cudaSuccess) return cuda_fail(e, "end capture");
    t->pgraph = g;
    e = cudaGraphInstantiate(&t->pexec, g, 0);
    if (e != cudaSuccess) return cuda_fail(e, "graph instantiate");
    t->pgraph_rows = rows;
    return LQ_OK;
}

// Prompt prefill: tokens[0..n) at positions start..start+n-1 of sequence 0,
// in steps of up to kPromptRows rows; the last token's logits go to h_logits.
int run_prompt(Transformer* t, const int* tokens, int n, int start) {
    if (!t->x) return lq_fail(LQ_EINVAL, "model has no decode state (a failed transformer_reserve_batch)");
    if (n < 1 || start < 0 || (int64_t)start + n > t->max_seq)
        return lq_fail(LQ_EINVAL, "prompt of %d tokens at position %d does not fit the %d positions", n, start,
                       t->max_seq);
    for (int i = 0; i < n; ++i)
        if (tokens[i] < 0 || tokens[i] >= t->c.vocab_size)
            return lq_fail(LQ_EINVAL, "token %d out of range [0, %d)", tokens[i], t->c.vocab_size);
    cudaStream_t st = t->stream;
    for (int done = 0; done < n;) {
        const int rows = n - done < kPromptRows ? n - done : kPromptRows;
        for (int b = 0; b < rows; ++b) {
            t->h_meta[2 * b] = tokens[done + b];
            t->h_meta[2 * b + 1] = start + done + b;
        }
        int rc = ensure_prompt_graph(t, rows);
        if (rc) return rc;
        cudaError_t e = cudaMemcpyAsync(t->meta, t->h_meta, 2 * rows * sizeof(int), cudaMemcpyHostToDevice, st);
        if (e == cudaSuccess) e = cudaGraphLaunch(t->pexec, st);
        done += rows;
        if (e == cudaSuccess && done == n)
            e = cudaMemcpyAsync(t->h_logits, t->logits + (size_t)(rows - 1) * t->c.vocab_size,
                                (size_t)t->c.vocab_size * sizeof(float), cudaMemcpyDeviceToHost, st);
        if (e == cudaSuccess) e = cudaMemcpyAsync(t->h_err, t->err, sizeof(int), cudaMemcpyDeviceToHost, st);
        if (e == cudaSuccess) e = cudaStreamSynchronize(st);
        if (e != cudaSuccess) return cuda_fail(e, "prompt step");
        if (t->h_err[0] != 0) {
            const int code = t->h_err[0];
            cudaMemsetAsync(t->err, 0, sizeof(int), st);
            cudaStreamSynchronize(st);
            return lq_fail(LQ_ETIMEOUT, "device-side wait gave up in a prompt step (code 0x%x)", code);
        }
    }
    return LQ_OK;
}

// One step for `batch` sequences: H2D tokens/positions, graph, optional D2H.
int run_step(Transformer* t, const int* tokens, const int* pos, int batch, bool want_logits, bool want_next) {
    if (!t->x) return lq_fail(LQ_EINVAL, "model has no decode state (a failed transformer_reserve_batch)");
    if (batch < 1 || batch > t->max_batch)
        return lq_fail(LQ_EINVAL, "batch %d out of range [1, %d]", batch, t->max_batch);
    for (int b = 0; b < batch; ++b) {
        if (tokens[b] < 0 || tokens[b] >= t->c.vocab_size)
            return lq_fail(LQ_EINVAL, "token %d out of range [0, %d)", tokens[b], t->c.vocab_size);
        if (pos[b] < 0 || pos[b] >= t->max_seq)
            return lq_fail(LQ_EINVAL, "pos %d out of range [0, %d)", pos[b], t->max_seq);
        t->h_meta[2 * b] = tokens[b];
        t->h_meta[2 * b + 1] = pos[b];
    }
    int rc = ensure_graph(t, batch);
    if (rc) return rc;
    cudaStream_t st = t->stream;
    cudaError_t e = cudaMemcpyAsync(t->meta, t->h_meta, 2 * batch * sizeof(int), cudaMemcpyHostToDevice, st);
    if (e == cudaSuccess && t->ktr) e = cudaMemsetAsync(t->ktr, 0xFF, 3 * kKtSlots * sizeof(uint64_t) * t->ktr_cap, st);
    if (e == cudaSuccess) e = cudaGraphLaunch(t->exec, st);
    if (e == cudaSuccess && want_logits)
        e = cudaMemcpyAsync(t->h_logits, t->logits, (size_t)batch * t->c.vocab_size * sizeof(float),
                            cudaMemcpyDeviceToHost, st);
    if (e == cudaSuccess && want_next)
        e = cudaMemcpyAsync(t->h_next, t->next, batch * sizeof(int), cudaMemcpyDeviceToHost, st);
    if (e == cudaSuccess) e = cudaMemcpyAsync(t->h_err, t->err, sizeof(int), cudaMemcpyDeviceToHost, st);
    if (e == cudaSuccess) e = cudaStreamSynchronize(st);
    if (e != cudaSuccess) return cuda_fail(e, "decode step");
    if (t->h_err[0] != 0) {
        const int code = t->h_err[0];
        cudaMemsetAsync(t->err, 0, sizeof(int), st);
        cudaStreamSynchronize(st);
        return lq_fail(LQ_ETIMEOUT, "device-side wait gave up in the decode step (code 0x%x)", code);
    }
    return LQ_OK;
}

}  // namespace lq

namespace {

// How tensor parallelism splits a stacked [L * rows, cols] tensor: 0 = whole
// (embedding-side and classifier tensors, replicated), 1 = output rows of
// every layer (wq, wk, wv, w1, w3), 2 = input columns (wo, w2).
int tp_split(int id) {
    switch (id) {
        case LQ_T_WQ: case LQ_T_WK: case LQ_T_WV: case LQ_T_W1: case LQ_T_W3: return 1;
        case LQ_T_WO: case LQ_T_W2: return 2;
    }
    return 0;
}

// this process's rows x cols of tensor d
void tp_local_shape(const Transformer* t, const LqTensorDesc& d, int64_t* rows, int64_t* cols) {
    *rows = d.rows;
    *cols = d.cols;
    if (!t->tp) return;
    if (tp_split(d.id) == 1) *rows = d.rows / t->tp_size;
    if (tp_split(d.id) == 2) *cols = d.cols / t->tp_size;
}

// Peer all-reduce setup (collective): allocate and zero this process's
// exchange region, export it (CUDA IPC), gather every process's handle with
// one NCCL all-gather and map the peers' regions.  The all-gather completes
// only after every process has zeroed its region, so no flag is written
// before its owner has cleared it.
int xr_setup(Transformer* t) {
    const int size = t->tp_size, rank = t->tp_rank;
    if (size > lq::kTpMax) return lq_fail(LQ_EUNSUPPORTED, "peer all-reduce over %d GPUs (at most %d)", size, lq::kTpMax);
    t->xr_rows = act_rows(t);
    const size_t bytes = lq::kXrCountersBytes + 2 * xr_slot_bytes(t);
    cudaError_t e = cudaMalloc(&t->xr, bytes);
    if (e != cudaSuccess) return cuda_fail(e, "exchange region");
    cudaStream_t st = nullptr;
    char* hbuf = nullptr;
    cudaIpcMemHandle_t own;
    e = cudaStreamCreateWithFlags(&st, cudaStreamNonBlocking);
    if (e == cudaSuccess) e = cudaMemsetAsync(t->xr, 0, bytes, st);
    if (e == cudaSuccess) e = cudaIpcGetMemHandle(&own, t->xr);
    if (e == cudaSuccess) e = cudaMalloc(&hbuf, sizeof(cudaIpcMemHandle_t) * size);
    if (e == cudaSuccess)
        e = cudaMemcpyAsync(hbuf + sizeof(own) * rank, &own, sizeof(own), cudaMemcpyHostToDevice, st);
    int rc = e == cudaSuccess ? LQ_OK : cuda_fail(e, "exchange region export");
    if (!rc) {
        const ncclResult_t r = nccl()->all_gather(hbuf + sizeof(own) * rank, hbuf, sizeof(own), ncclChar,
                                                  static_cast<ncclComm_t>(t->comm), st);
        if (r != ncclSuccess) rc = lq_fail(LQ_ECUDA, "exchange handle all-gather: %s", nccl()->error_string(r));
    }
    std::vector<cudaIpcMemHandle_t> all(size);
    if (!rc) {
        e = cudaMemcpyAsync(all.data(), hbuf, sizeof(own) * size, cudaMemcpyDeviceToHost, st);
        if (e == cudaSuccess) e = cudaStreamSynchronize(st);
        if (e != cudaSuccess) rc = cuda_fail(e, "exchange handle all-gather");
    }
    for (int p = 0; p < size && !rc; ++p) {
        if (p == rank) {
            t->xr_peer[p] = t->xr;
            continue;
        }
        e = cudaIpcOpenMemHandle(&t->xr_peer[p], all[p], cudaIpcMemLazyEnablePeerAccess);
        if (e != cudaSuccess) rc = cuda_fail(e, "mapping a peer's exchange region");
    }
    if (hbuf) cudaFree(hbuf);
    if (st) cudaStreamDestroy(st);
    return rc;
}

// Undo xr_setup.  Collective: one NCCL all-reduce first, so that every
// process has finished every step (whose kernels read the peers' regions)
// before any region is unmapped or freed.
void xr_teardown(Transformer* t) {
    if (!t->xr) return;
    bool synced = false;
    if (t->comm && t->stream) {
        float* one = nullptr;
        if (cudaMalloc(&one, sizeof(float)) == cudaSuccess) {
            synced = nccl()->all_reduce(one, one, 1, ncclFloat, ncclSum, static_cast<ncclComm_t>(t->comm), t->stream) ==
                         ncclSuccess &&
                     cudaStreamSynchronize(t->stream) == cudaSuccess;
            cudaFree(one);
        }
    }
    for (int p = 0; p < t->tp_size && p < lq::kTpMax; ++p)
        if (t->xr_peer[p] && p != t->tp_rank) cudaIpcCloseMemHandle(t->xr_peer[p]);
    for (void*& q : t->xr_peer) q = nullptr;
    // without the barrier a peer may still read this region: leave it allocated
    if (synced) cudaFree(t->xr);
    t->xr = nullptr;
}

int tp_join(Transformer* t, int rank, int size, const void* id) {
    t->tp = true;
    t->tp_rank = rank;
    t->tp_size = size;
    if (size == 1) return LQ_OK;
    const Nccl* f = nccl();
    if (!f) return lq_fail(LQ_EUNSUPPORTED, "tensor parallelism needs NCCL (libnccl.so.2), which could not be loaded");
    ncclUniqueId uid;
    memcpy(&uid, id, sizeof(uid));
    ncclComm_t comm = nullptr;
    const ncclResult_t r = f->comm_init_rank(&comm, size, uid, rank);
    if (r != ncclSuccess) return lq_fail(LQ_ECUDA, "NCCL communicator (rank %d of %d): %s", rank, size, f->error_string(r));
    t->comm = comm;
    if (const char* m = getenv("LQ_TP_ALLREDUCE")) t->tp_nccl = strcmp(m, "nccl") == 0;
    if (const char* w = getenv("LQ_TP_WAIT_MS")) {
        const long ms = atol(w);
        if (ms > 0) t->tp_wait_ns = (uint64_t)ms * 1000000ull;
    }
    return t->tp_nccl ? LQ_OK : xr_setup(t);
}

// Read the checkpoint's tensors (mmap'd at data + hb) into t, this process's
// share of each under tensor parallelism.
int upload_weights(Transformer* t, const uint8_t* data, size_t hb, int shared) {
    const Config& c = t->c;
    const int kind = t->kind, gs = t->gs, L = c.n_layers;
    LqTensorDesc td[LQ_NT];
    lq_tensor_table(&c, td);
    const uint8_t* p = data + hb;
    int rc = LQ_OK;
    for (int i = 0; i < LQ_NT && !rc; ++i) {
        const LqTensorDesc& d = td[i];
        cudaError_t e = cudaSuccess;
        if (d.id == LQ_T_WCLS && shared) {
            // extension: quantize the fp32 embedding as the classifier
            rc = alloc_q(t->wcls, d.rows, d.cols, gs, kind);
            if (rc) break;
            std::vector<uint8_t> q((size_t)(d.rows * rbytes(d.cols, kind)));
            std::vector<float> sc((size_t)(d.rows * (d.cols / gs)));
            std::vector<float> emb((size_t)(d.rows * d.cols));
            cudaMemcpy(emb.data(), t->emb, emb.size() * 4, cudaMemcpyDeviceToHost);
            lq_quantize_rows_host(emb.data(), d.rows, d.cols, gs, kind, q.data(), sc.data());
            e = cudaMemcpy(t->wcls.q, q.data(), q.size(), cudaMemcpyHostToDevice);
            if (e == cudaSuccess) e = cudaMemcpy(t->wcls.s, sc.data(), sc.size() * 4, cudaMemcpyHostToDevice);
        } else if (d.quantized) {
            QW* w = weight_by_id(t, d.id);
            int64_t rows, cols;
            tp_local_shape(t, d, &rows, &cols);
            rc = alloc_q(*w, rows, cols, gs, kind);
            if (rc) break;
            const size_t rbf = (size_t)rbytes(d.cols, kind), ngf = (size_t)(d.cols / gs);
            const size_t qb = (size_t)d.rows * rbf, sb = (size_t)d.rows * ngf * 4;
            const int split = t->tp ? tp_split(d.id) : 0;
            if (split == 0) {
                e = cudaMemcpy(w->q, p, qb, cudaMemcpyHostToDevice);
                if (e == cudaSuccess) e = cudaMemcpy(w->s, p + qb, sb, cudaMemcpyHostToDevice);
            } else {
                const int64_t rl = d.rows / L;  // rows of one layer
                for (int l = 0; l < L && e == cudaSuccess; ++l) {
                    if (split == 1) {
                        // this process's rows of layer l
                        const int64_t r0 = l * rl + t->tp_rank * (rl / t->tp_size), nr = rl / t->tp_size;
                        e = cudaMemcpy(w->q + (size_t)l * nr * rbf, p + (size_t)r0 * rbf, (size_t)nr * rbf,
                                       cudaMemcpyHostToDevice);
                        if (e == cudaSuccess)
                            e = cudaMemcpy(w->s + (size_t)l * nr * ngf, p + qb + (size_t)r0 * ngf * 4, (size_t)nr * ngf * 4,
                                           cudaMemcpyHostToDevice);
                    } else {
                        // this process's columns of every row of layer l (whole groups)
                        const size_t rbl = (size_t)rbytes(cols, kind), ngl = (size_t)(cols / gs);
                        const size_t c0b = (size_t)rbytes(t->tp_rank * cols, kind), c0g = (size_t)(t->tp_rank * cols / gs);
                        e = cudaMemcpy2D(w->q + (size_t)l * rl * rbl, rbl, p + (size_t)l * rl * rbf + c0b, rbf, rbl,
                                         (size_t)rl, cudaMemcpyHostToDevice);
                        if (e == cudaSuccess)
                            e = cudaMemcpy2D(w->s + (size_t)l * rl * ngl, ngl * 4, p + qb + ((size_t)l * rl * ngf + c0g) * 4,
                                             ngf * 4, ngl * 4, (size_t)rl, cudaMemcpyHostToDevice);
                    }
                }
            }
            p += qb + sb;
        } else {
            float** f = f32_by_id(t, d.id);
            const size_t n = (size_t)(d.rows * d.cols);
            rc = dalloc(f, n);
            if (rc) break;
            e = cudaMemcpy(*f, p, n * 4, cudaMemcpyHostToDevice);
            p += n * 4;
        }
        if (!rc && e != cudaSuccess) rc = cuda_fail(e, "weight upload");
    }
    return rc;
}

int build_file(Transformer** out, const char* path, int max_seq_len, bool tp, int rank, int size, const void* id) {
    if (!out || !path) return lq_fail(LQ_EINVAL, "build_transformer: null argument");
    *out = nullptr;
    int fd = open(path, O_RDONLY);
    if (fd < 0) return lq_fail(LQ_EIO, "couldn't open file %s", path);
    struct stat st;
    fstat(fd, &st);
    const size_t size_b = (size_t)st.st_size;
    const uint8_t* data = size_b ? (const uint8_t*)mmap(nullptr, size_b, PROT_READ, MAP_PRIVATE, fd, 0)
                                 : (const uint8_t*)MAP_FAILED;
    close(fd);
    if (data == MAP_FAILED) return lq_fail(LQ_EIO, "mmap failed: %s", path);
    Config c;
    int kind, gs, shared;
    size_t hb;
    int rc = lq_parse_header(data, size_b, &c, &kind, &gs, &shared, &hb);
    if (!rc) rc = check_config(&c, gs, tp ? size : 1);
    LqTensorDesc td[LQ_NT];
    if (!rc) rc = lq_tensor_table(&c, td);
    // size check (the reference does none: runq.c:269-277)
    if (!rc) {
        size_t need = hb;
        for (int i = 0; i < LQ_NT; ++i) {
            if (td[i].id == LQ_T_WCLS && shared) break;
            need += td[i].quantized ? (size_t)lq_qtensor_bytes(td[i].rows, td[i].cols, gs, kind)
                                    : (size_t)(td[i].rows * td[i].cols * 4);
        }
        if (need > size_b) rc = lq_fail(LQ_EFORMAT, "truncated checkpoint: %zu bytes, need %zu", size_b, need);
    }
    Transformer* t = nullptr;
    if (!rc) {
        t = new_transformer(&c, kind, gs, max_seq_len, 1);
        t->shared = shared;
        if (tp) rc = tp_join(t, rank, size, id);
        if (!rc) rc = upload_weights(t, data, hb, shared);
        if (!rc) rc = alloc_state(t);
    }
    munmap((void*)data, size_b);
    if (rc) {
        if (t) free_transformer(t);
        return rc;
    }
    *out = t;
    return LQ_OK;
}

int build_random(Transformer** out, const Config* cfg, int kind, int gs, uint64_t seed, int max_seq_len, bool tp,
                 int rank, int size, const void* id) {
    if (!out || !cfg) return lq_fail(LQ_EINVAL, "build_transformer_random: null argument");
    *out = nullptr;
    if (kind != LQ_KIND_INT8 && kind != LQ_KIND_INT4) return lq_fail(LQ_EINVAL, "kind must be INT8 or INT4");
    if (!(gs == 32 || gs == 64 || gs == 128 || gs == 256)) return lq_fail(LQ_EUNSUPPORTED, "group size %d", gs);
    int rc = check_config(cfg, gs, tp ? size : 1);
    if (rc) return rc;
    LqTensorDesc td[LQ_NT];
    lq_tensor_table(cfg, td);
    Transformer* t = new_transformer(cfg, kind, gs, max_seq_len, 1);
    if (tp) rc = tp_join(t, rank, size, id);
    const float std = 0.02f;
    const int L = cfg->n_layers;
    for (int i = 0; i < LQ_NT && !rc; ++i) {
        const LqTensorDesc& d = td[i];
        cudaError_t e = cudaSuccess;
        if (d.quantized) {
            QW* w = weight_by_id(t, d.id);
            int64_t rows, cols;
            tp_local_shape(t, d, &rows, &cols);
            rc = alloc_q(*w, rows, cols, gs, kind);
            if (rc) break;
            const int split = t->tp ? tp_split(d.id) : 0;
            if (split == 0) {
                e = synth_quant_launch(w->q, w->s, d.rows, d.cols, gs, kind, seed, d.id, std, 0, nullptr);
            } else {
                // the generator is indexed by (row, column) of the whole tensor: each
                // process generates exactly its share of the unsplit model's weights
                const int64_t rl = d.rows / L, nr = rows / L;
                const size_t rbl = (size_t)rbytes(cols, kind), ngl = (size_t)(cols / gs);
                for (int l = 0; l < L && e == cudaSuccess; ++l) {
                    if (split == 1)
                        e = synth_quant_launch(w->q + (size_t)l * nr * rbl, w->s + (size_t)l * nr * ngl, nr, cols, gs, kind,
                                               seed, d.id, std, l * rl + t->tp_rank * nr, nullptr);
                    else
                        e = synth_quant_cols_launch(w->q + (size_t)l * rl * rbl, w->s + (size_t)l * rl * ngl, rl, cols,
                                                    d.cols, t->tp_rank * cols, gs, kind, seed, d.id, std, l * rl,
                                                    nullptr);
                }
            }
        } else {
            float** f = f32_by_id(t, d.id);
            const int64_t n = d.rows * d.cols;
            rc = dalloc(f, (size_t)n);
            if (rc) break;
            const int ones = d.id != LQ_T_EMB;
            e = synth_f32_launch(*f, n, seed, d.id, std, ones, nullptr);
        }
        if (e != cudaSuccess) rc = cuda_fail(e, "random init");
    }
    if (!rc) {
        cudaError_t e = cudaDeviceSynchronize();
        if (e != cudaSuccess) rc = cuda_fail(e, "random init");
    }
    if (!rc) rc = alloc_state(t);
    if (rc) {
        free_transformer(t);
        return rc;
    }
    *out = t;
    return LQ_OK;
}

}  // namespace

extern "C" {

int build_transformer(Transformer** out, const char* path, int max_seq_len) {
    return build_file(out, path, max_seq_len, false, 0, 1, nullptr);
}

int build_transformer_random(Transformer** out, const Config* cfg, int kind, int gs, uint64_t seed,
                             int max_seq_len) {
    return build_random(out, cfg, kind, gs, seed, max_seq_len, false, 0, 1, nullptr);
}

int lq_tp_unique_id(void* id) {
    if (!id) return lq_fail(LQ_EINVAL, "lq_tp_unique_id: null argument");
    const Nccl* f = nccl();
    if (!f) return lq_fail(LQ_EUNSUPPORTED, "tensor parallelism needs NCCL (libnccl.so.2), which could not be loaded");
    ncclUniqueId uid;
    const ncclResult_t r = f->get_unique_id(&uid);
    if (r != ncclSuccess) return lq_fail(LQ_ECUDA, "ncclGetUniqueId: %s", f->error_string(r));
    memcpy(id, &uid, sizeof(uid));
    return LQ_OK;
}

static int tp_args_ok(int rank, int size, const void* id) {
    if (size < 1 || size > lq::kTpMax || rank < 0 || rank >= size)
        return lq_fail(LQ_EINVAL, "tp rank %d of %d (at most %d processes)", rank, size, lq::kTpMax);
    if (size > 1 && !id) return lq_fail(LQ_EINVAL, "tensor parallelism over %d GPUs needs the group id", size);
    return LQ_OK;
}

int build_transformer_tp(Transformer** out, const char* path, int max_seq_len, int tp_rank, int tp_size,
                         const void* id) {
    int rc = tp_args_ok(tp_rank, tp_size, id);
    return rc ? rc : build_file(out, path, max_seq_len, true, tp_rank, tp_size, id);
}

int build_transformer_random_tp(Transformer** out, const Config* cfg, int kind, int gs, uint64_t seed,
                                int max_seq_len, int tp_rank, int tp_size, const void* id) {
    int rc = tp_args_ok(tp_rank, tp_size, id);
    return rc ? rc : build_random(out, cfg, kind, gs, seed, max_seq_len, true, tp_rank, tp_size, id);
}

float* forward(Transformer* t, int token, int pos) {
    if (!t) {
        lq_fail(LQ_EINVAL, "forward: null transformer");
        return nullptr;
    }
    if (run_step(t, &token, &pos, 1, true, false) != LQ_OK) return nullptr;
    return t->h_logits;
}

float* forward_prompt(Transformer* t, const int* tokens, int n_tokens, int start_pos) {
    if (!t || !tokens) {
        lq_fail(LQ_EINVAL, "forward_prompt: null argument");
        return nullptr;
    }
    if (run_prompt(t, tokens, n_tokens, start_pos) != LQ_OK) return nullptr;
    return t->h_logits;
}

int forward_argmax(Transformer* t, int token, int pos, int* next_token) {
    if (!t || !next_token) return lq_fail(LQ_EINVAL, "forward_argmax: null argument");
    int rc = run_step(t, &token, &pos, 1, false, true);
    if (rc) return rc;
    *next_token = t->h_next[0];
    return LQ_OK;
}

void free_transformer(Transformer* t) {
    if (!t) return;
    free_state(t);  // the captured graph (which holds the all-reduces) goes before the communicator
    if (t->ktr) cudaFree(t->ktr);
    free(t->ktr_kind);
    xr_teardown(t);
    if (t->comm && nccl()) nccl()->comm_destroy(static_cast<ncclComm_t>(t->comm));
    t->comm = nullptr;
    QW* ws[] = {&t->wq, &t->wk, &t->wv, &t->wo, &t->w1, &t->w2, &t->w3, &t->wcls};
    for (QW* w : ws) {
        cudaFree(w->q);
        cudaFree(w->s);
    }
    void* bufs[] = {t->emb, t->rms_att, t->rms_ffn, t->rms_final};
    for (void* b : bufs) cudaFree(b);
    if (t->stream) cudaStreamDestroy(t->stream);
    delete t;
}

int transformer_reserve_batch(Transformer* t, int max_batch) {
    if (!t) return lq_fail(LQ_EINVAL, "transformer_reserve_batch: null transformer");
    if (max_batch < 1 || max_batch > 1024) return lq_fail(LQ_EINVAL, "max_batch %d out of range [1, 1024]", max_batch);
    free_state(t);
    t->max_batch = max_batch;
    cudaGetLastError();
    int rc = alloc_state(t);
    // the peer all-reduce's exchange region holds a slot row per activation
    // row: set it up again (collectively: every process makes this call with
    // the same arguments) when the new activation rows exceed it
    if (!rc && t->xr && act_rows(t) > t->xr_rows) {
        xr_teardown(t);
        rc = xr_setup(t);
    }
    return rc;
}

float* forward_batch(Transformer* t, const int* tokens, const int* pos, int batch) {
    if (!t || !tokens || !pos) {
        lq_fail(LQ_EINVAL, "forward_batch: null argument");
        return nullptr;
    }
    if (run_step(t, tokens, pos, batch, true, false) != LQ_OK) return nullptr;
    return t->h_logits;
}

int forward_batch_argmax(Transformer* t, const int* tokens, const int* pos, int batch, int* next_tokens) {
    if (!t || !tokens || !pos || !next_tokens) return lq_fail(LQ_EINVAL, "forward_batch_argmax: null argument");
    int rc = run_step(t, tokens, pos, batch, false, true);
    if (rc) return rc;
    for (int b = 0; b < batch; ++b) next_tokens[b] = t->h_next[b];
    return LQ_OK;
}

int lq_tp_wait_selftest(int tp_size, int wait_us, double* first_ms, double* second_ms) {
    if (tp_size < 2 || tp_size > lq::kTpMax || wait_us < 1 || wait_us > 10000000)
        return lq_fail(LQ_EINVAL, "lq_tp_wait_selftest: tp_size in [2, %d], wait_us in [1, 1e7]", lq::kTpMax);
    // rank 0 of a tp_size group whose other members never push: its own
    // counters and slot live on this device, the other ranks' words stay 0
    const int n = 256, gs = 64, ng = n / gs;
    const size_t slot = (size_t)tp_size * n * sizeof(uint64_t);
    const size_t bytes = lq::kXrCountersBytes + slot + 4 * (size_t)n * sizeof(float) + n + 2 * ng * 4 + 256;
    char* buf = nullptr;
    cudaStream_t st = nullptr;
    cudaEvent_t ev[3] = {};
    cudaError_t e = cudaMalloc(&buf, bytes);
    if (e == cudaSuccess) e = cudaMemset(buf, 0, bytes);
    if (e == cudaSuccess) e = cudaStreamCreateWithFlags(&st, cudaStreamNonBlocking);
    for (int i = 0; i < 3 && e == cudaSuccess; ++i) e = cudaEventCreate(&ev[i]);
    int rc = LQ_OK;
    if (e == cudaSuccess) {
        char* p = buf + lq::kXrCountersBytes + slot;
        float* x = reinterpret_cast<float*>(p);
        float* w = x + n;
        float* xo = w + n;
        std::vector<float> ones(n, 1.0f);
        e = cudaMemcpy(w, ones.data(), n * sizeof(float), cudaMemcpyHostToDevice);
        PeerAddArgs a{};
        a.q.mode = IN_ADD_RMSNORM;
        a.q.n = n;
        a.q.gs = gs;
        a.q.nb = 1;
        a.q.x = x;
        a.q.rms_w = w;
        a.q.x_out = xo;
        a.q.xq = reinterpret_cast<int8_t*>(xo + 2 * n);
        a.q.xs = reinterpret_cast<float*>(reinterpret_cast<char*>(a.q.xq) + n);
        a.q.xsum = reinterpret_cast<int*>(a.q.xs + ng);
        a.err = reinterpret_cast<int*>(a.q.xsum + ng);
        a.counters = reinterpret_cast<uint32_t*>(buf);
        a.slot = reinterpret_cast<const uint64_t*>(buf + lq::kXrCountersBytes);
        a.ll_rows = 1;
        a.tp_rank = 0;
        a.tp_size = tp_size;
        a.wait_ns = (uint64_t)wait_us * 1000ull;
        if (e == cudaSuccess) e = cudaEventRecord(ev[0], st);
        if (e == cudaSuccess) e = peer_add_quant_launch(a, st, false);
        if (e == cudaSuccess) e = cudaEventRecord(ev[1], st);
        if (e == cudaSuccess) e = peer_add_quant_launch(a, st, false);  // the step's next call: no second wait
        if (e == cudaSuccess) e = cudaEventRecord(ev[2], st);
        if (e == cudaSuccess) e = cudaStreamSynchronize(st);
        float t1 = 0.0f, t2 = 0.0f;
        if (e == cudaSuccess) e = cudaEventElapsedTime(&t1, ev[0], ev[1]);
        if (e == cudaSuccess) e = cudaEventElapsedTime(&t2, ev[1], ev[2]);
        if (first_ms) *first_ms = t1;
        if (second_ms) *second_ms = t2;
        if (e == cudaSuccess) {
            int h = 0;
            e = cudaMemcpy(&h, a.err, sizeof(int), cudaMemcpyDeviceToHost);
            if (e == cudaSuccess)
                rc = h ? lq_fail(LQ_ETIMEOUT, "device-side wait gave up (code 0x%x)", h)
                       : lq_fail(LQ_EINVAL, "lq_tp_wait_selftest: the wait did not give up");
        }
    }
    if (e != cudaSuccess) rc = cuda_fail(e, "lq_tp_wait_selftest");
    for (cudaEvent_t x : ev)
        if (x) cudaEventDestroy(x);
    if (st) cudaStreamDestroy(st);
    if (buf) cudaFree(buf);
    return rc;
}

int transformer_trace(Transformer* t, int enable) {
    if (!t) return lq_fail(LQ_EINVAL, "transformer_trace: null transformer");
    if (t->stream) cudaStreamSynchronize(t->stream);
    // the captured graphs hold the trace pointers: capture again at the next step
    if (t->exec) cudaGraphExecDestroy(t->exec);
    if (t->graph) cudaGraphDestroy(t->graph);
    if (t->pexec) cudaGraphExecDestroy(t->pexec);
    if (t->pgraph) cudaGraphDestroy(t->pgraph);
    t->exec = nullptr;
    t->graph = nullptr;
    t->graph_batch = 0;
    t->pexec = nullptr;
    t->pgraph = nullptr;
    t->pgraph_rows = 0;
    if (t->ktr) cudaFree(t->ktr);
    free(t->ktr_kind);
    t->ktr = nullptr;
    t->ktr_kind = nullptr;
    t->ktr_cap = t->ktr_n = 0;
    if (!enable) return LQ_OK;
    const int cap = 16384;
    cudaError_t e = cudaMalloc(&t->ktr, 3 * kKtSlots * sizeof(uint64_t) * cap);
    if (e == cudaSuccess) e = cudaMemset(t->ktr, 0xFF, 3 * kKtSlots * sizeof(uint64_t) * cap);
    t->ktr_kind = static_cast<int*>(calloc(cap, sizeof(int)));
    if (e != cudaSuccess || !t->ktr_kind) {
        if (t->ktr) cudaFree(t->ktr);
        free(t->ktr_kind);
        t->ktr = nullptr;
        t->ktr_kind = nullptr;
        return e != cudaSuccess ? cuda_fail(e, "transformer_trace") : lq_fail(LQ_ENOMEM, "transformer_trace");
    }
    t->ktr_cap = cap;
    return LQ_OK;
}

int transformer_trace_read(Transformer* t, int max_kernels, int* kinds, uint64_t* stamps, int* count) {
    if (!t || !count) return lq_fail(LQ_EINVAL, "transformer_trace_read: null argument");
    if (!t->ktr) return lq_fail(LQ_EINVAL, "transformer_trace_read: tracing is off (transformer_trace)");
    const int n = t->ktr_n < max_kernels ? t->ktr_n : max_kernels;
    *count = t->ktr_n;
    if (n <= 0) return LQ_OK;
    std::vector<uint64_t> raw((size_t)3 * kKtSlots * n);
    cudaError_t e = cudaStreamSynchronize(t->stream);
    if (e == cudaSuccess) e = cudaMemcpy(raw.data(), t->ktr, raw.size() * sizeof(uint64_t), cudaMemcpyDeviceToHost);
    if (e != cudaSuccess) return cuda_fail(e, "transformer_trace_read");
    for (int i = 0; i < n; ++i) {
        if (kinds) kinds[i] = t->ktr_kind[i];
        if (!stamps) continue;
        // reduce the per-slot stamps: earliest start and wait, latest end
        // (ends are stored complemented, so the latest end is the smallest)
        const uint64_t* k = raw.data() + (size_t)3 * kKtSlots * i;
        uint64_t s0 = ~0ull, s1 = ~0ull, s2 = ~0ull;
        for (int j = 0; j < kKtSlots; ++j) {
            s0 = k[j] < s0 ? k[j] : s0;
            s1 = k[kKtSlots + j] < s1 ? k[kKtSlots + j] : s1;
            s2 = k[2 * kKtSlots + j] < s2 ? k[2 * kKtSlots + j] : s2;
        }
        stamps[3 * i] = s0;
        stamps[3 * i + 1] = s1;
        stamps[3 * i + 2] = s2 == ~0ull ? ~0ull : ~s2;
    }
    return LQ_OK;
}

int transformer_config(const Transformer* t, Config* cfg, int* kind, int* group_size) {
    if (!t) return lq_fail(LQ_EINVAL, "transformer_config: null transformer");
    if (cfg) *cfg = t->c;
    if (kind) *kind = t->kind;
    if (group_size) *group_size = t->gs;
    return LQ_OK;
}

}  // extern "C"
