// Transformer state (C++ only; opaque in the C ABI).
#pragma once
#include <cstdint>
#include <cuda.h>
#include <cuda_runtime.h>

#include "lq_host.h"

namespace lq {

struct QW {
    uint8_t* q = nullptr;  // device, stacked over layers [L*rows, row_bytes]
    float* s = nullptr;    // device, [L*rows, cols/gs]
    int64_t rows = 0, cols = 0;
};

int forward_launch(Transformer* t, int batch);
// the next kernel's step-trace stamps (null when tracing is off); records its kind
uint64_t* kt_next(Transformer* t, int kind);
int run_step(Transformer* t, const int* tokens, const int* pos, int batch, bool want_logits, bool want_next);
int run_prompt(Transformer* t, const int* tokens, int n, int start);
int kernels_per_step(const Transformer* t, int batch);

}  // namespace lq

struct Transformer {
    Config c{};
    int kind = 0, gs = 0, shared = 0;
    int dev = 0, num_sms = 148;
    int max_seq = 0, max_batch = 1;
    int head_size = 0, kv_dim = 0, kv_mul = 1, max_splits = 1;
    cudaStream_t stream = nullptr;
    // weights
    float *emb = nullptr, *rms_att = nullptr, *rms_ffn = nullptr, *rms_final = nullptr;
    lq::QW wq, wk, wv, wo, w1, w2, w3, wcls;
    // activations and caches (device); leading dimension max_batch
    float *x = nullptr, *q = nullptr, *att = nullptr, *h1 = nullptr, *h3 = nullptr, *logits = nullptr;
    int8_t* xq = nullptr;  // quantized activation feeding the next GEMV
    float* xqs = nullptr;
    int* xqsum = nullptr;
    float *kc = nullptr, *vc = nullptr;  // [B][L][kv_heads][max_seq][head_size]
    alignas(64) CUtensorMap kmap{};      // kc as rows of head_size floats, for the attention kernel
    float* part = nullptr;               // attention partials [B][heads][max_splits][head_size + 4]
    int* meta = nullptr;                 // [B][token, pos]
    int* next = nullptr;                 // [B] argmax
    int* err = nullptr;                  // device error word
    float2* rope = nullptr;              // [max_seq][head_size/2] cos/sin table
    // tensor parallelism (Megatron split): this process's share of the heads and hidden rows
    int tp_rank = 0, tp_size = 1;
    bool tp = false;                     // TP step: partial products, all-reduce, residual add in the quantizer
    void* comm = nullptr;                // NCCL communicator (tp_size > 1)
    int nh_l = 0, nkv_l = 0, dq_l = 0, hid_l = 0;  // local query heads, kv heads, q width, hidden rows
    float *x2 = nullptr, *ybuf = nullptr;  // second residual buffer; all-reduced partial [B][dim]
    // peer all-reduce (tp_size > 1): this process's exchange region and every
    // process's region as mapped here (rank order, own one included); with
    // tp_nccl set (LQ_TP_ALLREDUCE=nccl) the step all-reduces ybuf with NCCL
    void* xr = nullptr;
    int xr_rows = 0;                     // slot rows of the exchange region (activation rows at set-up)
    void* xr_peer[8] = {};
    bool tp_nccl = false;
    uint64_t tp_wait_ns = 0;             // peer flag wait limit (LQ_TP_WAIT_MS; 0 = the 2 s default)
    // tensor-core GEMM path (steps of mma_min or more sequences)
    int mma_min = 16;
    int xs_ld = 0;                       // max_batch rounded up to 64 (xs_t: a [groups][64] table per 64 rows)
    float* xs_t = nullptr;               // activation scales transposed, per chunk of 64 rows
    float* qg_part = nullptr;            // stream-K partials
    int* qg_cnt = nullptr;               // per-tile arrival counters
    // pinned host mirrors
    float* h_logits = nullptr;
    int *h_meta = nullptr, *h_next = nullptr, *h_err = nullptr;
    // step trace (transformer_trace): three stamps per kernel of the step and the kernels' kinds
    uint64_t* ktr = nullptr;
    int ktr_cap = 0, ktr_n = 0;
    int* ktr_kind = nullptr;
    // prompt steps (forward_prompt): every row is a position of sequence
    // prompt_seq (-1 while capturing the decode step); their own graph
    int prompt_seq = -1;
    cudaGraph_t pgraph = nullptr;
    cudaGraphExec_t pexec = nullptr;
    int pgraph_rows = 0;
    // graph
    cudaGraph_t graph = nullptr;
    cudaGraphExec_t exec = nullptr;
    int graph_batch = 0;
};
