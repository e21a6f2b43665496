// Kernel argument blocks and launchers (host-visible, C++ only).
#pragma once
#include <cstdint>
#include <cuda_runtime.h>

namespace lq {

// What the GEMV does with a finished row value v (per segment).
enum Epilogue : int {
    EPI_STORE = 0,        // y[r] = v
    EPI_ADD = 1,          // y[r] += v            (residual stream)
    EPI_ROPE_Q = 2,       // rotary pair (r, r+1) of the query, stored to y
    EPI_ROPE_KCACHE = 3,  // rotary pair of the key, stored to the K cache at pos
    EPI_VCACHE = 4,       // value stored to the V cache at pos
    EPI_SWIGLU = 5,       // paired tensors: y[r] = silu(v1) * v3 (runq.c:405-410)
    EPI_PUSH = 6,         // tensor-parallel partial, pushed to every process's exchange slot (PeerAddArgs)
};

// Where the int8 activation comes from (the GEMV prologue builds it in
// shared memory; every CTA computes the identical quantization).
enum InputMode : int {
    IN_QUANT = 0,        // pre-quantized xq/xs (the C-ABI matmul)
    IN_F32 = 1,          // fp32 x, quantized in the prologue
    IN_RMSNORM = 2,      // rmsnorm(x) * w, then quantized
    IN_RMSNORM_EMB = 3,  // x = emb[token] (CTA 0 also writes it to x_out), then as IN_RMSNORM
    IN_ADD_RMSNORM = 4,  // x = x + y (CTA 0 also writes it to x_out), then as IN_RMSNORM (activation quantizer only)
};

constexpr int kTpMax = 8;  // tensor-parallel processes

struct GemvSeg {
    const uint8_t* wq;  // packed weights [rows, row_bytes]
    const float* ws;    // group scales [rows, cols / gs]
    float* y;           // destination (meaning depends on epi)
    int rows;
    int epi;
    const uint8_t* wq2;  // EPI_SWIGLU: the second tensor (w3), same shape
    const float* ws2;
};

constexpr int kMaxSegs = 3;
constexpr int kConsumerWarps = 8;
constexpr int kGemvThreads = kConsumerWarps * 32;

struct GemvArgs {
    GemvSeg seg[kMaxSegs];
    int nseg;
    int cols;        // n (input length)
    int gs;          // group size: 32, 64, 128 or 256
    int nb;          // activation rows (batch); template NB must equal it
    int nvalid;      // rows b < nvalid are stored; rows nvalid..nb-1 are padding (0 = all)
    // input
    int in_mode;
    const int8_t* xq;  // IN_QUANT [nb, cols]
    const float* xs;   // IN_QUANT [nb, cols/gs]
    const int* xsum_in;  // IN_QUANT, optional: group sums of xq [nb, cols/gs] (computed when null)
    const float* xf;   // fp32 source [nb, cols] (IN_F32, IN_RMSNORM)
    const float* rms_w;
    const float* emb;  // IN_RMSNORM_EMB table [vocab, cols]
    float* x_out;      // IN_RMSNORM_EMB residual stream init
    int y_stride;      // elements between batch rows of y (EPI_STORE / EPI_ADD)
    // decode state
    const int* meta;   // per batch row: [token, pos]
    const float2* rope;  // [max_seq][head_size/2] (cos, sin) of pos * freq
    int head_size;
    float* kcache;     // layer base, [kv_heads][max_seq][head_size] per sequence
    float* vcache;
    int max_seq;
    int64_t kv_seq_stride;  // elements between sequences' caches
    int* err;
    uint64_t* trace;  // optional per-CTA phase timestamps (globaltimer ns), [grid][4]; null = off
    uint64_t* kt;     // optional step-trace stamps of this launch (lq_device.cuh kt_*); null = off
    // EPI_PUSH: the slot of every process (rank order), this process's call
    // counter, and the slot geometry (row of batch row b: ll_row0 + b)
    uint64_t* ll[kTpMax];
    const uint32_t* ll_call;
    int ll_tp, ll_rank, ll_rows, ll_row0;
    // schedule (filled by the planner)
    int split;       // 0: stages of whole rows; 1: stages are slices of one row
    int stage_rows;  // rows per stage (whole-row mode)
    int slice_bytes; // slice size (slice mode)
    int nstages;
    int wcap, scap;  // per-stage weight / scale capacity in bytes (both tensors when paired)
    int x_bytes;     // shared-memory bytes for the staged activation
    int paired;      // segments carry a second tensor (EPI_SWIGLU)
};

// Tensor-core GEMM (tcgen05.mma kind::i8) for 1..64 activation rows:
// segments and epilogues as for the GEMV; a.xq = int8 activation of
// a.nvalid rows of a.cols bytes (the kernel pads to qgemm_npad(rows) with
// zero rows); xs_t = activation scales transposed [cols/gs][xs_ld] (1/16 of
// them for INT4 weights), xs_ld >= qgemm_npad(rows); part =
// qgemm_part_floats(num_sms) floats of scratch; cnt = per-tile arrival
// counters, zero-initialised, left zero.
bool qgemm_ok(const GemvArgs& a, int kind, int rows);
int qgemm_npad(int rows);
size_t qgemm_part_floats(int num_sms);
int qgemm_max_tiles(const GemvArgs& a);
cudaError_t qgemm_launch(const GemvArgs& a, int kind, const float* xs_t, int xs_ld, float* part, int* cnt,
                         cudaStream_t st, bool pdl, int num_sms);
// xs [rows][ng] -> xs_t [ng][ld] times mul (columns >= rows zero)
cudaError_t qgemm_scales_launch(const float* xs, int rows, int ng, int ld, float mul, float* xs_t, cudaStream_t st);

// Activation quantization kernel (quantize_act, v1-int8-vnni/runq.c:117-139,
// optionally after rmsnorm, runq.c:294-305): writes int8 xq [nb, n] in
// natural order, fp32 scales xs and int32 group sums xsum [nb, n/gs].
struct ActQuantArgs {
    int mode;          // IN_F32, IN_RMSNORM or IN_RMSNORM_EMB
    int n, gs, nb;
    const float* x;    // [nb, n] (IN_F32 / IN_RMSNORM / IN_ADD_RMSNORM)
    const float* y;    // [nb, n] IN_ADD_RMSNORM: the (all-reduced) output added to the residual x
    const float* rms_w;
    const float* emb;  // IN_RMSNORM_EMB: x = emb[meta[2b]]
    const int* meta;
    float* x_out;      // IN_RMSNORM_EMB: copy of the embedding row (residual stream)
    int8_t* xq;
    float* xs;
    int* xsum;
    // optional (tensor-core GEMM input): scales transposed per chunk of 64
    // rows, chunk c at xs_t + c * (n/gs) * 64 as [n/gs][npad_c] with npad_c =
    // 64 for the first xs_nfull chunks and xs_npad_last for the last one;
    // multiplied by xs_t_mul (1, or 1/16 for int4 weights held as 16*q)
    float* xs_t;
    int xs_nfull, xs_npad_last;
    float xs_t_mul;
    uint64_t* kt;      // optional step-trace stamps of this launch; null = off
};
cudaError_t act_quant_launch(const ActQuantArgs& a, cudaStream_t st, bool pdl);

// The quantizer in front of the wo product: merges the attention kernel's
// per-chunk partials of every head (or, for a single chunk, reads its
// normalised output q.x) and quantizes the row.  q.n = heads * head_size.
struct AttnQuantArgs {
    ActQuantArgs q;       // mode ignored; x = the attention output [nb][n]
    const float* part;    // [nb][n / head_size][max_splits][head_size + 4]: m, l, -, -, o
    int head_size, max_splits;
};
cudaError_t attn_quant_launch(const AttnQuantArgs& a, cudaStream_t st, bool pdl);

// Tensor-parallel all-reduce fused into the quantizer that follows a wo / w2
// product (low-latency protocol: every value travels with its call number).
// Each process owns an exchange region in its own device memory, mapped by
// every peer (CUDA IPC): counters[2] (calls done, CTAs arrived), then two
// slots of [tp][ll_rows][dim] 64-bit words.  The wo (slot 0) and w2 (slot 1)
// products push each partial value v of row b, column r as the word
// (call << 32) | bits(v) into row (own rank, b) of that slot of EVERY
// process (EPI_PUSH, relaxed system-scope stores over NVLink; the call is
// counters[0] + 1).  The quantizer polls its own slot until every word of
// every rank carries the call number, sums y = ((y_0 + y_1) + y_2) ... in
// rank order, x_out = x + y, then rmsnorm + quantize exactly like
// act_quant_kernel's IN_ADD_RMSNORM (same summation orders), so for two
// processes the result equals the NCCL all-reduce path bit for bit.  No
// flag and no second NVLink round trip: a word is ready when it arrives.
// A slot is rewritten two calls later: a process pushes call c + 2 only
// after its quantizer finished call c + 1, which needed every peer's push
// of c + 1, which each peer makes only after its quantizer finished reading
// call c.  Waits are bounded (wait_ns); a wait that gives up sets the error
// word and the later calls of the step skip their waits.
constexpr int kXrCountersBytes = 256;  // counters, padded
struct PeerAddArgs {
    ActQuantArgs q;                    // mode IN_ADD_RMSNORM fields except y
    const uint64_t* slot;              // this process's slot of the call: [tp][ll_rows][n] words
    int ll_rows;
    uint32_t* counters;                // this process's counters[2]
    int tp_rank, tp_size;
    int* err;
    uint64_t wait_ns;                  // limit of the wait for the peers' words (0: the default 2 s)
};
cudaError_t peer_add_quant_launch(const PeerAddArgs& a, cudaStream_t st, bool pdl);

// Plan and launch.  pdl: allow programmatic dependent launch overlap with
// the previous kernel on the stream.  Returns a cudaError_t.
cudaError_t gemv_launch(GemvArgs a, int kind, cudaStream_t st, bool pdl, int num_sms);

// True when the kernel accepts these shapes/pointers.
bool gemv_args_ok(const GemvArgs& a, int kind);

}  // namespace lq
