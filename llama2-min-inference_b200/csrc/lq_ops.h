// Launchers for the non-GEMV kernels (host-visible, C++ only).
#pragma once
#include <cstddef>
#include <cstdint>
#include <cuda.h>
#include <cuda_runtime.h>

namespace lq {

constexpr int kChunk = 64;         // attention positions per CTA

struct AttnArgs {
    // K cache as a 2-D byte tensor [rows][head_size * 4] (one row per cached
    // position), boxes of 128 bytes x kChunk rows with the 128-byte swizzle
    // (kv_tensor_map); krow = row of kcache[0]
    alignas(64) CUtensorMap kmap;
    int64_t krow;
    const float* q;      // [batch][q_stride], query heads already rotated
    const float* kcache; // layer base; [kv_heads][max_seq][head_size] per sequence
    const float* vcache;
    float* out;          // [batch][q_stride] normalised attention output
    float* part;         // [batch][n_heads][max_splits][head_size + 4] partials: m, l, -, -, o[head_size]
    const int* meta;     // [batch][token, pos]
    int* err;            // device error word (a bounded wait that gave up)
    int64_t kv_seq_stride;
    int q_stride;
    int n_heads, n_kv_heads, kv_mul, head_size, max_seq, max_splits;
    uint64_t* kt;        // optional step-trace stamps of this launch; null = off
};

cudaError_t quantize_act_launch(const float* x, int64_t rows, int64_t n, int gs, int8_t* xq, float* xs,
                                cudaStream_t st);
size_t attention_smem_bytes(int head_size, int kv_mul);
// the attention kernel's K-cache map over `rows` cached positions of head_size floats
bool kv_tensor_map(CUtensorMap* m, const float* kcache, int head_size, uint64_t rows);
cudaError_t attention_launch(const AttnArgs& a, int batch, cudaStream_t st, bool pdl);
cudaError_t argmax_launch(const float* logits, int n, int batch, int stride, int* out, cudaStream_t st,
                          bool pdl, uint64_t* kt = nullptr);
cudaError_t synth_f32_launch(float* out, int64_t n, uint64_t seed, int tid, float std, int ones,
                             cudaStream_t st);
cudaError_t synth_quant_launch(uint8_t* q, float* s, int64_t rows, int64_t cols, int gs, int kind,
                               uint64_t seed, int tid, float std, int64_t row0, cudaStream_t st);
// columns [col0, col0+cols) of rows [row0, row0+rows) of a tensor with cols_full columns
cudaError_t synth_quant_cols_launch(uint8_t* q, float* s, int64_t rows, int64_t cols, int64_t cols_full, int64_t col0,
                                    int gs, int kind, uint64_t seed, int tid, float std, int64_t row0,
                                    cudaStream_t st);

}  // namespace lq
