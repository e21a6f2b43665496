// Per-device context shared by the C-ABI sources (C++ only).
#pragma once
#include <cstddef>
#include <cstdint>
#include <cuda_runtime.h>

#include <vector>

#include "lq_host.h"

namespace lq {

struct DevCtx {
    int dev = 0;
    int num_sms = 148;
    int* err = nullptr;         // device error word for stand-alone operator calls
    void* scratch = nullptr;    // staging for host-pointer calls
    size_t scratch_bytes = 0;
    // tensor-core GEMM (matmul with >= 16 activation rows)
    float* qg_part = nullptr;   // stream-K partials
    int* qg_cnt = nullptr;      // per-tile arrival counters (left zero by every launch)
    float* qg_xst = nullptr;    // transposed activation scales [ng][64]
    size_t qg_xst_floats = 0;
    // matmul_f32 with page-locked host x and y: the call's copy in, quantize,
    // GEMV and copy out replayed as one CUDA graph per (buffers, weight,
    // shape); built on the second call with the same key, dropped whenever
    // the scratch the graphs use is reallocated
    struct CallGraph {
        const void* x;
        void* y;
        const void* wq;
        const float* ws;
        int kind, gs, n, d, flags;
        cudaGraphExec_t exec;  // null until built (or when building failed)
        bool failed;
        uint64_t used;
    };
    std::vector<CallGraph> graphs;
    cudaStream_t capture = nullptr;  // private stream the graphs are captured on
    uint64_t tick = 0;
};

DevCtx* ctx();  // context of the current device (created on first use)
int ensure_scratch(DevCtx* c, size_t bytes);
int cuda_fail(cudaError_t e, const char* what);
int check_device_error(int* err_dev, cudaStream_t st);
int noalloc_check_error(cudaStream_t st);  // matmul_f32_noalloc's error word (noalloc.cu)
cudaStream_t stream();
int launch_flags();     // lq_set_launch_flags
uint64_t* trace_buffer();  // lq_set_trace
int matmul_f32_device(float* yd, const float* xd, const QuantizedTensor* w, int n, int d, int8_t* xq, float* xs,
                      int* xsum, int* err, cudaStream_t st, bool pdl_first, int num_sms, uint64_t* trace);

}  // namespace lq
