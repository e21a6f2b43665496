// Decode-step epilogues shared by the GEMV and the tensor-core GEMM: a
// finished output row pair (r, r+1) of one activation row b is stored,
// added to the residual stream, rotated (RoPE) into q or the K cache,
// written to the V cache, or combined with its w3 partner (SwiGLU).
#pragma once
#include "lq_device.cuh"
#include "lq_kernels.h"
#include "lq_math.h"

namespace lq {

// RoPE, v1-int8-vnni/runq.c:351-365.  cos/sin of pos * freq come from a
// table the host fills with the reference's own formula (1/powf(10000,
// hd/hs), cosf, sinf), so the rotation needs no device transcendentals and
// matches the CPU bit for bit.
__device__ __forceinline__ void rope_pair(const float2* rope, float& v0, float& v1, int r, int head_size, int pos) {
    const float2 cs = rope[(size_t)pos * (head_size >> 1) + ((r % head_size) >> 1)];
    const float a0 = v0, a1 = v1;
    v0 = a0 * cs.x - a1 * cs.y;
    v1 = a0 * cs.y + a1 * cs.x;
}

// Finish rows r and r+1 (when has2) of segment g for batch row b.  For
// EPI_SWIGLU, v0/v1 are the w1 row values and u0/u1 the w3 row values.
__device__ __forceinline__ void finish_rows(const GemvArgs& a, const GemvSeg& g, int b, int r, float v0, float v1, float u0,
                            float u1, bool has2) {
    if (b >= a.nvalid) return;  // padding row of a partial batch chunk
    const int pos = (g.epi == EPI_ROPE_Q || g.epi == EPI_ROPE_KCACHE || g.epi == EPI_VCACHE) ? a.meta[2 * b + 1] : 0;
    switch (g.epi) {
        case EPI_STORE: {
            float* y = g.y + (size_t)b * a.y_stride;
            y[r] = v0;
            if (has2) y[r + 1] = v1;
        } break;
        case EPI_ADD: {
            float* y = g.y + (size_t)b * a.y_stride;
            y[r] += v0;
            if (has2) y[r + 1] += v1;
        } break;
        case EPI_SWIGLU: {
            float* y = g.y + (size_t)b * a.y_stride;
            y[r] = lq_swiglu(v0, u0);
            if (has2) y[r + 1] = lq_swiglu(v1, u1);
        } break;
        case EPI_ROPE_Q: {
            rope_pair(a.rope, v0, v1, r, a.head_size, pos);
            float* y = g.y + (size_t)b * a.y_stride;
            y[r] = v0;
            y[r + 1] = v1;
        } break;
        case EPI_PUSH: {
            // (call << 32) | bits(v) into row (own rank, b) of every process's slot
            const uint64_t e = (uint64_t)(*a.ll_call + 1u) << 32;
            const uint64_t w0 = e | __float_as_uint(v0), w1 = e | __float_as_uint(v1);
            const size_t off = ((size_t)a.ll_rank * a.ll_rows + a.ll_row0 + b) * a.y_stride + r;
            for (int p = 0; p < a.ll_tp; ++p) {
                if (has2)
                    st_relaxed_sys_v2(a.ll[p] + off, w0, w1);  // r even, y_stride even: 16-byte aligned
                else
                    st_relaxed_sys_u64(a.ll[p] + off, w0);
            }
        } break;
        case EPI_ROPE_KCACHE:
        case EPI_VCACHE: {
            if (g.epi == EPI_ROPE_KCACHE) rope_pair(a.rope, v0, v1, r, a.head_size, pos);
            float* c = (g.epi == EPI_ROPE_KCACHE ? a.kcache : a.vcache) + (size_t)b * a.kv_seq_stride;
            const int hs = a.head_size;
            const size_t o = ((size_t)(r / hs) * a.max_seq + pos) * hs + (r % hs);
            c[o] = v0;
            if (has2) c[o + 1] = v1;  // r even, hs even: r+1 is in the same head
        } break;
    }
}

}  // namespace lq
