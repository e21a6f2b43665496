// Decode-step kernels around the GEMV: activation quantize (stand-alone),
// split-KV attention, greedy argmax, and the on-device synthetic weight
// generator.
#include <cfloat>

#include "lq_device.cuh"
#include "lq_math.h"
#include "lq_ops.h"

namespace lq {

// ---------------------------------------------------------------------------
// stand-alone activation quantize: quantize_act, v1-int8-vnni/runq.c:117-139
// (GPU form: quantize_act_kernel, v2-cuda/run.cu:102-127).  One warp per group.

__global__ void quantize_act_kernel(const float* __restrict__ x, int64_t ngroups, int gs,
                                    int8_t* __restrict__ xq, float* __restrict__ xs) {
    const int lane = threadIdx.x & 31;
    const int64_t warps = (int64_t)gridDim.x * (blockDim.x >> 5);
    for (int64_t g = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); g < ngroups;
         g += warps) {
        const float* xg = x + g * gs;
        float amax = 0.0f;
        for (int j = lane; j < gs; j += 32) amax = fmaxf(amax, fabsf(xg[j]));
        amax = warp_max(amax);
        float s = amax / 127.0f;
        if (s == 0.0f) s = 1e-8f;
        for (int j = lane; j < gs; j += 32) {
            int q = __float2int_rn(xg[j] / s);
            q = max(-127, min(127, q));
            xq[g * gs + j] = (int8_t)q;
        }
        if (lane == 0) xs[g] = s;
    }
}

cudaError_t quantize_act_launch(const float* x, int64_t rows, int64_t n, int gs, int8_t* xq,
                                float* xs, cudaStream_t st) {
    const int64_t ng = rows * (n / gs);
    int64_t blocks = (ng + 7) / 8;
    if (blocks > 4096) blocks = 4096;
    if (blocks < 1) blocks = 1;
    quantize_act_kernel<<<(unsigned)blocks, 256, 0, st>>>(x, ng, gs, xq, xs);
    return cudaGetLastError();
}

// ---------------------------------------------------------------------------
// split-KV attention (flash-decoding) for one decode position.
//
// Semantics: runq.c:369-391 — per query head h, scores q.k_t / sqrt(hs) for
// t <= pos, softmax, output sum_t p_t v_t (fp32).  Structure: one CTA per
// (kv head, chunk of kChunk positions, sequence); the CTA serves all query
// heads of its kv head (GQA: K/V are read from HBM once).  A CTA writes its
// unnormalised partial (max, sum, o); the last CTA of a kv head (arrival
// counter) merges the partials and writes the normalised output.  A single
// chunk writes the output directly.  The output stays fp32: the wo GEMV
// quantizes it in its prologue (runq.c:394 order: quantize the normalised
// output — not v5's unnormalised-scale variant).

__global__ void __launch_bounds__(kAttnThreads) attention_kernel(const __grid_constant__ AttnArgs a) {
    extern __shared__ __align__(16) float asmem[];
    __shared__ __align__(8) uint64_t kv_bar;
    pdl_trigger();
    kt_start(a.kt);
    const int kvh = blockIdx.x, split = blockIdx.y, b = blockIdx.z;
    const int hs = a.head_size, km = a.kv_mul;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    constexpr int NW = kAttnThreads / 32;
    // the positions were written before the step's first kernel started, so
    // they can be read before waiting for the preceding kernel
    const int pos = a.meta[2 * b + 1];
    const int nsplit = pos / kChunk + 1;
    if (split >= nsplit) return;
    const int t0 = split * kChunk;
    const int nt = min(kChunk, pos + 1 - t0);

    float* ks = asmem;                  // [kChunk][hs]
    float* vs = ks + kChunk * hs;       // [kChunk][hs]
    float* qs = vs + kChunk * hs;       // [km][hs]
    float* sc = qs + km * hs;           // [km][kChunk]
    float* ml = sc + km * kChunk;       // [km][2]

    // K and V of the chunk by two bulk copies (TMA).  A chunk without the
    // current position holds only earlier steps' keys and values, so its copy
    // starts before the preceding kernel (which writes position pos) is done.
    const size_t cbase = (size_t)b * a.kv_seq_stride + ((size_t)kvh * a.max_seq + t0) * hs;
    const uint32_t bytes = (uint32_t)(nt * hs * sizeof(float));
    if (tid == 0) {
        mbar_init(&kv_bar, 1);
        fence_mbar_init();
        if (t0 + nt - 1 == pos) pdl_wait();
        const uint64_t pol = l2_evict_first_policy();
        mbar_arrive_expect_tx(&kv_bar, 2 * bytes);
        bulk_g2s(ks, a.kcache + cbase, bytes, &kv_bar, pol);
        bulk_g2s(vs, a.vcache + cbase, bytes, &kv_bar, pol);
    }
    pdl_wait();
    kt_waited(a.kt);
    const float* qg = a.q + (size_t)b * a.q_stride + (size_t)kvh * km * hs;
    for (int i = tid; i < km * hs; i += kAttnThreads) qs[i] = qg[i];
    __syncthreads();  // also orders the barrier's initialisation before the waits below
    const bool landed = mbar_wait(&kv_bar, 0, a.err, DEV_TIMEOUT_FULL);
    if (!__syncthreads_and(landed)) {
        // give up on this chunk; confirm the copies before the CTA's shared memory is released
        if (tid == 0) mbar_wait(&kv_bar, 0, a.err, DEV_TIMEOUT_DRAIN);
        return;
    }

    // scores: warp per position, lanes over dims.  Four positions at a time per
    // warp: independent dot products and reductions interleave (each one in
    // the same order as alone).
    const float rs = sqrtf((float)hs);
    constexpr int U = 4;
    for (int t0w = warp; t0w < nt; t0w += U * NW) {
        for (int j = 0; j < km; ++j) {
            const float* qj = qs + j * hs;
            float p[U];
#pragma unroll
            for (int u = 0; u < U; ++u) p[u] = 0.0f;
#pragma unroll 4
            for (int i = lane; i < hs; i += 32) {
                const float qv = qj[i];
#pragma unroll
                for (int u = 0; u < U; ++u) {
                    const int t = t0w + u * NW;
                    if (t < nt) p[u] = fmaf(qv, ks[t * hs + i], p[u]);
                }
            }
#pragma unroll
            for (int o = 16; o > 0; o >>= 1)
#pragma unroll
                for (int u = 0; u < U; ++u) p[u] += __shfl_xor_sync(0xffffffffu, p[u], o);
            if (lane == 0)
#pragma unroll
                for (int u = 0; u < U; ++u) {
                    const int t = t0w + u * NW;
                    if (t < nt) sc[j * kChunk + t] = p[u] / rs;
                }
        }
    }
    __syncthreads();
    // per head: max, exp, sum (warp per head)
    for (int j = warp; j < km; j += NW) {
        float m = -FLT_MAX;
        for (int t = lane; t < nt; t += 32) m = fmaxf(m, sc[j * kChunk + t]);
        m = warp_max(m);
        float l = 0.0f;
        for (int t = lane; t < nt; t += 32) {
            const float e = lq_expf(sc[j * kChunk + t] - m);
            sc[j * kChunk + t] = e;
            l += e;
        }
        l = warp_sum(l);
        if (lane == 0) {
            ml[2 * j] = m;
            ml[2 * j + 1] = l;
        }
    }
    __syncthreads();
    // o[j][d] = sum_t p[j][t] * v[t][d]
    float* out = a.out + (size_t)b * a.q_stride + (size_t)kvh * km * hs;
    const int hq0 = kvh * km;
    for (int i = tid; i < km * hs; i += kAttnThreads) {
        const int j = i / hs, d = i - j * hs;
        const float* pj = sc + j * kChunk;
        float o = 0.0f;
#pragma unroll 8
        for (int t = 0; t < nt; ++t) o = fmaf(pj[t], vs[t * hs + d], o);
        if (nsplit == 1) {
            out[i] = o / ml[2 * j + 1];
        } else {
            float* part = a.part + (((size_t)b * a.n_heads + hq0 + j) * a.max_splits + split) * (hs + 2);
            part[2 + d] = o;
            if (d == 0) {
                part[0] = ml[2 * j];
                part[1] = ml[2 * j + 1];
            }
        }
    }
    if (nsplit == 1) {
        kt_end_cta(a.kt);
        return;
    }
    // last-arriving CTA of this kv head merges the partials
    __threadfence();
    __syncthreads();
    __shared__ int is_last;
    if (tid == 0) {
        int* cnt = a.counters + (size_t)b * a.n_kv_heads + kvh;
        is_last = atomicAdd(cnt, 1) == nsplit - 1;
        if (is_last) *cnt = 0;  // re-arm for the next step
    }
    __syncthreads();
    if (!is_last) {
        kt_end_cta(a.kt);
        return;
    }
    __threadfence();
    // The partials of a group of heads are first copied into shared memory
    // (the K / V chunk buffers are free by now) by every thread at once, so
    // the merge waits for one round of L2 loads, not one per chunk; the merge
    // arithmetic itself is unchanged: M = max over the chunks, then L and o
    // accumulated with fmaf in chunk order.
    const int per_head = nsplit * (hs + 2);
    const int cap = 2 * kChunk * hs;                    // floats of the K and V buffers
    const int hb = cap / per_head < 1 ? 1 : (cap / per_head < km ? cap / per_head : km);
    const bool staged = per_head <= cap;
    for (int j0 = 0; j0 < km; j0 += hb) {
        const int nh = km - j0 < hb ? km - j0 : hb;
        if (staged) {
            __syncthreads();  // the previous group's reads of the buffer are done
            for (int hh = 0; hh < nh; ++hh) {
                const float* src = a.part + (((size_t)b * a.n_heads + hq0 + j0 + hh) * a.max_splits) * (hs + 2);
                float* dst = ks + hh * per_head;
                for (int i = tid; i < per_head; i += kAttnThreads) dst[i] = __ldcg(src + i);
            }
            __syncthreads();
        }
        for (int i = tid; i < nh * hs; i += kAttnThreads) {
            const int jj = i / hs, d = i - jj * hs, j = j0 + jj;
            const float* base = staged ? ks + jj * per_head
                                       : a.part + (((size_t)b * a.n_heads + hq0 + j) * a.max_splits) * (hs + 2);
            float M = -FLT_MAX;
#pragma unroll 8
            for (int s = 0; s < nsplit; ++s) M = fmaxf(M, base[(size_t)s * (hs + 2)]);
            float L = 0.0f, o = 0.0f;
#pragma unroll 4
            for (int s = 0; s < nsplit; ++s) {
                const float* ps = base + (size_t)s * (hs + 2);
                const float w = lq_expf(ps[0] - M);
                L = fmaf(ps[1], w, L);
                o = fmaf(ps[2 + d], w, o);
            }
            out[j * hs + d] = o / L;
        }
    }
    kt_end_cta(a.kt);
}

size_t attention_smem_bytes(int head_size, int kv_mul) {
    return sizeof(float) * ((size_t)2 * kChunk * head_size + (size_t)kv_mul * head_size +
                            (size_t)kv_mul * kChunk + 2 * (size_t)kv_mul);
}

cudaError_t attention_launch(const AttnArgs& a, int batch, cudaStream_t st, bool pdl) {
    const size_t smem = attention_smem_bytes(a.head_size, a.kv_mul);
    static size_t set_bytes = 0;
    if (smem > 48 * 1024 && smem > set_bytes) {
        cudaError_t e =
            cudaFuncSetAttribute(attention_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        if (e != cudaSuccess) return e;
        set_bytes = smem;
    }
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(a.n_kv_heads, a.max_splits, batch);
    cfg.blockDim = dim3(kAttnThreads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, attention_kernel, a);
}

// ---------------------------------------------------------------------------
// greedy argmax, sample_argmax runq.c:578-585: first index of the maximum.

__global__ void __launch_bounds__(1024) argmax_kernel(const float* __restrict__ logits, int n, int stride,
                                                      int* __restrict__ out, uint64_t* kt) {
    pdl_trigger();
    kt_start(kt);
    pdl_wait();
    kt_waited(kt);
    const float* v = logits + (size_t)blockIdx.x * stride;
    float bv = -FLT_MAX;
    int bi = -1;
    for (int i = threadIdx.x; i < n; i += blockDim.x) {
        const float x = v[i];
        if (bi < 0 || x > bv) {
            bv = x;
            bi = i;
        }
    }
    __shared__ float sv[32];
    __shared__ int si[32];
    for (int o = 16; o > 0; o >>= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
        const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
        if (oi >= 0 && (bi < 0 || ov > bv || (ov == bv && oi < bi))) {
            bv = ov;
            bi = oi;
        }
    }
    if ((threadIdx.x & 31) == 0) {
        sv[threadIdx.x >> 5] = bv;
        si[threadIdx.x >> 5] = bi;
    }
    __syncthreads();
    if (threadIdx.x < 32) {
        const int nw = blockDim.x >> 5;
        bv = threadIdx.x < nw ? sv[threadIdx.x] : -FLT_MAX;
        bi = threadIdx.x < nw ? si[threadIdx.x] : -1;
        for (int o = 16; o > 0; o >>= 1) {
            const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
            const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
            if (oi >= 0 && (bi < 0 || ov > bv || (ov == bv && oi < bi))) {
                bv = ov;
                bi = oi;
            }
        }
        if (threadIdx.x == 0) out[blockIdx.x] = bi < 0 ? 0 : bi;
    }
    kt_end_cta(kt);
}

cudaError_t argmax_launch(const float* logits, int n, int batch, int stride, int* out, cudaStream_t st,
                          bool pdl, uint64_t* kt) {
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(batch);
    cfg.blockDim = dim3(1024);
    cfg.stream = st;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, argmax_kernel, logits, n, stride, out, kt);
}

// ---------------------------------------------------------------------------
// synthetic weights on the device (bit-identical to lq_synth_value and the
// host quantizer in ckpt.c)

__device__ __forceinline__ uint64_t mix64(uint64_t z) {
    z += 0x9E3779B97F4A7C15ull;
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}

__device__ __forceinline__ float synth(uint64_t seedmix, int tid, uint64_t idx, float scale) {
    const uint64_t base = seedmix + ((uint64_t)tid << 48) + idx * 6ull;
    int32_t s = 0;
#pragma unroll
    for (int j = 0; j < 6; ++j) {
        const uint64_t h = mix64(base + (uint64_t)j);
        s += (int32_t)(h & 0xFFFFFFu) + (int32_t)((h >> 32) & 0xFFFFFFu);
    }
    s -= 6 << 24;
    return __int2float_rn(s) * scale;
}

__global__ void synth_f32_kernel(float* out, int64_t n, uint64_t seedmix, int tid, float scale, int ones) {
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
        out[i] = ones ? 1.0f : synth(seedmix, tid, (uint64_t)i, scale);
}

// one thread per group: weights of rows [row0, row0+rows), columns
// [col0, col0+cols) of tensor `tid` whose rows hold cols_full values
__global__ void synth_quant_kernel(uint8_t* q, float* s, int64_t rows, int64_t cols, int gs, int kind,
                                   uint64_t seedmix, int tid, float scale, int64_t row0, int64_t cols_full,
                                   int64_t col0) {
    const int64_t ng = cols / gs;
    const int64_t total = rows * ng;
    float v[256];
    for (int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; t < total;
         t += (int64_t)gridDim.x * blockDim.x) {
        const int64_t r = t / ng, g = t - r * ng;
        const uint64_t e0 = (uint64_t)(row0 + r) * cols_full + col0 + g * gs;
        float amax = 0.0f;
        for (int j = 0; j < gs; ++j) {
            v[j] = synth(seedmix, tid, e0 + j, scale);
            amax = fmaxf(amax, fabsf(v[j]));
        }
        float sc = amax / (kind == 8 ? 127.0f : 8.0f);
        if (sc == 0.0f) sc = 1e-8f;
        s[t] = sc;
        if (kind == 8) {
            uint8_t* qr = q + r * cols + g * gs;
            for (int j = 0; j < gs; ++j) {
                float x = rintf(v[j] / sc);
                x = fminf(127.0f, fmaxf(-127.0f, x));
                qr[j] = (uint8_t)(int)(x + 128.0f);
            }
        } else {
            uint8_t* qr = q + r * (cols / 2) + g * gs / 2;
            for (int j = 0; j < gs; j += 2) {
                float x0 = rintf(v[j] / sc), x1 = rintf(v[j + 1] / sc);
                x0 = fminf(7.0f, fmaxf(-8.0f, x0));
                x1 = fminf(7.0f, fmaxf(-8.0f, x1));
                qr[j / 2] = (uint8_t)(((unsigned)(int)x0 & 0xFu) | (((unsigned)(int)x1 & 0xFu) << 4));
            }
        }
    }
}

static uint64_t host_mix64(uint64_t z) {
    z += 0x9E3779B97F4A7C15ull;
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}

cudaError_t synth_f32_launch(float* out, int64_t n, uint64_t seed, int tid, float std, int ones,
                             cudaStream_t st) {
    const float scale = std * 5.9604644775390625e-8f;
    int64_t blocks = (n + 255) / 256;
    if (blocks > 65536) blocks = 65536;
    synth_f32_kernel<<<(unsigned)blocks, 256, 0, st>>>(out, n, host_mix64(seed), tid, scale, ones);
    return cudaGetLastError();
}

cudaError_t synth_quant_launch(uint8_t* q, float* s, int64_t rows, int64_t cols, int gs, int kind,
                               uint64_t seed, int tid, float std, int64_t row0, cudaStream_t st) {
    const float scale = std * 5.9604644775390625e-8f;
    const int64_t groups = rows * (cols / gs);
    int64_t blocks = (groups + 127) / 128;
    if (blocks > 65536) blocks = 65536;
    synth_quant_kernel<<<(unsigned)blocks, 128, 0, st>>>(q, s, rows, cols, gs, kind, host_mix64(seed), tid,
                                                          scale, row0, cols, 0);
    return cudaGetLastError();
}

cudaError_t synth_quant_cols_launch(uint8_t* q, float* s, int64_t rows, int64_t cols, int64_t cols_full, int64_t col0,
                                    int gs, int kind, uint64_t seed, int tid, float std, int64_t row0,
                                    cudaStream_t st) {
    const float scale = std * 5.9604644775390625e-8f;
    const int64_t groups = rows * (cols / gs);
    int64_t blocks = (groups + 127) / 128;
    if (blocks > 65536) blocks = 65536;
    synth_quant_kernel<<<(unsigned)blocks, 128, 0, st>>>(q, s, rows, cols, gs, kind, host_mix64(seed), tid,
                                                          scale, row0, cols_full, col0);
    return cudaGetLastError();
}

}  // namespace lq
