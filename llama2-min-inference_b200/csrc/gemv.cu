// Group-quantized GEMV for sm_100a.
//
// y[r] = sum_g (ws[r,g] * xs[g]) * D[r,g],  D[r,g] = exact int32 group dot.
//
// Reference arithmetic: matmul_q8, v1-int8-vnni/runq.c:142-159 (INT8: the
// stored byte is q+128, VPDPBUSD unsigned x signed, bias removed with the
// activation group sum); matmul_q4_vec_kernel, v5-cuda-fused/run.cu:276-330
// (INT4 two's-complement nibbles, even element in the low nibble, per-group
// fp32 scale applied after the integer dot).
//
// Design (B200):
//  * The weight rows a CTA owns are one contiguous byte range (row-major
//    [d, n] layout), and so are their scales.  One elected producer thread
//    streams them with 1-D bulk copies (cp.async.bulk, the TMA engine) into a
//    ring of ~8 KB shared-memory stages, completion tracked by mbarriers,
//    L2 policy evict-first (weights are read once per token).
//  * Each stage belongs to one consumer warp (whole-row stages round-robin;
//    row slices by row pair), so eight stages are computed concurrently with
//    no cross-warp synchronisation, while the producer keeps the rest of the
//    ring in flight.
//  * Inside a warp each lane owns whole groups: it reads the group's 16-byte
//    chunks in a lane-rotated order (bank-conflict free for the stage and the
//    staged activation) and forms the exact int32 group dot with dp4a, with
//    no shuffles.  INT8 keeps the file's biased bytes: dp4a.u32.s32 gives
//    D + 128*sum(x) and the activation group sum is subtracted.  INT4 nibbles
//    become offset bytes (q+8) with one LOP3 per 4 values, dotted against an
//    activation staged as two byte planes (even / odd elements), giving
//    D + 8*sum(x).  Both corrections are exact integer identities.
//  * The activation is built in the prologue of every CTA (quantize, or
//    rmsnorm + quantize), one thread per group, so no separate kernel or
//    global scratch is needed for it.
//  * Programmatic dependent launch: inside a model the producer starts
//    streaming weights before griddepcontrol.wait, so a GEMV's first stages
//    load while the previous kernel finishes.
//  * Every wait is bounded (2 s); on expiry the kernel records an error code,
//    the producer confirms its in-flight copies (bounded) and all threads
//    return.
#include <cstdio>
#include <cstdlib>

#include "lq_device.cuh"
#include "lq_kernels.h"
#include "lq_math.h"

namespace lq {

constexpr int kW = kConsumerWarps;
constexpr int kCT = kW * 32;

__host__ __device__ inline int align_up(int v, int a) { return (v + a - 1) / a * a; }

struct Layout {
    int off_bars, off_red, off_x, off_xs, off_xsum, off_stage, stage_bytes, total;
};

__host__ __device__ inline Layout make_layout(const GemvArgs& a) {
    Layout L;
    const int ng = a.cols / a.gs;
    L.off_bars = 0;
    L.off_red = align_up(a.nstages * 8, 16);
    L.off_x = align_up(L.off_red + kW * 4, 128);
    L.off_xs = align_up(L.off_x + a.x_bytes, 16);
    L.off_xsum = align_up(L.off_xs + a.nb * ng * 4, 16);
    L.off_stage = align_up(L.off_xsum + a.nb * ng * 4, 128);
    L.stage_bytes = a.wcap + a.scap;
    L.total = L.off_stage + a.nstages * L.stage_bytes;
    return L;
}

// ---------------------------------------------------------------------------
// activation prologue

// INT4 activation layout: two planes of n/2 bytes; element k lives in plane
// (k & 1) at byte (k >> 3) * 4 + ((k >> 1) & 3), so the 16 bytes that pair
// with weight chunk c are at offset 16c of each plane.
__device__ __forceinline__ int int4_act_offset(int k, int n) {
    return (k & 1) * (n >> 1) + (k >> 3) * 4 + ((k >> 1) & 3);
}

// rint(x / s) exactly as IEEE division would give it, without dividing in
// the common case: t = x * (1/s) is within 1.5 ulp of x/s, so rint(t) equals
// rint(x/s) unless t lies within a few ulp of a half-integer; only then is
// the correctly rounded quotient computed.
__device__ __forceinline__ int quant_div(float x, float s, float rcp) {
    const float t = x * rcp;
    const float r = rintf(t);
    if (fabsf(fabsf(t - r) - 0.5f) <= fabsf(t) * 2.384185791015625e-7f) return __float2int_rn(x / s);
    return (int)r;
}

// Deterministic sum over the consumer threads (same order in every CTA).
__device__ float consumer_sum(float v, float* red, int ctid) {
    v = warp_sum(v);
    if ((ctid & 31) == 0) red[ctid >> 5] = v;
    named_bar_sync(1, kCT);
    float s = 0.0f;
#pragma unroll
    for (int w = 0; w < kW; ++w) s += red[w];
    named_bar_sync(1, kCT);
    return s;
}

template <int KIND>
__device__ void stage_input(const GemvArgs& a, int8_t* xsm, float* xs, int* xsum, float* red, int ctid) {
    const int n = a.cols, gs = a.gs, ng = n / gs;
    if (a.in_mode == IN_QUANT) {
        // copy int8 rows (INT4: split into even/odd planes), 8 bytes a step
        const int total8 = a.nb * n / 8;
        for (int i = ctid; i < total8; i += kCT) {
            const uint2 v = reinterpret_cast<const uint2*>(a.xq)[i];
            const int b = (i * 8) / n, k0 = i * 8 - b * n;
            int8_t* xrow = xsm + (size_t)b * n;
            if (KIND == 4) {
                *reinterpret_cast<uint32_t*>(xrow + (k0 >> 1)) = __byte_perm(v.x, v.y, 0x6420);
                *reinterpret_cast<uint32_t*>(xrow + (n >> 1) + (k0 >> 1)) = __byte_perm(v.x, v.y, 0x7531);
            } else {
                *reinterpret_cast<uint2*>(xrow + k0) = v;
            }
        }
        for (int g = ctid; g < a.nb * ng; g += kCT) {
            const int4* q = reinterpret_cast<const int4*>(a.xq + (size_t)g * gs);
            int s = 0;
            for (int j = 0; j < gs / 16; ++j) {
                const int4 v = q[j];
                s = __dp4a(v.x, 0x01010101, s);
                s = __dp4a(v.y, 0x01010101, s);
                s = __dp4a(v.z, 0x01010101, s);
                s = __dp4a(v.w, 0x01010101, s);
            }
            xs[g] = a.xs[g];
            xsum[g] = s;
        }
        return;
    }
    for (int b = 0; b < a.nb; ++b) {
        const float* src = a.xf ? a.xf + (size_t)b * n : nullptr;
        float inv = 1.0f;
        if (a.in_mode == IN_RMSNORM_EMB) {
            const int token = a.meta[2 * b];
            src = a.emb + (size_t)token * n;
            if (blockIdx.x == 0)
                for (int i = ctid; i < n; i += kCT) a.x_out[(size_t)b * n + i] = src[i];
        }
        const bool norm = a.in_mode == IN_RMSNORM || a.in_mode == IN_RMSNORM_EMB;
        if (norm) {
            // rmsnorm, v1-int8-vnni/runq.c:294-305: 1/sqrt(mean(x^2) + 1e-5);
            // thread t sums float4 chunks t, t+256, ... in order
            float ss = 0.0f;
            for (int c = ctid; c < n / 4; c += kCT) {
                const float4 v = reinterpret_cast<const float4*>(src)[c];
                ss = fmaf(v.x, v.x, ss);
                ss = fmaf(v.y, v.y, ss);
                ss = fmaf(v.z, v.z, ss);
                ss = fmaf(v.w, v.w, ss);
            }
            ss = consumer_sum(ss, red, ctid);
            inv = 1.0f / sqrtf(ss / (float)n + 1e-5f);
        }
        int8_t* xrow = xsm + (size_t)b * n;
        // quantize_act, runq.c:117-139: eight lanes per group, eight values
        // per lane (group max and sum over the eight lanes by xor shuffles)
        const int lpg = gs / 8;  // lanes per group: 4, 8, 16 or 32
        const int tasks = ng * lpg;
        for (int t0 = 0; t0 < tasks; t0 += kCT) {
            const int t = t0 + ctid;
            const bool on = t < tasks;
            const int k0 = (on ? t : 0) * 8;  // first of this lane's 8 values
            float v[8];
            float amax = 0.0f;
            if (on) {
                const float4 a0 = *reinterpret_cast<const float4*>(src + k0);
                const float4 a1 = *reinterpret_cast<const float4*>(src + k0 + 4);
                v[0] = a0.x; v[1] = a0.y; v[2] = a0.z; v[3] = a0.w;
                v[4] = a1.x; v[5] = a1.y; v[6] = a1.z; v[7] = a1.w;
                if (norm) {
                    const float4 w0 = *reinterpret_cast<const float4*>(a.rms_w + k0);
                    const float4 w1 = *reinterpret_cast<const float4*>(a.rms_w + k0 + 4);
                    const float w[8] = {w0.x, w0.y, w0.z, w0.w, w1.x, w1.y, w1.z, w1.w};
#pragma unroll
                    for (int i = 0; i < 8; ++i) v[i] = w[i] * (inv * v[i]);
                }
#pragma unroll
                for (int i = 0; i < 8; ++i) amax = fmaxf(amax, fabsf(v[i]));
            }
            for (int o = 1; o < lpg; o <<= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
            float sc = amax / 127.0f;
            if (sc == 0.0f) sc = 1e-8f;
            const float rcp = 1.0f / sc;
            int qs = 0;
            uint32_t lo = 0, hi = 0;
            if (on) {
                int q[8];
#pragma unroll
                for (int i = 0; i < 8; ++i) {
                    q[i] = max(-127, min(127, quant_div(v[i], sc, rcp)));
                    qs += q[i];
                }
                if (KIND == 4) {  // even values to plane 0, odd values to plane 1
                    lo = (q[0] & 0xFF) | ((q[2] & 0xFF) << 8) | ((q[4] & 0xFF) << 16) | ((uint32_t)(q[6] & 0xFF) << 24);
                    hi = (q[1] & 0xFF) | ((q[3] & 0xFF) << 8) | ((q[5] & 0xFF) << 16) | ((uint32_t)(q[7] & 0xFF) << 24);
                    *reinterpret_cast<uint32_t*>(xrow + (k0 >> 1)) = lo;
                    *reinterpret_cast<uint32_t*>(xrow + (n >> 1) + (k0 >> 1)) = hi;
                } else {
                    lo = (q[0] & 0xFF) | ((q[1] & 0xFF) << 8) | ((q[2] & 0xFF) << 16) | ((uint32_t)(q[3] & 0xFF) << 24);
                    hi = (q[4] & 0xFF) | ((q[5] & 0xFF) << 8) | ((q[6] & 0xFF) << 16) | ((uint32_t)(q[7] & 0xFF) << 24);
                    *reinterpret_cast<uint2*>(xrow + k0) = make_uint2(lo, hi);
                }
            }
            for (int o = 1; o < lpg; o <<= 1) qs += __shfl_xor_sync(0xffffffffu, qs, o);
            if (on && (t & (lpg - 1)) == 0) {
                const int g = t / lpg;
                xs[b * ng + g] = sc;
                xsum[b * ng + g] = qs;
            }
        }
    }
}

// ---------------------------------------------------------------------------
// dot products

// D + bias*sum(x) over one 16-byte weight chunk (chunk c of the row).
template <int KIND>
__device__ __forceinline__ int chunk_dot(const uint4 w, const int8_t* xrow, int c, int n, int d) {
    if (KIND == 8) {
        const uint4 x = *reinterpret_cast<const uint4*>(xrow + 16 * c);
        d = dp4a_us(w.x, x.x, d);
        d = dp4a_us(w.y, x.y, d);
        d = dp4a_us(w.z, x.z, d);
        d = dp4a_us(w.w, x.w, d);
        return d;
    } else {
        const uint4 xe = *reinterpret_cast<const uint4*>(xrow + 16 * c);
        const uint4 xo = *reinterpret_cast<const uint4*>(xrow + (n >> 1) + 16 * c);
        const uint32_t M = 0x0F0F0F0Fu, F = 0x08080808u;
        d = dp4a_us((w.x ^ F) & M, xe.x, d);
        d = dp4a_us(((w.x >> 4) ^ F) & M, xo.x, d);
        d = dp4a_us((w.y ^ F) & M, xe.y, d);
        d = dp4a_us(((w.y >> 4) ^ F) & M, xo.y, d);
        d = dp4a_us((w.z ^ F) & M, xe.z, d);
        d = dp4a_us(((w.z >> 4) ^ F) & M, xo.z, d);
        d = dp4a_us((w.w ^ F) & M, xe.w, d);
        d = dp4a_us(((w.w >> 4) ^ F) & M, xo.w, d);
        return d;
    }
}

__device__ __forceinline__ uint4 ldg_stream(const uint8_t* p) {
    uint4 v;
    asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0, %1, %2, %3}, [%4];"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
                 : "l"(p));
    return v;
}

// Lane map for one warp pass over 32/LPG groups of NR rows:
//   LPG (lanes per group) = 1 when a group is one 16-byte chunk, else 2;
//   the two lanes of a group take alternate chunks, so every load
//   instruction of the warp reads whole 32-byte sectors;
//   CPL = chunks per lane; the chunk order is rotated by the group's
//   position in its 8-lane shared-memory phase, which makes the activation
//   reads bank-conflict free.
// Each lane forms its partial integer dot, one xor-shuffle completes the
// exact int32 group dot, and the group's first lane accumulates
// out[r][b] += (ws * xs) * D, groups in increasing order per lane.
template <int KIND, int NB, int CPG, int NR>
__device__ __forceinline__ void block_dot(const uint8_t* const* rows, const float* const* scl, int nv, int ng,
                                          int n, const int8_t* xsm, const float* xs, const int* xsum, int lane,
                                          float out[NR][NB]) {
    constexpr int BIAS = KIND == 8 ? 128 : 8;
    constexpr int LPG = CPG == 1 ? 1 : 2;
    constexpr int CPL = CPG / LPG;
    constexpr int GPP = 32 / LPG;  // groups per warp pass
    const int h = LPG == 2 ? (lane & 1) : 0;
    const int gi = lane / LPG;     // group slot in the pass
    const int ph = gi & 3;         // position inside the 8-lane phase
    const int rot = CPL == 2 ? (ph >> 1) : (CPL >= 4 ? (ph & (CPL - 1)) : 0);
#pragma unroll 1
    for (int g0 = 0; g0 < ng; g0 += GPP) {
        const int g = g0 + gi;
        const bool on = g < ng;
        uint4 w[NR][CPL];
#pragma unroll
        for (int r = 0; r < NR; ++r)
#pragma unroll
            for (int k = 0; k < CPL; ++k) {
                const int c = g * CPG + LPG * ((k + rot) & (CPL - 1)) + h;
                w[r][k] = (on && r < nv) ? ldg_stream(rows[r] + (size_t)c * 16) : make_uint4(0, 0, 0, 0);
            }
        float sw[NR];
#pragma unroll
        for (int r = 0; r < NR; ++r) sw[r] = (on && r < nv && h == 0) ? __ldg(scl[r] + g) : 0.0f;
#pragma unroll
        for (int b = 0; b < NB; ++b) {
            const int8_t* xrow = xsm + (size_t)b * n;
            const float xsc = on ? xs[b * ng + g] : 0.0f;
            const int xsu = on ? BIAS * xsum[b * ng + g] : 0;
#pragma unroll
            for (int r = 0; r < NR; ++r) {
                int d = 0;
#pragma unroll
                for (int k = 0; k < CPL; ++k) {
                    const int c = g * CPG + LPG * ((k + rot) & (CPL - 1)) + h;
                    if (on) d = chunk_dot<KIND>(w[r][k], xrow, c, n, d);
                }
                if (LPG == 2) d += __shfl_xor_sync(0xffffffffu, d, 1);
                if (h == 0 && on && r < nv) out[r][b] = fmaf(sw[r] * xsc, (float)(d - xsu), out[r][b]);
            }
        }
    }
}

// ---------------------------------------------------------------------------
// epilogue

__device__ __forceinline__ void rope_pair(float& v0, float& v1, int r, int head_size, int pos) {
    // RoPE, v1-int8-vnni/runq.c:351-365
    const int hd = r % head_size;
    const float freq = 1.0f / powf(10000.0f, hd / (float)head_size);
    const float val = pos * freq;
    const float fcr = cosf(val), fci = sinf(val);
    const float a0 = v0, a1 = v1;
    v0 = a0 * fcr - a1 * fci;
    v1 = a0 * fci + a1 * fcr;
}

// Finish rows r and r+1 (when has2) of segment g for batch row b.  For
// EPI_SWIGLU, v0/v1 are the w1 row values and u0/u1 the w3 row values.
__device__ void finish_rows(const GemvArgs& a, const GemvSeg& g, int b, int r, float v0, float v1, float u0,
                            float u1, bool has2) {
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
            rope_pair(v0, v1, r, a.head_size, pos);
            float* y = g.y + (size_t)b * a.y_stride;
            y[r] = v0;
            y[r + 1] = v1;
        } break;
        case EPI_ROPE_KCACHE:
        case EPI_VCACHE: {
            if (g.epi == EPI_ROPE_KCACHE) rope_pair(v0, v1, r, a.head_size, pos);
            float* c = (g.epi == EPI_ROPE_KCACHE ? a.kcache : a.vcache) + (size_t)b * a.kv_seq_stride;
            const int hs = a.head_size;
            const size_t o = ((size_t)(r / hs) * a.max_seq + pos) * hs + (r % hs);
            c[o] = v0;
            if (has2) c[o + 1] = v1;  // r even, hs even: r+1 is in the same head
        } break;
    }
}

// ---------------------------------------------------------------------------
// the kernel
//
// Work unit: a row pair (r, r+1) of one segment, which also carries the
// second tensor's pair for EPI_SWIGLU.  Warp w of the grid takes the
// contiguous pair range [w*P/W, (w+1)*P/W).  Before griddepcontrol.wait a
// warp asks the TMA engine to prefetch its first rows into L2
// (cp.async.bulk.prefetch), so inside a model the weight stream of a GEMV
// starts while the previous kernel is still finishing.

constexpr int kPrefetchBytes = 8192;  // per warp, at kernel start

__device__ __forceinline__ void prefetch_l2(const void* p, uint32_t bytes) {
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(p), "r"(bytes) : "memory");
}

__device__ __forceinline__ void pair_of(const GemvArgs& a, int p, int& seg, int& r, bool& has2) {
    seg = 0;
    int np = (a.seg[0].rows + 1) >> 1;
    while (p >= np) {
        p -= np;
        ++seg;
        np = (a.seg[seg].rows + 1) >> 1;
    }
    r = 2 * p;
    has2 = r + 1 < a.seg[seg].rows;
}

template <int KIND, int NB, int CPG>
__global__ void __launch_bounds__(kGemvThreads, NB == 1 ? 4 : (NB == 2 ? 2 : 1)) gemv_kernel(const __grid_constant__ GemvArgs a, int prefetch) {
    extern __shared__ __align__(128) uint8_t smem[];
    pdl_trigger();
    const Layout L = make_layout(a);
    float* red = reinterpret_cast<float*>(smem + L.off_red);
    int8_t* xsm = reinterpret_cast<int8_t*>(smem + L.off_x);
    float* xs = reinterpret_cast<float*>(smem + L.off_xs);
    int* xsum = reinterpret_cast<int*>(smem + L.off_xsum);
    const int n = a.cols, ng = n / a.gs;
    const int rb = KIND == 8 ? n : n / 2;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    int P = 0;
    for (int i = 0; i < a.nseg; ++i) P += (a.seg[i].rows + 1) >> 1;
    const long long W = (long long)gridDim.x * kW, wg = (long long)blockIdx.x * kW + warp;
    const int p0 = (int)(wg * P / W), p1 = (int)((wg + 1) * P / W);

    if (lane == 0 && p0 < p1) {
        // this warp's first rows (and scales) into L2
        int seg, r;
        bool has2;
        pair_of(a, p0, seg, r, has2);
        const GemvSeg& g = a.seg[seg];
        const int rows_left = min(g.rows - r, 2 * (p1 - p0));
        const uint32_t wb = (uint32_t)min((long long)rows_left * rb, (long long)kPrefetchBytes) & ~15u;
        if (wb) {
            prefetch_l2(g.wq + (size_t)r * rb, wb);
            if (a.paired) prefetch_l2(g.wq2 + (size_t)r * rb, wb);
        }
    }
    pdl_wait();
    stage_input<KIND>(a, xsm, xs, xsum, red, threadIdx.x);
    __syncthreads();

    constexpr int NR = CPG >= 4 ? 2 : 4;  // rows loaded together: 8 x 16 B per lane in flight (CPG <= 4)
    for (int p = p0; p < p1;) {
        int seg, r;
        bool has2;
        pair_of(a, p, seg, r, has2);
        const GemvSeg& g = a.seg[seg];
        // rows of this step: the pair, its SwiGLU partner pair, or (NR = 4,
        // unpaired) the next pair of the same segment
        const uint8_t* rows[NR];
        const float* scl[NR];
        int nv = 0, npairs = 1;
        rows[0] = g.wq + (size_t)r * rb;
        scl[0] = g.ws + (size_t)r * ng;
        rows[1] = rows[0] + rb;
        scl[1] = scl[0] + ng;
        nv = has2 ? 2 : 1;
        bool second = false;  // NR == 4: slots 2,3 hold another pair
        if (NR == 4) {
            if (a.paired) {
                rows[2] = g.wq2 + (size_t)r * rb;
                scl[2] = g.ws2 + (size_t)r * ng;
                rows[3] = rows[2] + rb;
                scl[3] = scl[2] + ng;
                nv = 4;
            } else if (p + 1 < p1 && r + 3 < g.rows) {
                rows[2] = rows[0] + 2 * rb;
                scl[2] = scl[0] + 2 * ng;
                rows[3] = rows[0] + 3 * rb;
                scl[3] = scl[0] + 3 * ng;
                nv = 4;
                npairs = 2;
                second = true;
            }
        }
        float v[NR][NB];
#pragma unroll
        for (int i = 0; i < NR; ++i)
#pragma unroll
            for (int b = 0; b < NB; ++b) v[i][b] = 0.0f;
        block_dot<KIND, NB, CPG, NR>(rows, scl, nv, ng, n, xsm, xs, xsum, lane, v);
        float u[2][NB];
#pragma unroll
        for (int b = 0; b < NB; ++b) u[0][b] = u[1][b] = 0.0f;
        if (a.paired && NR == 2) {
            const uint8_t* rows2[2] = {g.wq2 + (size_t)r * rb, g.wq2 + (size_t)(r + 1) * rb};
            const float* scl2[2] = {g.ws2 + (size_t)r * ng, g.ws2 + (size_t)(r + 1) * ng};
            float t[2][NB];
#pragma unroll
            for (int b = 0; b < NB; ++b) t[0][b] = t[1][b] = 0.0f;
            block_dot<KIND, NB, CPG, 2>(rows2, scl2, has2 ? 2 : 1, ng, n, xsm, xs, xsum, lane, t);
#pragma unroll
            for (int b = 0; b < NB; ++b) {
                u[0][b] = t[0][b];
                u[1][b] = t[1][b];
            }
        } else if (a.paired) {
#pragma unroll
            for (int b = 0; b < NB; ++b) {
                u[0][b] = v[2 % NR][b];
                u[1][b] = v[3 % NR][b];
            }
        }
#pragma unroll
        for (int i = 0; i < NR; ++i)
#pragma unroll
            for (int b = 0; b < NB; ++b) v[i][b] = warp_sum(v[i][b]);
#pragma unroll
        for (int b = 0; b < NB; ++b) {
            u[0][b] = warp_sum(u[0][b]);
            u[1][b] = warp_sum(u[1][b]);
        }
        if (lane == 0) {
#pragma unroll
            for (int b = 0; b < NB; ++b) {
                finish_rows(a, g, b, r, v[0][b], v[1][b], u[0][b], u[1][b], has2);
                if (second) finish_rows(a, g, b, r + 2, v[2 % NR][b], v[3 % NR][b], 0.0f, 0.0f, true);
            }
        }
        p += npairs;
    }
}

// ---------------------------------------------------------------------------
// host side

static bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

static bool gs_ok(int gs) { return gs == 32 || gs == 64 || gs == 128 || gs == 256; }

bool gemv_args_ok(const GemvArgs& a, int kind) {
    if (!gs_ok(a.gs) || a.cols % a.gs || a.nseg < 1 || a.nseg > kMaxSegs) return false;
    for (int i = 0; i < a.nseg; ++i) {
        if (!aligned16(a.seg[i].wq)) return false;
        if (a.paired && !aligned16(a.seg[i].wq2)) return false;
    }
    return true;
}

template <int KIND, int NB, int CPG>
static cudaError_t launch_cpg(GemvArgs a, cudaStream_t st, bool pdl, int num_sms, int ctas_per_sm) {
    a.x_bytes = align_up(a.nb * a.cols, 16);
    a.nstages = 0;
    a.wcap = a.scap = 0;
    int P = 0;
    for (int i = 0; i < a.nseg; ++i) P += (a.seg[i].rows + 1) / 2;
    if (P == 0) return cudaSuccess;
    const Layout L = make_layout(a);
    auto kern = gemv_kernel<KIND, NB, CPG>;
    static int set_bytes = 0;
    if (L.total > 48 * 1024 && L.total > set_bytes) {
        cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024);
        if (e != cudaSuccess) return e;
        set_bytes = 227 * 1024;
    }
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cudaLaunchConfig_t cfg = {};
    int grid = (P + kW - 1) / kW;
    if (grid > num_sms * ctas_per_sm) grid = num_sms * ctas_per_sm;
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(kGemvThreads);
    cfg.dynamicSmemBytes = L.total;
    cfg.stream = st;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, kern, a, pdl ? 1 : 0);
}

template <int KIND, int NB>
static cudaError_t launch_nb(const GemvArgs& a, cudaStream_t st, bool pdl, int num_sms, int cps) {
    const int cpg = (KIND == 8 ? a.gs : a.gs / 2) / 16;
    switch (cpg) {
        case 1: return launch_cpg<KIND, NB, 1>(a, st, pdl, num_sms, cps);
        case 2: return launch_cpg<KIND, NB, 2>(a, st, pdl, num_sms, cps);
        case 4: return launch_cpg<KIND, NB, 4>(a, st, pdl, num_sms, cps);
        case 8: return launch_cpg<KIND, NB, 8>(a, st, pdl, num_sms, cps);
        default: return launch_cpg<KIND, NB, 16>(a, st, pdl, num_sms, cps);
    }
}

static int g_ctas_per_sm = 0;

cudaError_t gemv_launch(GemvArgs a, int kind, cudaStream_t st, bool pdl, int num_sms) {
    if (!gemv_args_ok(a, kind)) return cudaErrorInvalidValue;
    if (!g_ctas_per_sm) {
        const char* e = getenv("LQ_GEMV_CTAS_PER_SM");
        g_ctas_per_sm = e ? atoi(e) : 4;
        if (g_ctas_per_sm < 1 || g_ctas_per_sm > 8) g_ctas_per_sm = 4;
    }
    const int cps = g_ctas_per_sm;
    if (kind == 8) {
        switch (a.nb) {
            case 1: return launch_nb<8, 1>(a, st, pdl, num_sms, cps);
            case 2: return launch_nb<8, 2>(a, st, pdl, num_sms, cps);
            case 4: return launch_nb<8, 4>(a, st, pdl, num_sms, cps);
            case 8: return launch_nb<8, 8>(a, st, pdl, num_sms, cps);
        }
    } else {
        switch (a.nb) {
            case 1: return launch_nb<4, 1>(a, st, pdl, num_sms, cps);
            case 2: return launch_nb<4, 2>(a, st, pdl, num_sms, cps);
            case 4: return launch_nb<4, 4>(a, st, pdl, num_sms, cps);
            case 8: return launch_nb<4, 8>(a, st, pdl, num_sms, cps);
        }
    }
    return cudaErrorInvalidValue;
}

}  // namespace lq
