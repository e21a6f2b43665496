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
#include <cfloat>
#include <cstdio>
#include <cstdlib>

#include "lq_device.cuh"
#include "lq_epilogue.cuh"
#include "lq_kernels.h"
#include "lq_math.h"
#include "lq_ops.h"

namespace lq {

constexpr int kW = kConsumerWarps;
constexpr int kCT = kW * 32;

__host__ __device__ inline int align_up(int v, int a) { return (v + a - 1) / a * a; }

// The stand-alone activation quantizer's thread count.  The rmsnorm sum of
// squares is defined by its reduction order (256 threads, thread t takes
// float4 chunks t, t+256, ...; warps summed in order), which the GEMV
// prologue reproduces whatever its own thread count.
constexpr int kAqThreads = 256;
constexpr int kRedFloats = kAqThreads + 8;  // shared reduction scratch of the prologue

struct Layout {
    int off_bars, off_red, off_x, off_xs, off_xsum, off_stage, stage_bytes, total;
};

__host__ __device__ inline Layout make_layout(const GemvArgs& a) {
    Layout L;
    const int ng = a.cols / a.gs;
    L.off_bars = 0;
    L.off_red = align_up(a.nstages * 8, 16);
    L.off_x = align_up(L.off_red + kRedFloats * 4, 128);
    L.off_xs = align_up(L.off_x + a.x_bytes, 16);
    L.off_xsum = align_up(L.off_xs + a.nb * ng * 4, 16);
    L.off_stage = align_up(L.off_xsum + a.nb * ng * 4, 128);
    L.stage_bytes = a.wcap + a.scap;
    L.total = L.off_stage + a.nstages * L.stage_bytes;
    return L;
}

__host__ __device__ inline bool gs_ok_dev(int gs) { return gs == 32 || gs == 64 || gs == 128 || gs == 256; }

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

// rmsnorm scale 1/sqrt(mean(x^2) + 1e-5) (v1-int8-vnni/runq.c:294-305) with
// the sum of squares associated exactly as act_quant_kernel associates it:
// virtual thread t (0..255) takes float4 chunks t, t+256, ... with fmaf,
// each virtual warp is summed by the xor butterfly, the eight warp sums are
// added in order.  nt real threads (any multiple of 32) stand in for the 256.
__device__ float rms_inv_aq(const float* src, int n, float* red, int ctid, int nt) {
    const int nc = n >> 2;
    for (int vt = ctid; vt < kAqThreads; vt += nt) {
        float ss = 0.0f;
        int c = vt;
        for (; c + 3 * kAqThreads < nc; c += 4 * kAqThreads) {
            float4 q[4];
#pragma unroll
            for (int u = 0; u < 4; ++u) q[u] = reinterpret_cast<const float4*>(src)[c + u * kAqThreads];
#pragma unroll
            for (int u = 0; u < 4; ++u) {
                ss = fmaf(q[u].x, q[u].x, ss);
                ss = fmaf(q[u].y, q[u].y, ss);
                ss = fmaf(q[u].z, q[u].z, ss);
                ss = fmaf(q[u].w, q[u].w, ss);
            }
        }
        for (; c < nc; c += kAqThreads) {
            const float4 q = reinterpret_cast<const float4*>(src)[c];
            ss = fmaf(q.x, q.x, ss);
            ss = fmaf(q.y, q.y, ss);
            ss = fmaf(q.z, q.z, ss);
            ss = fmaf(q.w, q.w, ss);
        }
        red[vt] = ss;
    }
    named_bar_sync(1, nt);
    if (ctid < 32) {
        float t = 0.0f;
        for (int w = 0; w < kAqThreads / 32; ++w) t += warp_sum(red[w * 32 + ctid]);
        if (ctid == 0) red[kAqThreads] = t;
    }
    named_bar_sync(1, nt);
    const float t = red[kAqThreads];
    named_bar_sync(1, nt);  // red is reused by the next activation row
    return 1.0f / sqrtf(t / (float)n + 1e-5f);
}

// Build the int8 activation of the launch's rows in shared memory: group
// sums and scales for groups [g0, g1) of every row (all groups when the CTA
// is not part of a cluster; a cluster's CTAs then exchange their slices).
template <int KIND>
__device__ void stage_input(const GemvArgs& a, int8_t* xsm, float* xs, int* xsum, float* red, int ctid, int nt,
                            int g0, int g1) {
    const int n = a.cols, gs = a.gs, ng = n / gs;
    if (a.in_mode == IN_QUANT) {
        // copy int8 rows (INT4: split into even/odd planes), 8 bytes a step;
        // every load of this thread is issued before any store
        const int upr = (g1 - g0) * gs / 8;  // 8-byte units of one row's slice
        const int total8 = a.nb * upr;
        constexpr int U = 4;
        for (int i0 = ctid; i0 < total8; i0 += U * nt) {
            uint2 v[U];
#pragma unroll
            for (int u = 0; u < U; ++u) {
                const int i = i0 + u * nt;
                if (i < total8) {
                    const int b = i / upr, k0 = g0 * gs + (i - b * upr) * 8;
                    v[u] = *reinterpret_cast<const uint2*>(a.xq + (size_t)b * n + k0);
                }
            }
#pragma unroll
            for (int u = 0; u < U; ++u) {
                const int i = i0 + u * nt;
                if (i >= total8) break;
                const int b = i / upr, k0 = g0 * gs + (i - b * upr) * 8;
                int8_t* xrow = xsm + (size_t)b * n;
                if (KIND == 4) {
                    *reinterpret_cast<uint32_t*>(xrow + (k0 >> 1)) = __byte_perm(v[u].x, v[u].y, 0x6420);
                    *reinterpret_cast<uint32_t*>(xrow + (n >> 1) + (k0 >> 1)) = __byte_perm(v[u].x, v[u].y, 0x7531);
                } else {
                    *reinterpret_cast<uint2*>(xrow + k0) = v[u];
                }
            }
        }
        const int sg = g1 - g0;
        if (a.xsum_in) {
            for (int i = ctid; i < a.nb * sg; i += nt) {
                const int g = (i / sg) * ng + g0 + i % sg;
                xs[g] = a.xs[g];
                xsum[g] = a.xsum_in[g];
            }
        } else {
            named_bar_sync(1, nt);
            // group sums from the staged copy (INT4: the group's even and odd
            // values are two contiguous runs of gs/2 bytes, one per plane)
            for (int i = ctid; i < a.nb * sg; i += nt) {
                const int b = i / sg, gg = g0 + i % sg, g = b * ng + gg;
                const int8_t* xrow = xsm + (size_t)b * n;
                int s = 0;
                if (KIND == 4) {
                    const int* p0 = reinterpret_cast<const int*>(xrow + gg * (gs / 2));
                    const int* p1 = reinterpret_cast<const int*>(xrow + (n >> 1) + gg * (gs / 2));
                    for (int j = 0; j < gs / 8; ++j) s = __dp4a(p1[j], 0x01010101, __dp4a(p0[j], 0x01010101, s));
                } else {
                    const int* p0 = reinterpret_cast<const int*>(xrow + gg * gs);
                    for (int j = 0; j < gs / 4; ++j) s = __dp4a(p0[j], 0x01010101, s);
                }
                xs[g] = a.xs[g];
                xsum[g] = s;
            }
        }
        return;
    }
    // quantize_act (runq.c:117-139), optionally after rmsnorm: thread t of a
    // pass takes 8 consecutive values; a group spans gs/8 consecutive lanes,
    // whose max and sum come from xor shuffles.  The loop is kept rolled (one
    // copy of its body): these kernels are short, and every instruction of
    // the prologue is fetched cold.
    const bool norm = a.in_mode == IN_RMSNORM || a.in_mode == IN_RMSNORM_EMB;
    const int lpg = gs / 8;   // lanes per group: 4, 8, 16 or 32
    const int nvalid = (a.nvalid > 0 && a.nvalid < a.nb) ? a.nvalid : a.nb;
    for (int b = 0; b < a.nb; ++b) {
        int8_t* xrow = xsm + (size_t)b * n;
        if (b >= nvalid) {
            // padding row of a partial chunk: its inputs (and its token) lie
            // past the caller's rows, and its results are not stored
            for (int i = ctid * 16; i < n; i += nt * 16) *reinterpret_cast<uint4*>(xrow + i) = make_uint4(0, 0, 0, 0);
            for (int g = ctid; g < ng; g += nt) {
                xs[b * ng + g] = 0.0f;
                xsum[b * ng + g] = 0;
            }
            continue;
        }
        const float* src = a.xf ? a.xf + (size_t)b * n : nullptr;
        if (a.in_mode == IN_RMSNORM_EMB) {
            const int token = a.meta[2 * b];
            src = a.emb + (size_t)token * n;
            if (blockIdx.x == 0)
                for (int i = ctid; i < n; i += nt) a.x_out[(size_t)b * n + i] = src[i];
        }
        const float inv = norm ? rms_inv_aq(src, n, red, ctid, nt) : 1.0f;
        // software pipelined: the next pass's loads are issued before this
        // pass's arithmetic (tasks of groups [g0, g1) only)
        float4 c0 = make_float4(0.f, 0.f, 0.f, 0.f), c1 = c0;
        const int t_end = g1 * lpg;
        if (g0 * lpg + ctid < t_end) {
            c0 = *reinterpret_cast<const float4*>(src + (g0 * lpg + ctid) * 8);
            c1 = *reinterpret_cast<const float4*>(src + (g0 * lpg + ctid) * 8 + 4);
        }
#pragma unroll 1
        for (int base = g0 * lpg; base < t_end; base += nt) {
            const int t = base + ctid;
            const bool on = t < t_end;
            float v[8] = {c0.x, c0.y, c0.z, c0.w, c1.x, c1.y, c1.z, c1.w};
            const int tn = t + nt;
            if (tn < t_end) {
                c0 = *reinterpret_cast<const float4*>(src + tn * 8);
                c1 = *reinterpret_cast<const float4*>(src + tn * 8 + 4);
            }
            const int k0 = (on ? t : 0) * 8;
            if (norm && on) {
                // rmsnorm scaling w * (inv * x), as act_quant_kernel applies it
                const float4 w0 = *reinterpret_cast<const float4*>(a.rms_w + k0);
                const float4 w1 = *reinterpret_cast<const float4*>(a.rms_w + k0 + 4);
                const float w[8] = {w0.x, w0.y, w0.z, w0.w, w1.x, w1.y, w1.z, w1.w};
#pragma unroll
                for (int i = 0; i < 8; ++i) v[i] = w[i] * (inv * v[i]);
            }
            float amax = 0.0f;
#pragma unroll
            for (int i = 0; i < 8; ++i) amax = fmaxf(amax, fabsf(v[i]));
            for (int o = 1; o < lpg; o <<= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
            float sc = amax / 127.0f;
            if (sc == 0.0f) sc = 1e-8f;
            const float rcp = 1.0f / sc;
            int qs = 0;
            if (on) {
                int q[8];
#pragma unroll
                for (int i = 0; i < 8; ++i) {
                    q[i] = max(-127, min(127, quant_div(v[i], sc, rcp)));
                    qs += q[i];
                }
                uint32_t lo, hi;
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
        // w ^ 0x88.. turns each two's-complement nibble into q+8; the low
        // nibbles dot the even plane, the high nibbles (kept in place, i.e.
        // 16*(q+8)) dot the odd plane into a second sum that is 16x
        const uint32_t L4 = 0x0F0F0F0Fu, H4 = 0xF0F0F0F0u;
        const uint32_t a0 = w.x ^ 0x88888888u, a1 = w.y ^ 0x88888888u, a2 = w.z ^ 0x88888888u,
                       a3 = w.w ^ 0x88888888u;
        int dl = dp4a_us(a0 & L4, xe.x, 0);
        int dh = dp4a_us(a0 & H4, xo.x, 0);
        dl = dp4a_us(a1 & L4, xe.y, dl);
        dh = dp4a_us(a1 & H4, xo.y, dh);
        dl = dp4a_us(a2 & L4, xe.z, dl);
        dh = dp4a_us(a2 & H4, xo.z, dh);
        dl = dp4a_us(a3 & L4, xe.w, dl);
        dh = dp4a_us(a3 & H4, xo.w, dh);
        return d + dl + (dh >> 4);
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

// epilogue (rope_pair, finish_rows): lq_epilogue.cuh

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
    kt_start(a.kt);
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
    kt_waited(a.kt);
    stage_input<KIND>(a, xsm, xs, xsum, red, threadIdx.x, blockDim.x, 0, ng);
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
    kt_end_cta(a.kt);
}

// ---------------------------------------------------------------------------
// the bulk-copy (TMA) kernel, used when every scale row starts on a 16-byte
// boundary (group count a multiple of 4, true for every Llama shape)
//
// One CTA per SM, eight warps.  Warp w of the grid owns the contiguous pair
// range [w*P/W, (w+1)*P/W) and runs its own two-slot copy pipeline: lane 0
// issues 1-D bulk copies (cp.async.bulk, the TMA engine) of the warp's next
// item into a free slot, the warp computes the other slot from shared
// memory.  An item is either K whole row pairs (short rows; one contiguous
// copy per tensor) or one slice of both rows of a pair (long rows).  The
// first two items are requested at kernel start — before the activation
// prologue and, inside a model, before griddepcontrol.wait — so the weight
// stream overlaps everything else.

constexpr int kTmaMaxWarps = 16;
constexpr int kSlotW = 8192;  // weight bytes per slot (all tensors)

struct TItem {
    int seg, row, nrows, boff, bytes;  // rows [row, row+nrows) of segment seg; slice [boff, boff+bytes)
    bool last;                         // last slice of the pair (or whole rows)
};

// walks a warp's items in order; identical in every lane
struct TIter {
    int p, p1, j;  // pair index, end, slice index
};

__device__ __forceinline__ bool titem_next(const GemvArgs& a, TIter& it, int rb, TItem& o) {
    if (it.p >= it.p1) return false;
    int seg = 0, p = it.p, np = a.seg[0].rows >> 1;
    while (p >= np) {
        p -= np;
        ++seg;
        np = a.seg[seg].rows >> 1;
    }
    o.seg = seg;
    o.row = 2 * p;
    if (!a.split) {
        const int k = min(min(a.stage_rows >> 1, np - p), it.p1 - it.p);
        o.nrows = 2 * k;
        o.boff = 0;
        o.bytes = o.nrows * rb;
        o.last = true;
        it.p += k;
    } else {
        o.nrows = 2;
        o.boff = it.j * a.slice_bytes;
        o.bytes = min(a.slice_bytes, rb - o.boff);
        o.last = o.boff + o.bytes == rb;
        if (o.last) {
            it.j = 0;
            ++it.p;
        } else {
            ++it.j;
        }
    }
    return true;
}

__device__ __forceinline__ void titem_issue(const GemvArgs& a, const TItem& it, uint8_t* slot, uint64_t* bar, int rb,
                                            int ng, int gb, int tw, uint64_t pol) {
    const GemvSeg& g = a.seg[it.seg];
    const int mult = a.paired ? 2 : 1;
    const int sb = (it.bytes / gb) * 4;  // scale bytes per row slice
    uint8_t* sdst = slot + kSlotW;        // scales follow the weights
    if (!a.split) {
        const uint32_t wbytes = (uint32_t)(it.nrows * rb), sbytes = (uint32_t)(it.nrows * ng * 4);
        mbar_arrive_expect_tx(bar, mult * (wbytes + sbytes));
        bulk_g2s(slot, g.wq + (size_t)it.row * rb, wbytes, bar, pol);
        bulk_g2s(sdst, g.ws + (size_t)it.row * ng, sbytes, bar, pol);
        if (a.paired) {
            bulk_g2s(slot + tw, g.wq2 + (size_t)it.row * rb, wbytes, bar, pol);
            bulk_g2s(sdst + sbytes, g.ws2 + (size_t)it.row * ng, sbytes, bar, pol);
        }
    } else {
        const int region = a.scap / (2 * mult);  // scale bytes reserved per (tensor, row)
        mbar_arrive_expect_tx(bar, (uint32_t)(mult * 2 * (it.bytes + sb)));
        for (int t = 0; t < mult; ++t) {
            const uint8_t* wq = t ? g.wq2 : g.wq;
            const float* ws = t ? g.ws2 : g.ws;
            for (int h = 0; h < 2; ++h) {
                const int r = it.row + h;
                bulk_g2s(slot + t * tw + h * (tw / 2), wq + (size_t)r * rb + it.boff, (uint32_t)it.bytes, bar, pol);
                bulk_g2s(sdst + (t * 2 + h) * region, ws + (size_t)r * ng + it.boff / gb, (uint32_t)sb, bar, pol);
            }
        }
    }
}

// one warp, one row (slice) in shared memory: lane owns groups lane,
// lane+32, ...; chunks read in a lane-rotated order (bank-conflict free)
template <int KIND, int NB, int CPG>
__device__ __forceinline__ void smem_row_dot(const uint8_t* w, const float* sc, int g0, int ngs, const int8_t* xsm,
                                             const float* xs, const int* xsum, int n, int ng, int lane,
                                             float acc[NB]) {
    constexpr int BIAS = KIND == 8 ? 128 : 8;
    const int rot = CPG >= 8 ? (lane & 7) : ((lane * CPG) >> 3) & (CPG - 1);
    for (int gl = lane; gl < ngs; gl += 32) {
        const uint8_t* wg = w + (size_t)gl * CPG * 16;
        const int g = g0 + gl;
        int d0[NB], d1[NB];
#pragma unroll
        for (int b = 0; b < NB; ++b) d0[b] = d1[b] = 0;
#pragma unroll
        for (int k = 0; k < CPG; ++k) {
            const int kk = (k + rot) & (CPG - 1);
            const uint4 wv = *reinterpret_cast<const uint4*>(wg + 16 * kk);
#pragma unroll
            for (int b = 0; b < NB; ++b) {
                if (k & 1) d1[b] = chunk_dot<KIND>(wv, xsm + (size_t)b * n, g * CPG + kk, n, d1[b]);
                else d0[b] = chunk_dot<KIND>(wv, xsm + (size_t)b * n, g * CPG + kk, n, d0[b]);
            }
        }
        const float sw = sc[gl];
#pragma unroll
        for (int b = 0; b < NB; ++b) {
            const int D = d0[b] + d1[b] - BIAS * xsum[b * ng + g];
            acc[b] = fmaf(sw * xs[b * ng + g], (float)D, acc[b]);
        }
    }
}

// R rows (slices of equal length) at once: the activation chunk is read
// once for all R rows, and the R integer chains run side by side.
template <int KIND, int NB, int CPG, int R>
__device__ __forceinline__ void smem_rows_dot(const uint8_t* const* w, const float* const* sc, int g0, int ngs,
                                              const int8_t* xsm, const float* xs, const int* xsum, int n, int ng,
                                              int lane, float (*acc)[NB]) {
    constexpr int BIAS = KIND == 8 ? 128 : 8;
    const int rot = CPG >= 8 ? (lane & 7) : ((lane * CPG) >> 3) & (CPG - 1);
    for (int gl = lane; gl < ngs; gl += 32) {
        const int g = g0 + gl;
        int d[R][NB];
#pragma unroll
        for (int r = 0; r < R; ++r)
#pragma unroll
            for (int b = 0; b < NB; ++b) d[r][b] = 0;
#pragma unroll
        for (int k = 0; k < CPG; ++k) {
            const int kk = (k + rot) & (CPG - 1);
            const int c = g * CPG + kk;
            uint4 wv[R];
#pragma unroll
            for (int r = 0; r < R; ++r) wv[r] = *reinterpret_cast<const uint4*>(w[r] + ((size_t)gl * CPG + kk) * 16);
#pragma unroll
            for (int b = 0; b < NB; ++b) {
                const int8_t* xrow = xsm + (size_t)b * n;
                if (KIND == 8) {
                    const uint4 x = *reinterpret_cast<const uint4*>(xrow + 16 * c);
#pragma unroll
                    for (int r = 0; r < R; ++r) {
                        int t = dp4a_us(wv[r].x, x.x, d[r][b]);
                        t = dp4a_us(wv[r].y, x.y, t);
                        t = dp4a_us(wv[r].z, x.z, t);
                        d[r][b] = dp4a_us(wv[r].w, x.w, t);
                    }
                } else {
                    const uint4 xe = *reinterpret_cast<const uint4*>(xrow + 16 * c);
                    const uint4 xo = *reinterpret_cast<const uint4*>(xrow + (n >> 1) + 16 * c);
                    const uint32_t L4 = 0x0F0F0F0Fu, H4 = 0xF0F0F0F0u;
#pragma unroll
                    for (int r = 0; r < R; ++r) {
                        const uint32_t a0 = wv[r].x ^ 0x88888888u, a1 = wv[r].y ^ 0x88888888u,
                                       a2 = wv[r].z ^ 0x88888888u, a3 = wv[r].w ^ 0x88888888u;
                        int dl = dp4a_us(a0 & L4, xe.x, 0);
                        int dh = dp4a_us(a0 & H4, xo.x, 0);
                        dl = dp4a_us(a1 & L4, xe.y, dl);
                        dh = dp4a_us(a1 & H4, xo.y, dh);
                        dl = dp4a_us(a2 & L4, xe.z, dl);
                        dh = dp4a_us(a2 & H4, xo.z, dh);
                        dl = dp4a_us(a3 & L4, xe.w, dl);
                        dh = dp4a_us(a3 & H4, xo.w, dh);
                        d[r][b] += dl + (dh >> 4);
                    }
                }
            }
        }
#pragma unroll
        for (int b = 0; b < NB; ++b) {
            const float xsc = xs[b * ng + g];
            const int xsu = BIAS * xsum[b * ng + g];
#pragma unroll
            for (int r = 0; r < R; ++r) acc[r][b] = fmaf(sc[r][gl] * xsc, (float)(d[r][b] - xsu), acc[r][b]);
        }
    }
}

// SPLIT / PAIRED: the launch's a.split and a.paired, fixed per instantiation
// so that each kernel holds only the one dot loop it runs
template <int KIND, int NB, int CPG, bool SPLIT, bool PAIRED>
__global__ void __launch_bounds__(kTmaMaxWarps * 32, 1) gemv_tma_kernel(const __grid_constant__ GemvArgs a, int prefetch) {
    extern __shared__ __align__(128) uint8_t smem[];
    pdl_trigger();
    const Layout L = make_layout(a);
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + L.off_bars);
    float* red = reinterpret_cast<float*>(smem + L.off_red);
    int8_t* xsm = reinterpret_cast<int8_t*>(smem + L.off_x);
    float* xs = reinterpret_cast<float*>(smem + L.off_xs);
    int* xsum = reinterpret_cast<int*>(smem + L.off_xsum);
    const int n = a.cols, ng = n / a.gs;
    const int rb = KIND == 8 ? n : n / 2;
    const int gb = KIND == 8 ? a.gs : a.gs / 2;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int tw = PAIRED ? kSlotW / 2 : kSlotW;  // weight bytes per tensor in a slot
    int P = 0;
    for (int i = 0; i < a.nseg; ++i) P += a.seg[i].rows >> 1;
    const int nw = blockDim.x >> 5;
    const long long W = (long long)gridDim.x * nw, wg = (long long)blockIdx.x * nw + warp;
    TIter iss = {(int)(wg * P / W), (int)((wg + 1) * P / W), 0};
    TIter cmp = iss;
    uint64_t* bar = full + 2 * warp;
    uint8_t* slots = smem + L.off_stage + (size_t)warp * 2 * L.stage_bytes;
    uint64_t* tr = a.trace ? a.trace + (size_t)blockIdx.x * 4 : nullptr;
    if (tr && threadIdx.x == 0) tr[0] = globaltimer();
    kt_start(a.kt);

    if (lane == 0) {
        mbar_init(&bar[0], 1);
        mbar_init(&bar[1], 1);
    }
    fence_mbar_init();
    __syncwarp();
    uint64_t pol = 0;
    TItem it;
    if (lane == 0) {
        // `prefetch` of the warp's two first items are requested before the
        // wait for the previous kernel, the rest after it
        pol = l2_evict_first_policy();
        for (int s = 0; s < 2 && titem_next(a, iss, rb, it); ++s) {
            if (s == prefetch) pdl_wait();
            titem_issue(a, it, slots + (size_t)s * L.stage_bytes, &bar[s], rb, ng, gb, tw, pol);
        }
    }
    pdl_wait();
    kt_waited(a.kt);
    if (tr && threadIdx.x == 0) tr[1] = globaltimer();
    stage_input<KIND>(a, xsm, xs, xsum, red, threadIdx.x, blockDim.x, 0, ng);
    __syncthreads();
    if (tr && threadIdx.x == 0) tr[2] = globaltimer();
    // every lane walks the issue iterator too (lane 0 already advanced it)
    if (lane != 0)
        for (int s = 0; s < 2 && titem_next(a, iss, rb, it); ++s) {
        }

    float acc[2][NB], acc2[2][NB];
#pragma unroll
    for (int b = 0; b < NB; ++b) acc[0][b] = acc[1][b] = acc2[0][b] = acc2[1][b] = 0.0f;
    for (int k = 0; titem_next(a, cmp, rb, it); ++k) {
        const int s = k & 1;
        // the decision to give up is warp-uniform: the lanes then leave the
        // loop together (no lane is left inside a warp-wide shuffle)
        if (!__all_sync(0xffffffffu, mbar_wait(&bar[s], (k >> 1) & 1, a.err, DEV_TIMEOUT_FULL))) {
            // give up: confirm the copy of the other slot too, then leave
            if (lane == 0) mbar_wait(&bar[s ^ 1], ((k + 1) >> 1) & 1, a.err, DEV_TIMEOUT_DRAIN);
            break;
        }
        const uint8_t* sw = slots + (size_t)s * L.stage_bytes;
        const float* ss = reinterpret_cast<const float*>(sw + kSlotW);
        const GemvSeg& g = a.seg[it.seg];
        if (!SPLIT) {
            const float* ss2 = ss + it.nrows * ng;
            for (int r = 0; r < it.nrows; r += 2) {
                float v[4][NB];
#pragma unroll
                for (int q = 0; q < 4; ++q)
#pragma unroll
                    for (int b = 0; b < NB; ++b) v[q][b] = 0.0f;
                if (PAIRED) {
                    const uint8_t* wr[4] = {sw + (size_t)r * rb, sw + (size_t)(r + 1) * rb, sw + tw + (size_t)r * rb,
                                            sw + tw + (size_t)(r + 1) * rb};
                    const float* sr[4] = {ss + (size_t)r * ng, ss + (size_t)(r + 1) * ng, ss2 + (size_t)r * ng,
                                          ss2 + (size_t)(r + 1) * ng};
                    smem_rows_dot<KIND, NB, CPG, 4>(wr, sr, 0, ng, xsm, xs, xsum, n, ng, lane, v);
                } else {
                    const uint8_t* wr[2] = {sw + (size_t)r * rb, sw + (size_t)(r + 1) * rb};
                    const float* sr[2] = {ss + (size_t)r * ng, ss + (size_t)(r + 1) * ng};
                    smem_rows_dot<KIND, NB, CPG, 2>(wr, sr, 0, ng, xsm, xs, xsum, n, ng, lane, v);
                }
#pragma unroll
                for (int q = 0; q < (PAIRED ? 4 : 2); ++q)
#pragma unroll
                    for (int b = 0; b < NB; ++b) v[q][b] = warp_sum(v[q][b]);
                if (lane == 0) {
#pragma unroll
                    for (int b = 0; b < NB; ++b) finish_rows(a, g, b, it.row + r, v[0][b], v[1][b], v[2][b], v[3][b], true);
                }
            }
        } else {
            const int g0 = it.boff / gb, ngs = it.bytes / gb;
            const int mult = PAIRED ? 2 : 1;
            const int region = a.scap / (2 * mult);
            const uint8_t* sb = reinterpret_cast<const uint8_t*>(ss);
            float tmp[4][NB];
#pragma unroll
            for (int q = 0; q < 4; ++q)
#pragma unroll
                for (int b = 0; b < NB; ++b) tmp[q][b] = 0.0f;
            if (PAIRED) {
                const uint8_t* wr[4] = {sw, sw + tw / 2, sw + tw, sw + tw + tw / 2};
                const float* sr[4] = {reinterpret_cast<const float*>(sb), reinterpret_cast<const float*>(sb + region),
                                      reinterpret_cast<const float*>(sb + 2 * region),
                                      reinterpret_cast<const float*>(sb + 3 * region)};
                smem_rows_dot<KIND, NB, CPG, 4>(wr, sr, g0, ngs, xsm, xs, xsum, n, ng, lane, tmp);
            } else {
                const uint8_t* wr[2] = {sw, sw + tw / 2};
                const float* sr[2] = {reinterpret_cast<const float*>(sb), reinterpret_cast<const float*>(sb + region)};
                smem_rows_dot<KIND, NB, CPG, 2>(wr, sr, g0, ngs, xsm, xs, xsum, n, ng, lane, tmp);
            }
#pragma unroll
            for (int b = 0; b < NB; ++b) {
                acc[0][b] += tmp[0][b];
                acc[1][b] += tmp[1][b];
                acc2[0][b] += tmp[2][b];
                acc2[1][b] += tmp[3][b];
            }
            if (it.last) {
#pragma unroll
                for (int b = 0; b < NB; ++b) {
                    const float v0 = warp_sum(acc[0][b]), v1 = warp_sum(acc[1][b]);
                    const float u0 = PAIRED ? warp_sum(acc2[0][b]) : 0.0f, u1 = PAIRED ? warp_sum(acc2[1][b]) : 0.0f;
                    acc[0][b] = acc[1][b] = acc2[0][b] = acc2[1][b] = 0.0f;
                    if (lane == 0) finish_rows(a, g, b, it.row, v0, v1, u0, u1, true);
                }
            }
        }
        // refill this slot with the warp's item k + 2
        __syncwarp();
        TItem nx;
        const bool more = titem_next(a, iss, rb, nx);
        if (lane == 0 && more) {
            asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
            titem_issue(a, nx, slots + (size_t)s * L.stage_bytes, &bar[s], rb, ng, gb, tw, pol);
        }
    }
    kt_end_cta(a.kt);
    if (tr) {
        __syncthreads();
        if (threadIdx.x == 0) tr[3] = globaltimer();
    }
}

// ---------------------------------------------------------------------------
// stand-alone activation quantization (one pass, many CTAs): each thread
// takes 8 consecutive values, gs/8 lanes form a group; rmsnorm CTAs each
// compute the full sum of squares in the same fixed order.

// One task = 8 consecutive values of activation row b (gs/8 consecutive
// tasks, inside one warp, form a quantization group): optional rmsnorm
// scaling w * (inv * v), then quantize_act (runq.c:117-139) and store the
// int8 values, the group scale and the group sum.
__device__ __forceinline__ void quant_task8(const ActQuantArgs& a, int b, int task, bool on, bool norm, float inv,
                                            float (&v)[8]) {
    const int n = a.n, gs = a.gs, ng = n / gs;
    const int lpg = gs / 8;
    const int k0 = (on ? task : 0) * 8;
    float amax = 0.0f;
    if (on) {
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
    if (on) {
        int q[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            q[i] = max(-127, min(127, quant_div(v[i], sc, rcp)));
            qs += q[i];
        }
        const uint32_t lo = (q[0] & 0xFF) | ((q[1] & 0xFF) << 8) | ((q[2] & 0xFF) << 16) | ((uint32_t)(q[3] & 0xFF) << 24);
        const uint32_t hi = (q[4] & 0xFF) | ((q[5] & 0xFF) << 8) | ((q[6] & 0xFF) << 16) | ((uint32_t)(q[7] & 0xFF) << 24);
        *reinterpret_cast<uint2*>(a.xq + (size_t)b * n + k0) = make_uint2(lo, hi);
    }
    for (int o = 1; o < lpg; o <<= 1) qs += __shfl_xor_sync(0xffffffffu, qs, o);
    if (on && (task & (lpg - 1)) == 0) {
        const int g = task / lpg;
        a.xs[(size_t)b * ng + g] = sc;
        a.xsum[(size_t)b * ng + g] = qs;
        if (a.xs_t) {
            const int c = b >> 6, ld = c < a.xs_nfull ? 64 : a.xs_npad_last;
            a.xs_t[(size_t)c * ng * 64 + (size_t)g * ld + (b & 63)] = sc * a.xs_t_mul;
        }
    }
}

__global__ void __launch_bounds__(kAqThreads) act_quant_kernel(const __grid_constant__ ActQuantArgs a) {
    __shared__ float red[kAqThreads / 32];
    pdl_trigger();
    kt_start(a.kt);
    pdl_wait();
    kt_waited(a.kt);
    const int b = blockIdx.y, n = a.n, gs = a.gs, ng = n / gs;
    const int ctid = threadIdx.x;
    const float* src = a.x ? a.x + (size_t)b * n : nullptr;
    if (a.mode == IN_RMSNORM_EMB) {
        src = a.emb + (size_t)a.meta[2 * b] * n;
        if (blockIdx.x == 0)
            for (int i = ctid; i < n; i += kAqThreads) a.x_out[(size_t)b * n + i] = src[i];
    }
    // residual add (tensor-parallel step: y is the all-reduced partial); x_out
    // is a different buffer from x, so every CTA reads the unmodified x
    const bool add = a.mode == IN_ADD_RMSNORM;
    const float* yrow = add ? a.y + (size_t)b * n : nullptr;
    if (add && blockIdx.x == 0)
        for (int i = ctid; i < n; i += kAqThreads) a.x_out[(size_t)b * n + i] = src[i] + yrow[i];
    const bool norm = a.mode == IN_RMSNORM || a.mode == IN_RMSNORM_EMB || add;
    float inv = 1.0f;
    if (norm) {
        // rmsnorm sum of squares: thread t takes float4 chunks t, t+256, ...
        // (all of a row of up to 8192 values loaded at once)
        constexpr int U = 8;
        float ss = 0.0f;
        for (int c0 = ctid; c0 < n / 4; c0 += U * kAqThreads) {
            float4 v[U];
#pragma unroll
            for (int u = 0; u < U; ++u) {
                const int c = c0 + u * kAqThreads;
                v[u] = c < n / 4 ? reinterpret_cast<const float4*>(src)[c] : make_float4(0.f, 0.f, 0.f, 0.f);
                if (add && c < n / 4) {
                    const float4 w = reinterpret_cast<const float4*>(yrow)[c];
                    v[u].x += w.x;
                    v[u].y += w.y;
                    v[u].z += w.z;
                    v[u].w += w.w;
                }
            }
#pragma unroll
            for (int u = 0; u < U; ++u) {
                ss = fmaf(v[u].x, v[u].x, ss);
                ss = fmaf(v[u].y, v[u].y, ss);
                ss = fmaf(v[u].z, v[u].z, ss);
                ss = fmaf(v[u].w, v[u].w, ss);
            }
        }
        ss = warp_sum(ss);
        if ((ctid & 31) == 0) red[ctid >> 5] = ss;
        __syncthreads();
        float t = 0.0f;
#pragma unroll
        for (int w = 0; w < kAqThreads / 32; ++w) t += red[w];
        inv = 1.0f / sqrtf(t / (float)n + 1e-5f);
    }
    const int task = blockIdx.x * kAqThreads + ctid;  // 8 values per task
    const bool on = task < ng * (gs / 8);
    const int k0 = (on ? task : 0) * 8;
    float v[8];
    if (on) {
        const float4 a0 = *reinterpret_cast<const float4*>(src + k0);
        const float4 a1 = *reinterpret_cast<const float4*>(src + k0 + 4);
        v[0] = a0.x; v[1] = a0.y; v[2] = a0.z; v[3] = a0.w;
        v[4] = a1.x; v[5] = a1.y; v[6] = a1.z; v[7] = a1.w;
        if (add) {
            const float4 y0 = *reinterpret_cast<const float4*>(yrow + k0);
            const float4 y1 = *reinterpret_cast<const float4*>(yrow + k0 + 4);
            v[0] += y0.x; v[1] += y0.y; v[2] += y0.z; v[3] += y0.w;
            v[4] += y1.x; v[5] += y1.y; v[6] += y1.z; v[7] += y1.w;
        }
    }
    quant_task8(a, b, task, on, norm, inv, v);
    kt_end_cta(a.kt);
}

cudaError_t act_quant_launch(const ActQuantArgs& a, cudaStream_t st, bool pdl) {
    if (!gs_ok_dev(a.gs) || a.n % a.gs || a.n % 8) return cudaErrorInvalidValue;
    const int tasks = a.n / 8;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((tasks + kAqThreads - 1) / kAqThreads, a.nb);
    cfg.blockDim = dim3(kAqThreads);
    cfg.stream = st;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, act_quant_kernel, a);
}

// ---------------------------------------------------------------------------
// attention merge + quantize: a thread per value of the row, a CTA per 256
// values (whole quantization groups: gs divides 256).
//
// Merge (the split-KV merge order, runq.c:369-391 restated for chunks of
// kChunk positions): M = max over the chunks of m_s; w_s = exp(m_s - M);
// L = sum over the chunks in order of fmaf(l_s, w_s, L); o = sum over the
// chunks in order of fmaf(o_s, w_s, o); value = o / L.  The chunk values of
// one output are loaded in batches of kMergeBatch independent loads.
constexpr int kMergeBatch = 48;

__global__ void __launch_bounds__(kAqThreads) attn_quant_kernel(const __grid_constant__ AttnQuantArgs aa) {
    extern __shared__ float msm[];  // [nhc][max_splits] maxima, then weights; [nhc][max_splits] sums; [nhc] L
    __shared__ float gmax_w[kAqThreads / 32];
    __shared__ int gsum_w[kAqThreads / 32];
    const ActQuantArgs& a = aa.q;
    pdl_trigger();
    kt_start(a.kt);
    pdl_wait();
    kt_waited(a.kt);
    const int b = blockIdx.y, n = a.n, gs = a.gs, ng = n / gs, hs = aa.head_size;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int k0 = blockIdx.x * kAqThreads, k = k0 + tid;
    const bool on = k < n;
    const int nsplit = a.meta[2 * b + 1] / kChunk + 1;
    float v = 0.0f;
    if (nsplit == 1) {
        if (on) v = a.x[(size_t)b * n + k];
    } else {
        const int ms = aa.max_splits, ps = hs + 4;
        const int h0 = k0 / hs, h1 = (min(k0 + kAqThreads, n) - 1) / hs, nhc = h1 - h0 + 1;
        float* mw = msm;             // [nhc][ms]
        float* lw = msm + nhc * ms;  // [nhc][ms]
        float* Ls = lw + nhc * ms;   // [nhc]
        const float* prow = aa.part + (size_t)b * (n / hs) * ms * ps;
        // this thread's output's chunk values: the first batch is loaded
        // before the per-head weights are known, so both wait for one round
        const int hh_k = k / hs - h0, d_k = k - (k / hs) * hs;
        const float* src = prow + (size_t)(h0 + hh_k) * ms * ps + 4 + d_k;
        float x[kMergeBatch];
#pragma unroll
        for (int u = 0; u < kMergeBatch; ++u) x[u] = on && u < nsplit ? __ldcg(src + (size_t)u * ps) : 0.0f;
        for (int i = tid; i < nhc * nsplit; i += kAqThreads) {
            const int hh = i / nsplit, s2 = i - hh * nsplit;
            const float2 m_l = __ldcg(reinterpret_cast<const float2*>(prow + ((size_t)(h0 + hh) * ms + s2) * ps));
            mw[hh * ms + s2] = m_l.x;
            lw[hh * ms + s2] = m_l.y;
        }
        __syncthreads();
        for (int hh = warp; hh < nhc; hh += kAqThreads / 32) {
            float M = -FLT_MAX;
            for (int s2 = lane; s2 < nsplit; s2 += 32) M = fmaxf(M, mw[hh * ms + s2]);
            M = warp_max(M);
            for (int s2 = lane; s2 < nsplit; s2 += 32) mw[hh * ms + s2] = lq_expf(mw[hh * ms + s2] - M);
            __syncwarp();
            if (lane == 0) {
                float L = 0.0f;
                for (int s2 = 0; s2 < nsplit; ++s2) L = fmaf(lw[hh * ms + s2], mw[hh * ms + s2], L);
                Ls[hh] = L;
            }
        }
        __syncthreads();
        if (on) {
            const float* w = mw + hh_k * ms;
            float o = 0.0f;
            for (int s0 = 0; s0 < nsplit; s0 += kMergeBatch) {
                if (s0 > 0) {
#pragma unroll
                    for (int u = 0; u < kMergeBatch; ++u)
                        x[u] = s0 + u < nsplit ? __ldcg(src + (size_t)(s0 + u) * ps) : 0.0f;
                }
#pragma unroll
                for (int u = 0; u < kMergeBatch; ++u)
                    if (s0 + u < nsplit) o = fmaf(x[u], w[s0 + u], o);
            }
            v = o / Ls[hh_k];
        }
    }
    // quantize as quant_task8 does: group absmax, scale amax / 127, values
    // quant_div(v, scale) clamped to [-127, 127], group sum of the values
    const int wpg = gs / 32;  // warps per group
    const int gw0 = (warp / wpg) * wpg;
    float amax = warp_max(on ? fabsf(v) : 0.0f);
    if (lane == 0) gmax_w[warp] = amax;
    __syncthreads();
    amax = 0.0f;
    for (int w2 = 0; w2 < wpg; ++w2) amax = fmaxf(amax, gmax_w[gw0 + w2]);
    float sc = amax / 127.0f;
    if (sc == 0.0f) sc = 1e-8f;
    const float rcp = 1.0f / sc;
    const int q = on ? max(-127, min(127, quant_div(v, sc, rcp))) : 0;
    if (on) a.xq[(size_t)b * n + k] = (int8_t)q;
    int qs = q;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) qs += __shfl_xor_sync(0xffffffffu, qs, o);
    if (lane == 0) gsum_w[warp] = qs;
    __syncthreads();
    if (on && (k & (gs - 1)) == 0) {
        int tot = 0;
        for (int w2 = 0; w2 < wpg; ++w2) tot += gsum_w[gw0 + w2];
        const int g = k / gs;
        a.xs[(size_t)b * ng + g] = sc;
        a.xsum[(size_t)b * ng + g] = tot;
        if (a.xs_t) {
            const int c = b >> 6, ld = c < a.xs_nfull ? 64 : a.xs_npad_last;
            a.xs_t[(size_t)c * ng * 64 + (size_t)g * ld + (b & 63)] = sc * a.xs_t_mul;
        }
    }
    kt_end_cta(a.kt);
}

cudaError_t attn_quant_launch(const AttnQuantArgs& a, cudaStream_t st, bool pdl) {
    const int n = a.q.n, hs = a.head_size;
    if (!gs_ok_dev(a.q.gs) || n % a.q.gs || hs < 1 || n % hs || a.max_splits < 1) return cudaErrorInvalidValue;
    const int nhc = kAqThreads / hs + 2;
    const size_t smem = sizeof(float) * ((size_t)2 * nhc * a.max_splits + nhc);
    static size_t set_bytes = 0;
    if (smem > 48 * 1024 && smem > set_bytes) {
        cudaError_t e = cudaFuncSetAttribute(attn_quant_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        if (e != cudaSuccess) return e;
        set_bytes = smem;
    }
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((n + kAqThreads - 1) / kAqThreads, a.q.nb);
    cfg.blockDim = dim3(kAqThreads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, attn_quant_kernel, a);
}

// ---------------------------------------------------------------------------
// tensor-parallel all-reduce + residual add + rmsnorm + quantize (one CTA per
// activation row; protocol in lq_kernels.h)

constexpr int kPeerMaxN = 8192;  // one CTA of at most 1024 threads, 8 values each

__global__ void __launch_bounds__(1024) peer_add_quant_kernel(const __grid_constant__ PeerAddArgs pa) {
    extern __shared__ __align__(16) float srow[];  // x + y of this row [n]
    __shared__ float red[kAqThreads / 32];
    __shared__ uint32_t s_call;
    const ActQuantArgs& a = pa.q;
    pdl_trigger();
    kt_start(a.kt);
    pdl_wait();  // this process's partial (the previous kernel's output) is complete
    kt_waited(a.kt);
    const int b = blockIdx.y, n = a.n, ctid = threadIdx.x;
    if (ctid == 0) {
        const uint32_t e = *reinterpret_cast<volatile const uint32_t*>(&pa.counters[0]) + 1u;
        s_call = e;
        __threadfence();
        // the last CTA to read the call number advances it for the next call
        if (atomicAdd(&pa.counters[1], 1u) == gridDim.y - 1) {
            pa.counters[1] = 0;
            pa.counters[0] = e;
        }
    }
    __syncthreads();
    const uint32_t e = s_call;
    // once a wait has given up (this call or an earlier one of the step), the
    // step's result is void: no further waits, so the host hears of it after
    // one limit, not one per call
    bool failed = *reinterpret_cast<volatile const int*>(pa.err) != 0;
    const uint64_t limit = pa.wait_ns ? pa.wait_ns : kWaitLimitNs;
    // y = sum of the processes' partials in rank order, x_out = x + y (8
    // values per thread); each process's 8 words are polled until all carry
    // this call's number
    const int task = ctid;
    const bool on = task < n / 8;
    const int k0 = task * 8;
    const size_t off = (size_t)b * n + k0;
    float v[8];
    if (on) {
        float y[8];
        for (int p = 0; p < pa.tp_size; ++p) {
            const uint64_t* src = pa.slot + ((size_t)p * pa.ll_rows + b) * n + k0;
            uint64_t wd[8];
            uint64_t t0 = 0;
            for (uint32_t it = 0;; ++it) {
#pragma unroll
                for (int h = 0; h < 4; ++h) ld_relaxed_sys_v2(src + 2 * h, wd[2 * h], wd[2 * h + 1]);
                bool ready = true;
#pragma unroll
                for (int i = 0; i < 8; ++i) ready = ready && (uint32_t)(wd[i] >> 32) == e;
                if (ready || failed) break;
                if (it == 0) t0 = globaltimer();
                if ((it & 15u) == 15u) {
                    failed = *reinterpret_cast<volatile const int*>(pa.err) != 0;
                    if (!failed && globaltimer() - t0 > limit) {
                        set_err(pa.err, DEV_TIMEOUT_PEER);
                        failed = true;
                    }
                }
            }
#pragma unroll
            for (int i = 0; i < 8; ++i) {
                const float z = __uint_as_float((uint32_t)wd[i]);
                y[i] = p == 0 ? z : y[i] + z;
            }
        }
        const float4 x0 = *reinterpret_cast<const float4*>(a.x + off);
        const float4 x1 = *reinterpret_cast<const float4*>(a.x + off + 4);
        v[0] = x0.x + y[0]; v[1] = x0.y + y[1]; v[2] = x0.z + y[2]; v[3] = x0.w + y[3];
        v[4] = x1.x + y[4]; v[5] = x1.y + y[5]; v[6] = x1.z + y[6]; v[7] = x1.w + y[7];
        const float4 r0 = make_float4(v[0], v[1], v[2], v[3]), r1 = make_float4(v[4], v[5], v[6], v[7]);
        *reinterpret_cast<float4*>(a.x_out + off) = r0;
        *reinterpret_cast<float4*>(a.x_out + off + 4) = r1;
        *reinterpret_cast<float4*>(srow + k0) = r0;
        *reinterpret_cast<float4*>(srow + k0 + 4) = r1;
    }
    __syncthreads();
    // rmsnorm sum of squares in act_quant_kernel's order: 256 threads, thread
    // t takes float4 chunks t, t+256, ...; warps summed in order
    if (ctid < kAqThreads) {
        float ss = 0.0f;
        for (int c = ctid; c < n / 4; c += kAqThreads) {
            const float4 q = reinterpret_cast<const float4*>(srow)[c];
            ss = fmaf(q.x, q.x, ss);
            ss = fmaf(q.y, q.y, ss);
            ss = fmaf(q.z, q.z, ss);
            ss = fmaf(q.w, q.w, ss);
        }
        ss = warp_sum(ss);
        if ((ctid & 31) == 0) red[ctid >> 5] = ss;
    }
    __syncthreads();
    float t = 0.0f;
#pragma unroll
    for (int w = 0; w < kAqThreads / 32; ++w) t += red[w];
    const float inv = 1.0f / sqrtf(t / (float)n + 1e-5f);
    quant_task8(a, b, task, on, true, inv, v);
    kt_end_cta(a.kt);
}

cudaError_t peer_add_quant_launch(const PeerAddArgs& a, cudaStream_t st, bool pdl) {
    const int n = a.q.n;
    if (!gs_ok_dev(a.q.gs) || n % a.q.gs || n % 8 || n > kPeerMaxN || a.tp_size < 1 || a.tp_size > kTpMax ||
        a.q.nb < 1 || a.q.nb > a.ll_rows || !a.slot || !a.counters)
        return cudaErrorInvalidValue;
    const int threads = kAqThreads * ((n / 8 + kAqThreads - 1) / kAqThreads);
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(1, a.q.nb);
    cfg.blockDim = dim3(threads);
    cfg.dynamicSmemBytes = (size_t)n * sizeof(float);
    cfg.stream = st;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, peer_add_quant_kernel, a);
}

// ---------------------------------------------------------------------------
// host side

static bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

static bool gs_ok(int gs) { return gs_ok_dev(gs); }

bool gemv_args_ok(const GemvArgs& a, int kind) {
    if (!gs_ok(a.gs) || a.cols % a.gs || a.nseg < 1 || a.nseg > kMaxSegs) return false;
    if (a.cols % 8) return false;
    for (int i = 0; i < a.nseg; ++i) {
        if (!aligned16(a.seg[i].wq)) return false;
        if (a.paired && !aligned16(a.seg[i].wq2)) return false;
    }
    return true;
}

static bool tma_ok(const GemvArgs& a) {
    if ((a.cols / a.gs) % 4) return false;
    for (int i = 0; i < a.nseg; ++i) {
        if (a.seg[i].rows % 2) return false;
        if (!aligned16(a.seg[i].wq) || !aligned16(a.seg[i].ws)) return false;
        if (a.paired && (!aligned16(a.seg[i].wq2) || !aligned16(a.seg[i].ws2))) return false;
    }
    return true;
}

static int g_use_tma = -1;

// Shared-memory budget per bulk-copy GEMV CTA: two CTAs (of consecutive
// kernels) fit one SM's 228 KB with 1 KB reserved each.  LQ_GEMV_SMEM_KB
// overrides it (for tuning).
template <int KIND, int NB, int CPG>
static cudaError_t launch_tma(GemvArgs a, cudaStream_t st, bool pdl, int num_sms) {
    const int rb = KIND == 8 ? a.cols : a.cols / 2;
    const int gb = KIND == 8 ? a.gs : a.gs / 2;
    const int ng = a.cols / a.gs;
    const int mult = a.paired ? 2 : 1;
    const int tw = kSlotW / mult;
    a.x_bytes = align_up(a.nb * a.cols, 16);
    a.wcap = kSlotW;
    if (2 * rb <= tw) {
        a.split = 0;
        a.stage_rows = 2 * (tw / (2 * rb));
        a.slice_bytes = 0;
        a.scap = align_up(mult * a.stage_rows * ng * 4, 128);
    } else {
        a.split = 1;
        a.stage_rows = 2;
        a.slice_bytes = tw / 2;
        a.scap = align_up(2 * mult * align_up(a.slice_bytes / gb * 4, 16), 128);
    }
    int P = 0;
    for (int i = 0; i < a.nseg; ++i) P += a.seg[i].rows / 2;
    if (P == 0) return cudaSuccess;
    // as many warps (two slots each) as shared memory holds, up to 16
    int nw = 0;
    for (int w = kTmaMaxWarps; w >= 4 && !nw; w -= 2) {
        a.nstages = 2 * w;
        if (make_layout(a).total <= 227 * 1024) nw = w;
    }
    if (!nw) return cudaErrorInvalidValue;
    a.nstages = 2 * nw;
    const Layout L = make_layout(a);
    void (*kern)(GemvArgs, int) = a.split ? (a.paired ? gemv_tma_kernel<KIND, NB, CPG, true, true>
                                                     : gemv_tma_kernel<KIND, NB, CPG, true, false>)
                                          : (a.paired ? gemv_tma_kernel<KIND, NB, CPG, false, true>
                                                      : gemv_tma_kernel<KIND, NB, CPG, false, false>);
    static bool attr_set[2][2] = {};
    if (!attr_set[a.split][a.paired]) {
        cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024);
        if (e != cudaSuccess) return e;
        attr_set[a.split][a.paired] = true;
    }
    cudaLaunchConfig_t cfg = {};
    int grid = (P + nw - 1) / nw;
    if (grid > num_sms) grid = num_sms;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(nw * 32);
    cfg.dynamicSmemBytes = L.total;
    cfg.stream = st;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, kern, a, pdl ? 2 : 0);
}

template <int KIND, int NB, int CPG>
static cudaError_t launch_cpg(GemvArgs a, cudaStream_t st, bool pdl, int num_sms, int ctas_per_sm) {
    if (g_use_tma < 0) {
        const char* e = getenv("LQ_GEMV_TMA");
        g_use_tma = e ? atoi(e) : 1;
    }
    if (g_use_tma && tma_ok(a)) {
        const int rb = KIND == 8 ? a.cols : a.cols / 2;
        (void)rb;
        GemvArgs t = a;
        t.x_bytes = align_up(a.nb * a.cols, 16);
        if (make_layout(t).off_stage + 2 * 4 * (kSlotW + 4096) <= 227 * 1024)
            return launch_tma<KIND, NB, CPG>(a, st, pdl, num_sms);
    }
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
    if (a.nvalid <= 0 || a.nvalid > a.nb) a.nvalid = a.nb;
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
