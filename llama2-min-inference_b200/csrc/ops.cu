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
// heads of its kv head (GQA: K/V are read from HBM once) and writes each
// head's unnormalised partial (max m, sum l, o[hs]).  A single chunk writes
// the normalised output directly; otherwise the activation quantizer in
// front of the wo product merges the partials (attn_quant_kernel).  The
// output stays fp32 until that quantizer (runq.c:394 order: quantize the
// normalised output — not v5's unnormalised-scale variant).

// Butterfly step that halves the values a lane holds: lanes with bit `o` set
// keep the upper half of in[], the others the lower half, and each adds the
// half its partner (lane ^ o) sent.  For value i of a lane that kept the
// lower half the sum is in[i] + partner's in[i]; every sum pairs the same two
// lane values as a plain xor butterfly over that head would.
template <int C>
__device__ __forceinline__ void halve(const float (&in)[C], float (&out)[C / 2], int o, int lane) {
    const bool up = (lane & o) != 0;
#pragma unroll
    for (int i = 0; i < C / 2; ++i) {
        const float send = up ? in[i] : in[i + C / 2];
        const float keep = up ? in[i + C / 2] : in[i];
        out[i] = keep + __shfl_xor_sync(0xffffffffu, send, o);
    }
}

// Sum over the 32 lanes of KM values per lane (one per head), as KM xor
// butterflies (l + l^16, then 8, 4, 2, 1 apart) would each add them.  The
// head whose sum a lane ends with: head_of_lane<KM>(lane).
template <int KM>
__device__ __forceinline__ float multi_warp_sum(const float (&v)[KM], int lane) {
    if constexpr (KM == 1) {
        return warp_sum(v[0]);
    } else {
        float h[KM / 2];
        halve<KM>(v, h, 16, lane);
        if constexpr (KM == 2) {
            return warp_sum_below(h[0], 8);
        } else {
            float g[KM / 4];
            halve<KM / 2>(h, g, 8, lane);
            if constexpr (KM == 4) {
                return warp_sum_below(g[0], 4);
            } else {
                static_assert(KM == 8, "KM in {1, 2, 4, 8}");
                float f[1];
                halve<2>(g, f, 4, lane);
                return warp_sum_below(f[0], 2);
            }
        }
    }
}
template <int KM>
__device__ __forceinline__ int head_of_lane(int lane) {
    // bit 16 picks the upper half of the heads, bit 8 the upper half of the rest, ...
    return KM == 1 ? 0 : KM == 2 ? (lane >> 4) : KM == 4 ? (lane >> 3) : (lane >> 2);
}

// NT threads per CTA.  KM = kv_mul when it is 1, 2, 4 or 8 and head_size <=
// 128 (queries held in registers, the heads of a position reduced together);
// KM = 0 for any other shape (queries in shared memory, one head at a time).
// Both keep one arithmetic order.
template <int NT, int KM>
__global__ void __launch_bounds__(NT, 1024 / NT) attention_kernel(const __grid_constant__ AttnArgs a) {
    extern __shared__ __align__(16) unsigned char araw[];
    __shared__ __align__(8) uint64_t kv_bar;
    pdl_trigger();
    kt_start(a.kt);
    const int kvh = blockIdx.x, split = blockIdx.y, b = blockIdx.z;
    const int hs = a.head_size, km = KM ? KM : a.kv_mul;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    constexpr int NW = NT / 32;
    // the positions were written before the step's first kernel started, so
    // they can be read before waiting for the preceding kernel
    const int pos = a.meta[2 * b + 1];
    const int nsplit = pos / kChunk + 1;
    if (split >= nsplit) return;
    const int t0 = split * kChunk;
    const int nt = min(kChunk, pos + 1 - t0);

    // K of the chunk in nreg regions of kChunk rows x 128 bytes (dims 32m ..
    // 32m+31 of every position), each written by one tensor copy with the
    // 128-byte swizzle: 16-byte chunk c of row t sits at chunk c ^ (t & 7), so
    // a warp reading one row, or one chunk of 8 consecutive rows, meets no
    // bank conflict.  The swizzle needs 1024-byte aligned regions.
    const int nreg = (hs + 31) / 32;
    unsigned char* kbase = araw + ((1024 - (smem_addr(araw) & 1023u)) & 1023u);
    float* vs = reinterpret_cast<float*>(kbase + (size_t)nreg * kChunk * 128);  // [kChunk][hs]
    float* qs = vs + kChunk * hs;          // [km][hs] (KM = 0)
    float* sc = qs + (KM ? 0 : km * hs);   // [km][kChunk] scores, then weights
    float* ml = sc + km * kChunk;          // [km][2]

    // K by nreg tensor copies, V by one bulk copy (the chunk's positions are
    // contiguous rows of the cache).  A chunk without the current position
    // holds only earlier steps' keys and values, so its copies start before
    // the preceding kernel (which writes position pos) is done.
    const size_t cbase = (size_t)b * a.kv_seq_stride + ((size_t)kvh * a.max_seq + t0) * hs;
    const uint32_t vbytes = (uint32_t)(nt * hs * sizeof(float));
    if (tid == 0) {
        mbar_init(&kv_bar, 1);
        fence_mbar_init();
        if (t0 + nt - 1 == pos) pdl_wait();
        const uint64_t pol = l2_evict_first_policy();
        mbar_arrive_expect_tx(&kv_bar, (uint32_t)nreg * kChunk * 128 + vbytes);
        const int row = (int)(a.krow + (int64_t)(cbase / hs));
        for (int m = 0; m < nreg; ++m)
            tma_load_2d(kbase + (size_t)m * kChunk * 128, &a.kmap, 128 * m, row, &kv_bar, pol);
        bulk_g2s(vs, a.vcache + cbase, vbytes, &kv_bar, pol);
    }
    pdl_wait();
    kt_waited(a.kt);
    const float* qg = a.q + (size_t)b * a.q_stride + (size_t)kvh * km * hs;
    // dim lane + 32m of row t: region m, 16-byte chunk lane / 4 (swizzled), word lane % 4
    auto kval = [&](int t, int m) {
        return *reinterpret_cast<const float*>(kbase + (size_t)m * kChunk * 128 + t * 128 +
                                               ((((lane >> 2) ^ (t & 7)) << 4) | ((lane & 3) << 2)));
    };

    // scores q_j . k_t / sqrt(hs), the reference's warp-reduction order: 32
    // partial sums (partial l takes dims l, l+32, ... in increasing order with
    // fmaf; here lane l), added as an xor butterfly over the 32 lanes.  A warp
    // per position.
    const float rs = sqrtf((float)hs);
    if constexpr (KM > 0) {
        float qr[KM][4];
#pragma unroll
        for (int j = 0; j < KM; ++j)
#pragma unroll
            for (int m = 0; m < 4; ++m) qr[j][m] = lane + 32 * m < hs ? qg[j * hs + lane + 32 * m] : 0.0f;
        __syncthreads();  // orders the barrier's initialisation before the waits below
        const bool landed = mbar_wait(&kv_bar, 0, a.err, DEV_TIMEOUT_FULL);
        if (!__syncthreads_and(landed)) {
            // give up on this chunk; confirm the copies before the CTA's shared memory is released
            if (tid == 0) mbar_wait(&kv_bar, 0, a.err, DEV_TIMEOUT_DRAIN);
            return;
        }
        // a pass of a warp takes P = 8 / KM positions: 8 dot products (P
        // positions x KM heads) reduced together; lane group v = lane / 4
        // ends with dot v = (position p, head j), v = p * KM + j
        constexpr int P = 8 / KM;
        const int v = head_of_lane<8>(lane), pv = v / KM, jv = v - pv * KM;
        const bool writer = (lane & 3) == 0;
        for (int t0w = warp * P; t0w < nt; t0w += NW * P) {
            float acc[8];
#pragma unroll
            for (int i = 0; i < 8; ++i) acc[i] = 0.0f;
#pragma unroll
            for (int m = 0; m < 4; ++m) {
                if (lane + 32 * m < hs) {
#pragma unroll
                    for (int p = 0; p < P; ++p) {
                        // rows past the chunk's positions hold other data: read, never stored
                        const float kv = kval(t0w + p < kChunk ? t0w + p : kChunk - 1, m);
#pragma unroll
                        for (int j = 0; j < KM; ++j) acc[p * KM + j] = fmaf(qr[j][m], kv, acc[p * KM + j]);
                    }
                }
            }
            const float dot = multi_warp_sum<8>(acc, lane);
            if (writer && t0w + pv < nt) sc[jv * kChunk + t0w + pv] = dot / rs;
        }
    } else {
        for (int i = tid; i < km * hs; i += NT) qs[i] = qg[i];
        __syncthreads();
        const bool landed = mbar_wait(&kv_bar, 0, a.err, DEV_TIMEOUT_FULL);
        if (!__syncthreads_and(landed)) {
            if (tid == 0) mbar_wait(&kv_bar, 0, a.err, DEV_TIMEOUT_DRAIN);
            return;
        }
        for (int t = warp; t < nt; t += NW) {
            for (int j = 0; j < km; ++j) {
                float acc = 0.0f;
                for (int m = 0; m < nreg; ++m)
                    if (lane + 32 * m < hs) acc = fmaf(qs[j * hs + lane + 32 * m], kval(t, m), acc);
                acc = warp_sum(acc);
                if (lane == 0) sc[j * kChunk + t] = acc / rs;
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
    // o[j][d] = sum_t p[j][t] * v[t][d] in position order with fmaf.  The
    // unnormalised partial of head j: [m, l, -, -, o[hs]] (o 16-byte aligned)
    float* out = a.out + (size_t)b * a.q_stride + (size_t)kvh * km * hs;
    const int hq0 = kvh * km;
    auto partial = [&](int j) {
        return a.part + (((size_t)b * a.n_heads + hq0 + j) * a.max_splits + split) * (hs + 4);
    };
    if (KM >= 2) {
        // a thread per 4 dims of 2 heads
        const int nd4 = hs / 4;
        for (int i = tid; i < nd4 * (km / 2); i += NT) {
            const int jp = i / nd4, d = (i - jp * nd4) * 4, j = 2 * jp;
            const float* p0 = sc + j * kChunk;
            const float* p1 = p0 + kChunk;
            float o[8];
#pragma unroll
            for (int u = 0; u < 8; ++u) o[u] = 0.0f;
#pragma unroll 4
            for (int t = 0; t < nt; ++t) {
                const float4 v = *reinterpret_cast<const float4*>(vs + t * hs + d);
                const float a0 = p0[t], a1 = p1[t];
                o[0] = fmaf(a0, v.x, o[0]);
                o[1] = fmaf(a0, v.y, o[1]);
                o[2] = fmaf(a0, v.z, o[2]);
                o[3] = fmaf(a0, v.w, o[3]);
                o[4] = fmaf(a1, v.x, o[4]);
                o[5] = fmaf(a1, v.y, o[5]);
                o[6] = fmaf(a1, v.z, o[6]);
                o[7] = fmaf(a1, v.w, o[7]);
            }
#pragma unroll
            for (int h = 0; h < 2; ++h) {
                const float* oh = o + 4 * h;
                if (nsplit == 1) {
                    const float L = ml[2 * (j + h) + 1];
                    *reinterpret_cast<float4*>(out + (j + h) * hs + d) =
                        make_float4(oh[0] / L, oh[1] / L, oh[2] / L, oh[3] / L);
                } else {
                    float* pp = partial(j + h);
                    *reinterpret_cast<float4*>(pp + 4 + d) = make_float4(oh[0], oh[1], oh[2], oh[3]);
                    if (d == 0) {
                        pp[0] = ml[2 * (j + h)];
                        pp[1] = ml[2 * (j + h) + 1];
                    }
                }
            }
        }
    } else {
        // a thread per (head, dim)
        for (int i = tid; i < km * hs; i += NT) {
            const int j = i / hs, d = i - j * hs;
            const float* pj = sc + j * kChunk;
            float o = 0.0f;
#pragma unroll 8
            for (int t = 0; t < nt; ++t) o = fmaf(pj[t], vs[t * hs + d], o);
            if (nsplit == 1) {
                out[i] = o / ml[2 * j + 1];
            } else {
                float* pp = partial(j);
                pp[4 + d] = o;
                if (d == 0) {
                    pp[0] = ml[2 * j];
                    pp[1] = ml[2 * j + 1];
                }
            }
        }
    }
    kt_end_cta(a.kt);
}

size_t attention_smem_bytes(int head_size, int kv_mul) {
    const size_t kbytes = (size_t)((head_size + 31) / 32) * kChunk * 128;  // swizzled K regions
    return 1024 + kbytes +
           sizeof(float) * ((size_t)kChunk * head_size + (size_t)kv_mul * head_size + (size_t)kv_mul * kChunk +
                            2 * (size_t)kv_mul);
}

namespace {
template <int NT, int KM>
cudaError_t launch_attention(const AttnArgs& a, int batch, cudaStream_t st, bool pdl) {
    const size_t smem = attention_smem_bytes(a.head_size, a.kv_mul);
    auto kern = attention_kernel<NT, KM>;
    static size_t set_bytes = 0;
    if (smem > set_bytes) {
        // the largest shared-memory carveout: with the default the driver may
        // keep one CTA per SM where two fit
        cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        if (e == cudaSuccess)
            e = cudaFuncSetAttribute(kern, cudaFuncAttributePreferredSharedMemoryCarveout, cudaSharedmemCarveoutMaxShared);
        if (e != cudaSuccess) return e;
        set_bytes = smem;
    }
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(a.n_kv_heads, a.max_splits, batch);
    cfg.blockDim = dim3(NT);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, kern, a);
}
}  // namespace

cudaError_t attention_launch(const AttnArgs& a, int batch, cudaStream_t st, bool pdl) {
    if (a.head_size % 4) return cudaErrorInvalidValue;
    if (a.head_size <= 128) {
        switch (a.kv_mul) {
        case 1: return launch_attention<256, 1>(a, batch, st, pdl);
        case 2: return launch_attention<256, 2>(a, batch, st, pdl);
        case 4: return launch_attention<512, 4>(a, batch, st, pdl);
        case 8: return launch_attention<512, 8>(a, batch, st, pdl);
        default: break;
        }
    }
    return launch_attention<512, 0>(a, batch, st, pdl);
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
    // each thread scans its elements in increasing index order; the loads of
    // a pass (8 float4, or 8 scalars when the row is not 16-byte aligned) are
    // issued before the compares
    auto take = [&](float x, int i) {
        if (bi < 0 || x > bv) {
            bv = x;
            bi = i;
        }
    };
    if ((reinterpret_cast<uintptr_t>(v) & 15u) == 0) {
        const int n4 = n / 4;
        const float4* v4 = reinterpret_cast<const float4*>(v);
        for (int c0 = threadIdx.x; c0 < n4; c0 += 8 * blockDim.x) {
            float4 x[8];
#pragma unroll
            for (int u = 0; u < 8; ++u) {
                const int c = c0 + u * blockDim.x;
                x[u] = c < n4 ? v4[c] : make_float4(0.f, 0.f, 0.f, 0.f);
            }
#pragma unroll
            for (int u = 0; u < 8; ++u) {
                const int c = c0 + u * blockDim.x;
                if (c < n4) {
                    take(x[u].x, 4 * c);
                    take(x[u].y, 4 * c + 1);
                    take(x[u].z, 4 * c + 2);
                    take(x[u].w, 4 * c + 3);
                }
            }
        }
        for (int i = 4 * n4 + threadIdx.x; i < n; i += blockDim.x) take(v[i], i);
    } else {
        for (int i0 = threadIdx.x; i0 < n; i0 += 8 * blockDim.x) {
            float x[8];
#pragma unroll
            for (int u = 0; u < 8; ++u) x[u] = i0 + u * blockDim.x < n ? v[i0 + u * blockDim.x] : 0.0f;
#pragma unroll
            for (int u = 0; u < 8; ++u)
                if (i0 + u * blockDim.x < n) take(x[u], i0 + u * blockDim.x);
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
