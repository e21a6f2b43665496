// Batched decode GEMM on the 5th-generation tensor cores: tcgen05.mma
// kind::i8 with int32 accumulators in tensor memory (TMEM), for 16 to 64
// activation rows (B independent sequences, or prompt rows).
//
//   Y[b, r] = sum_g ws[r, g] * xs[b, g] * D[b, r, g],
//   D[b, r, g] = sum_{k in group g} q_w[r, k] * q_x[b, k]      (exact int32)
//
// i.e. the M-row form of matmul_q8 (v1-int8-vnni/runq.c:142-159), the
// semantics of the reference's batched matmul_q8_kernel (v2-cuda/run.cu:131-162).
// The per-group int32 dots are exact; the fp32 epilogue is
// acc = fmaf(ws * xs, (float)D, acc) over the groups in K order.
//
// One persistent CTA per SM, warp-specialised (704 threads):
//   warp 0       TMA producer: per stage (128 bytes of K) the weight tile of
//                128 rows (128 bytes, or the 64 packed bytes of INT4) and the
//                activation tile (npad rows x 128 bytes), 2-D tensor maps
//   warp 1       TMEM allocation and MMA issue: per 32-byte K step one
//                tcgen05.mma (M=128, N=npad, K=32, both operands s8,
//                K-major, 128-byte swizzle); each quantization group
//                accumulates into its own TMEM buffer (a 4-deep ring) and is
//                committed to an mbarrier when its last K step is issued
//   warps 2-5    operand conversion in shared memory: INT8 weights are stored
//                biased (q+128, the file encoding) and become s8 by xor 0x80;
//                INT4 nibbles become s8 bytes holding 16*q (the nibble in the
//                high half), so D comes out as 16*D and the activation scale
//                table carries xs/16 (both scalings are exact)
//   warps 6-21   epilogue: per group, tcgen05.ld of the int32 dots (TMEM lane
//                = weight row, column = activation row), exact int->float via
//                the 1.5*2^23 bias (|D| < 2^22), packed fp32x2 scale and fma
// Work split: stream-K over the sequence of (tile, stage) pairs of the whole
// launch: CTA i owns stages [i*W/G, (i+1)*W/G).  A tile owned by several
// CTAs leaves fp32 partials in global memory; the last CTA to arrive (an
// arrival counter per tile) sums them in stage order and runs the epilogue,
// so the result is deterministic for a given grid size.
//
// Every mbarrier wait is bounded (2 s); a wait that gives up records an
// error code, stops issuing work, lets the other roles run out the same way,
// waits (bounded) for its own copies and MMAs in flight, and frees TMEM.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <cstdio>
#include <cstdlib>
#include <cstring>

#include "lq_device.cuh"
#include "lq_epilogue.cuh"
#include "lq_kernels.h"
#include "lq_ops.h"

namespace lq {

namespace {

constexpr int kMmaWarp0 = 1;
constexpr int kMmaWarps = 2;     // MMA-issuing warps, taking turns by stage
constexpr int kConvWarp0 = kMmaWarp0 + kMmaWarps;
constexpr int kQgThreads = 32 * (kConvWarp0 + 4 + 16);
constexpr int kTileRows = 128;   // MMA M: weight rows per tile
constexpr int kStageK = 128;     // K bytes (int8 elements) per stage
constexpr int kMaxBuf = 8;       // TMEM group-accumulator ring: 8 / MULT buffers
constexpr int kConvWarps = 4;
constexpr int kEpiWarps = 16;
constexpr int kEpiWarp0 = kConvWarp0 + kConvWarps;
constexpr int kXsStages = 8;     // activation-scale ring: one entry (the stage's groups) per stage

enum : int {
    DEV_TIMEOUT_CONV = 0x111,   // MMA waited too long for a converted stage
    DEV_TIMEOUT_TFULL = 0x112,  // epilogue waited too long for a group's dots
    DEV_TIMEOUT_TEMPTY = 0x113, // MMA waited too long for a free TMEM buffer
    DEV_TIMEOUT_MMA = 0x114,    // final MMA completion wait gave up
};

struct QgemmArgs {
    CUtensorMap wmap[kMaxSegs][2];  // weight tiles (second: the paired w3 tensor)
    CUtensorMap xmap;               // activation [rows][cols] int8, boxes of npad rows (zero fill)
    GemvArgs ep;                    // segments and epilogue state; nb = npad, nvalid = real rows
    const float* xs_t;              // [ng][xs_ld] activation scales (already /16 for INT4)
    int xs_ld;
    float* part;                    // [grid][2][mult][npad][128] stream-K partials
    int* cnt;                       // [tiles] arrival counters (zero between launches)
    int tile_start[kMaxSegs + 1];   // first tile of each segment
    int tiles, kst, stages;         // tiles, K stages per row, smem ring depth
};

// ---- PTX wrappers (public PTX ISA: tcgen05, cp.async.bulk.tensor) --------

__device__ __forceinline__ uint64_t l2_evict_last_policy() {
    uint64_t p;
    asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(p));
    return p;
}

__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// Shared-memory matrix descriptor: K-major, 128-byte swizzle, 8-row core
// groups 1024 bytes apart (stride byte offset), version 1 (sm_100).
__device__ __forceinline__ uint64_t smem_desc_sw128(uint32_t addr) {
    return (uint64_t)((addr >> 4) & 0x3FFFu) | ((uint64_t)1 << 16) | ((uint64_t)(1024 >> 4) << 32) |
           ((uint64_t)1 << 46) | ((uint64_t)2 << 61);
}

__device__ __forceinline__ void mma_i8(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                       uint32_t accumulate) {
    asm volatile(
        "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
        " tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n}\n" ::"r"(d_tmem),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
        : "memory");
}

__device__ __forceinline__ void mma_commit(uint64_t* bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                     smem_addr(bar))
                 : "memory");
}

template <int NC>
__device__ __forceinline__ void tmem_ld(uint32_t taddr, int (&d)[NC]);

template <>
__device__ __forceinline__ void tmem_ld<4>(uint32_t taddr, int (&d)[4]) {
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x4.b32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(d[0]), "=r"(d[1]), "=r"(d[2]), "=r"(d[3])
                 : "r"(taddr));
}

template <>
__device__ __forceinline__ void tmem_ld<8>(uint32_t taddr, int (&d)[8]) {
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
                 : "=r"(d[0]), "=r"(d[1]), "=r"(d[2]), "=r"(d[3]), "=r"(d[4]), "=r"(d[5]), "=r"(d[6]),
                   "=r"(d[7])
                 : "r"(taddr));
}

template <>
__device__ __forceinline__ void tmem_ld<16>(uint32_t taddr, int (&d)[16]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
        : "=r"(d[0]), "=r"(d[1]), "=r"(d[2]), "=r"(d[3]), "=r"(d[4]), "=r"(d[5]), "=r"(d[6]), "=r"(d[7]),
          "=r"(d[8]), "=r"(d[9]), "=r"(d[10]), "=r"(d[11]), "=r"(d[12]), "=r"(d[13]), "=r"(d[14]), "=r"(d[15])
        : "r"(taddr));
}

template <>
__device__ __forceinline__ void tmem_ld<32>(uint32_t taddr, int (&d)[32]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
        "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
        : "=r"(d[0]), "=r"(d[1]), "=r"(d[2]), "=r"(d[3]), "=r"(d[4]), "=r"(d[5]), "=r"(d[6]), "=r"(d[7]),
          "=r"(d[8]), "=r"(d[9]), "=r"(d[10]), "=r"(d[11]), "=r"(d[12]), "=r"(d[13]), "=r"(d[14]), "=r"(d[15]),
          "=r"(d[16]), "=r"(d[17]), "=r"(d[18]), "=r"(d[19]), "=r"(d[20]), "=r"(d[21]), "=r"(d[22]), "=r"(d[23]),
          "=r"(d[24]), "=r"(d[25]), "=r"(d[26]), "=r"(d[27]), "=r"(d[28]), "=r"(d[29]), "=r"(d[30]), "=r"(d[31])
        : "r"(taddr));
}

__device__ __forceinline__ void tmem_ld_wait() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

// packed fp32x2 arithmetic (sm_100): two IEEE round-to-nearest results
__device__ __forceinline__ uint64_t f2_pack(float lo, float hi) {
    return (uint64_t)__float_as_uint(lo) | ((uint64_t)__float_as_uint(hi) << 32);
}
__device__ __forceinline__ float f2_lo(uint64_t v) { return __uint_as_float((uint32_t)v); }
__device__ __forceinline__ float f2_hi(uint64_t v) { return __uint_as_float((uint32_t)(v >> 32)); }
__device__ __forceinline__ uint64_t f2_mul(uint64_t a, uint64_t b) {
    uint64_t d;
    asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
    return d;
}
__device__ __forceinline__ uint64_t f2_add(uint64_t a, uint64_t b) {
    uint64_t d;
    asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
    return d;
}
__device__ __forceinline__ uint64_t f2_fma(uint64_t a, uint64_t b, uint64_t c) {
    uint64_t d;
    asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
    return d;
}

// ---- stream-K partition ---------------------------------------------------

__device__ __host__ __forceinline__ int64_t sk_start(int i, int64_t W, int G) { return (int64_t)i * W / G; }
// the CTA whose stage range holds stage s
__device__ __host__ __forceinline__ int sk_owner(int64_t s, int64_t W, int G) {
    return (int)(((s + 1) * G + W - 1) / W - 1);
}

struct Bars {
    uint64_t full[16], conv[16], empty[16], tfull[kMaxBuf], tempty[kMaxBuf], done[kMmaWarps];
    uint64_t xfull[kXsStages], xempty[kXsStages];
    uint32_t tmem_base;
    int abort_flag;
    int last_flag;
};

// wait that returns at once when the CTA has given up; records `code` on timeout
__device__ __forceinline__ bool mbar_test_wait(uint64_t* bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n"
        " selp.u32 %0, 1, 0, p;\n}\n"
        : "=r"(ok)
        : "r"(smem_addr(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}

__device__ __forceinline__ bool qwait(uint64_t* bar, uint32_t parity, int* err, int code, volatile int* abort_flag) {
    if (mbar_test_wait(bar, parity)) return true;  // already complete: no blocking probe
    if (*abort_flag) return false;
    if (mbar_try_wait(bar, parity)) return true;
    const uint64_t t0 = globaltimer();
    for (uint32_t i = 1;; ++i) {
        if (mbar_try_wait(bar, parity)) return true;
        if ((i & 63u) == 0) {
            if (*abort_flag) return false;
            if (globaltimer() - t0 > kWaitLimitNs) {
                set_err(err, code);
                *abort_flag = 1;
                return false;
            }
        }
    }
}

template <int KIND, int N, int MULT>
struct Layout {
    static constexpr int kA = 16384;                       // s8 operand tile, 128 x 128 bytes
    static constexpr int kP = KIND == 4 ? 8192 : 0;        // packed INT4 staging tile, 128 x 64 bytes
    static constexpr int kB = N * kStageK;                 // activation tile
    static constexpr int kStage = MULT * (kA + kP) + kB;   // multiple of 1024
    static constexpr uint32_t kTx = MULT * (KIND == 4 ? kP : kA) + kB;
    static constexpr int kNBuf = 8 / MULT;                 // TMEM group buffers (8 * N columns in all)
    static constexpr int kXsEntry = 4 * N * 4;             // activation scales of one stage (up to 4 groups)
    static constexpr int kXs = kXsStages * kXsEntry;       // activation-scale ring
};

// the epilogue of one finished row pair, out of line: it runs once per tile
// and column, and inlining all its cases would crowd the group loop's registers
__device__ __noinline__ void finish_pair(const GemvArgs& a, const GemvSeg& g, int b, int r, float v0, float v1,
                                         float u0, float u1) {
    finish_rows(a, g, b, r, v0, v1, u0, u1, true);
}

template <int KIND, int N, int MULT>
__global__ void __launch_bounds__(kQgThreads, 1) qgemm_kernel(const __grid_constant__ QgemmArgs a) {
    using Lay = Layout<KIND, N, MULT>;
    constexpr int kNBuf = Lay::kNBuf;
    extern __shared__ __align__(1024) unsigned char qsm_raw[];
    unsigned char* sm = reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(qsm_raw) + 1023) & ~(uintptr_t)1023);
    const int S = a.stages;
    float* xring = reinterpret_cast<float*>(sm + (size_t)S * Lay::kStage);
    Bars* bars = reinterpret_cast<Bars*>(sm + (size_t)S * Lay::kStage + Lay::kXs);
    volatile int* abort_flag = &bars->abort_flag;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int G = gridDim.x;
    const int K = a.kst;
    const int64_t W = (int64_t)a.tiles * K;
    const int64_t s0 = sk_start(blockIdx.x, W, G), s1 = sk_start(blockIdx.x + 1, W, G);
    const int nst = (int)(s1 - s0);  // this CTA's stages
    const int gs = a.ep.gs, gst = kStageK / gs;  // groups per stage
    const int ng = a.ep.cols / gs;
    int* err = a.ep.err;

    auto tileA = [&](int slot, int m) { return sm + (size_t)slot * Lay::kStage + m * Lay::kA; };
    auto tileP = [&](int slot, int m) { return sm + (size_t)slot * Lay::kStage + MULT * Lay::kA + m * Lay::kP; };
    auto tileB = [&](int slot) { return sm + (size_t)slot * Lay::kStage + MULT * (Lay::kA + Lay::kP); };

    if (threadIdx.x == 0) {
        for (int i = 0; i < S; ++i) {
            mbar_init(&bars->full[i], 1);
            mbar_init(&bars->conv[i], kConvWarps);
            mbar_init(&bars->empty[i], 1);
        }
        for (int i = 0; i < kNBuf; ++i) {
            mbar_init(&bars->tfull[i], 1);
            mbar_init(&bars->tempty[i], kEpiWarps);
        }
        for (int i = 0; i < kXsStages; ++i) {
            mbar_init(&bars->xfull[i], 1);
            mbar_init(&bars->xempty[i], kEpiWarps);
        }
        for (int i = 0; i < kMmaWarps; ++i) mbar_init(&bars->done[i], 1);
        bars->abort_flag = 0;
        bars->last_flag = 0;
        fence_mbar_init();
    }
    constexpr int kCols = (kNBuf * N * MULT) < 32 ? 32 : (kNBuf * N * MULT);
    if (warp == kMmaWarp0) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                         smem_addr(&bars->tmem_base)),
                     "r"(kCols)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = bars->tmem_base;
    pdl_trigger();
    kt_start(a.ep.kt);
    pdl_wait();
    kt_waited(a.ep.kt);

    if (warp == 0) {
        // ---------------- TMA producer ----------------
        // Lanes 0 and 1 wait for the stage slot and the scale-ring entry; then
        // one lane per copy issues it (weight tile per tensor, activation
        // tile, the stage's activation scales), so the copies start together.
        // Counters advance incrementally: no division in the loop.
        const uint64_t pw = l2_evict_first_policy(), px = l2_evict_last_policy();
        int slot = 0, xslot = 0;
        uint32_t ph = 0, xph = 0;
        int t = (int)(s0 / K), k = (int)(s0 % K);
        int seg = 0;
        while (seg + 1 < a.ep.nseg && t >= a.tile_start[seg + 1]) ++seg;
        int issued = 0;
        for (; issued < nst; ++issued) {
            bool ok = true;
            if (lane == 0) ok = qwait(&bars->empty[slot], ph ^ 1u, err, DEV_TIMEOUT_EMPTY, abort_flag);
            if (lane == 1) ok = qwait(&bars->xempty[xslot], xph ^ 1u, err, DEV_TIMEOUT_EMPTY, abort_flag);
            if (!__all_sync(0xffffffffu, ok)) break;
            const int row0 = (t - a.tile_start[seg]) * kTileRows;
            if (lane == 0) mbar_arrive_expect_tx(&bars->full[slot], Lay::kTx);
            if (lane == 1) mbar_arrive_expect_tx(&bars->xfull[xslot], gst * N * 4);
            __syncwarp();
            if (lane < MULT) {
                void* dst = KIND == 4 ? (void*)tileP(slot, lane) : (void*)tileA(slot, lane);
                tma_load_2d(dst, &a.wmap[seg][lane], KIND == 4 ? k * (kStageK / 2) : k * kStageK, row0,
                            &bars->full[slot], pw);
            } else if (lane == MULT) {
                tma_load_2d(tileB(slot), &a.xmap, k * kStageK, 0, &bars->full[slot], px);
            } else if (lane == MULT + 1) {
                // scales of the stage's groups: contiguous in the table (row pitch = npad)
                bulk_g2s(xring + xslot * (Lay::kXsEntry / 4), a.xs_t + (size_t)k * gst * N, gst * N * 4,
                         &bars->xfull[xslot], px);
            }
            if (++slot == S) {
                slot = 0;
                ph ^= 1u;
            }
            if (++xslot == kXsStages) {
                xslot = 0;
                xph ^= 1u;
            }
            if (++k == K) {
                k = 0;
                ++t;
                while (seg + 1 < a.ep.nseg && t >= a.tile_start[seg + 1]) ++seg;
            }
        }
        // confirm the copies still in flight (only an aborted run leaves any)
        if (lane == 0 && *abort_flag) {
            for (int j = issued - S; j < issued; ++j) {
                if (j < 0) continue;
                if (!mbar_wait(&bars->full[j % S], (uint32_t)((j / S) & 1), err, DEV_TIMEOUT_DRAIN)) break;
            }
            for (int j = issued - kXsStages; j < issued; ++j) {
                if (j < 0) continue;
                if (!mbar_wait(&bars->xfull[j % kXsStages], (uint32_t)((j / kXsStages) & 1), err, DEV_TIMEOUT_DRAIN))
                    break;
            }
        }
    } else if (warp < kMmaWarp0 + kMmaWarps) {
        // ---------------- MMA issue ----------------
        // kMmaWarps threads take turns by stage (an MMA issue costs the issuing
        // thread more time than the tensor core needs for these small tiles).
        // Per stage: wait for the converted operands and for the stage's last
        // TMEM buffer (the epilogue frees buffers in order), issue the MMAs
        // K-step-major across the stage's groups (consecutive MMAs write
        // different accumulators when a stage holds several groups), commit
        // each group's buffer to the epilogue and the slot to the producer.
        const int mw = warp - kMmaWarp0;
        if (lane == 0) {
            // s32 accumulate, A s8, B s8, both K-major, N = npad, M = 128
            const uint32_t idesc = (2u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(N >> 3) << 17) | (8u << 24);
            const int ksteps = gs / 32;
            // stage i = mw, mw + kMmaWarps, ...: slot i % S, groups i*gst .. i*gst + gst - 1
            int slot = mw % S;
            uint32_t ph = (uint32_t)((mw / S) & 1);
            int gbase = mw * gst;  // first group of the stage (CTA-local)
            bool issued = false;
            for (int i = mw; i < nst; i += kMmaWarps) {
                if (!qwait(&bars->conv[slot], ph, err, DEV_TIMEOUT_CONV, abort_flag)) break;
                const int glast = gbase + gst - 1;
                if (!qwait(&bars->tempty[glast % kNBuf], (uint32_t)(((glast / kNBuf) & 1) ^ 1), err,
                           DEV_TIMEOUT_TEMPTY, abort_flag))
                    break;
                tc_fence_after();
                const uint32_t abase = smem_addr(tileA(slot, 0)), bbase = smem_addr(tileB(slot));
                for (int kk = 0; kk < ksteps; ++kk) {
                    for (int gl = 0; gl < gst; ++gl) {
                        const int kb = gl * gs + kk * 32;
                        const int bb = (gbase + gl) % kNBuf;
#pragma unroll
                        for (int m = 0; m < MULT; ++m)
                            mma_i8(tmem + (uint32_t)(bb * N * MULT + m * N), smem_desc_sw128(abase + m * Lay::kA + kb),
                                   smem_desc_sw128(bbase + kb), idesc, kk > 0 ? 1u : 0u);
                    }
                }
                issued = true;
                for (int gl = 0; gl < gst; ++gl) mma_commit(&bars->tfull[(gbase + gl) % kNBuf]);
                mma_commit(&bars->empty[slot]);
                slot += kMmaWarps;
                if (slot >= S) {
                    slot -= S;
                    ph ^= 1u;
                }
                gbase += kMmaWarps * gst;
            }
            if (issued) {
                // every MMA this thread issued has completed before TMEM is freed
                mma_commit(&bars->done[mw]);
                mbar_wait(&bars->done[mw], 0, err, DEV_TIMEOUT_MMA);
            }
        }
    } else if (warp < kEpiWarp0) {
        // ---------------- operand conversion ----------------
        const int row = threadIdx.x - kConvWarp0 * 32;  // 0..127: one weight row per thread
        int slot = 0;
        uint32_t ph = 0;
        for (int i = 0; i < nst; ++i) {
            // warp-uniform decision: every lane leaves the loop together
            if (!__all_sync(0xffffffffu, qwait(&bars->full[slot], ph, err, DEV_TIMEOUT_FULL, abort_flag))) break;
#pragma unroll
            for (int m = 0; m < MULT; ++m) {
                uint4* arow = reinterpret_cast<uint4*>(tileA(slot, m) + row * 128);
                if (KIND == 8) {
                    // biased u8 (q + 128) -> s8 q; a bytewise xor, so the swizzle does not
                    // matter.  Chunk order rotated by row: conflict-free shared accesses.
#pragma unroll
                    for (int c = 0; c < 8; ++c) {
                        const int cc = (c + row) & 7;
                        uint4 v = arow[cc];
                        v.x ^= 0x80808080u;
                        v.y ^= 0x80808080u;
                        v.z ^= 0x80808080u;
                        v.w ^= 0x80808080u;
                        arow[cc] = v;
                    }
                } else {
                    // packed nibbles (even element low) -> s8 bytes 16*q in element order,
                    // 16-byte chunk c of the row stored at chunk c ^ (row & 7) (128-byte swizzle)
                    const uint4* prow = reinterpret_cast<const uint4*>(tileP(slot, m) + row * 64);
#pragma unroll
                    for (int c2r = 0; c2r < 4; ++c2r) {
                        const int c2 = (c2r + (row >> 1)) & 3;  // rotated: conflict-free reads
                        const uint4 p = prow[c2];
                        const uint32_t w[4] = {p.x, p.y, p.z, p.w};
                        uint32_t o[8];
#pragma unroll
                        for (int u = 0; u < 4; ++u) {
                            const uint32_t lo = (w[u] << 4) & 0xF0F0F0F0u;  // elements 0,2,4,6 of the word
                            const uint32_t hi = w[u] & 0xF0F0F0F0u;         // elements 1,3,5,7
                            o[2 * u] = __byte_perm(lo, hi, 0x5140);
                            o[2 * u + 1] = __byte_perm(lo, hi, 0x7362);
                        }
                        const int c0 = 2 * c2, c1 = 2 * c2 + 1;
                        arow[c0 ^ (row & 7)] = make_uint4(o[0], o[1], o[2], o[3]);
                        arow[c1 ^ (row & 7)] = make_uint4(o[4], o[5], o[6], o[7]);
                    }
                }
            }
            asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
            __syncwarp();
            if (lane == 0) mbar_arrive(&bars->conv[slot]);
            if (++slot == S) {
                slot = 0;
                ph ^= 1u;
            }
        }
    } else {
        // ---------------- epilogue ----------------
        constexpr int NC = N / (kEpiWarps / 4);  // columns per thread
        const int q = warp & 3, h = (warp - kEpiWarp0) >> 2;
        const int rr = 32 * q + lane;  // row within the tile = TMEM lane
        const int c0 = h * NC;
        const uint32_t tl = tmem + ((uint32_t)(32 * q) << 16);
        float acc[MULT][NC];
        int gc = 0, buf = 0, xslot = 0;
        uint32_t bph = 0, xph = 0;
        int64_t s = s0;
        while (s < s1) {
            const int t = (int)(s / K);
            const int64_t send = min(s1, (int64_t)(t + 1) * K);  // this CTA's piece of tile t
            int seg = 0;
            while (seg + 1 < a.ep.nseg && t >= a.tile_start[seg + 1]) ++seg;
            const GemvSeg& sg = a.ep.seg[seg];
            const int rloc = (t - a.tile_start[seg]) * kTileRows + rr;  // row within the segment
            // weight scales of this row: 16-byte loads of four groups, one quad ahead
            const float4* wsq[MULT];
            wsq[0] = reinterpret_cast<const float4*>(sg.ws + (size_t)rloc * ng);
            if (MULT == 2) wsq[MULT - 1] = reinterpret_cast<const float4*>(sg.ws2 + (size_t)rloc * ng);
            int qi = (int)((s - (int64_t)t * K) * gst) >> 2;
            float4 wcur[MULT], wnext[MULT];
#pragma unroll
            for (int m = 0; m < MULT; ++m) {
                wcur[m] = __ldg(wsq[m] + qi);
                wnext[m] = 4 * qi + 4 < ng ? __ldg(wsq[m] + qi + 1) : make_float4(0.f, 0.f, 0.f, 0.f);
            }
#pragma unroll
            for (int m = 0; m < MULT; ++m)
#pragma unroll
                for (int j = 0; j < NC; ++j) acc[m][j] = 0.0f;
            for (int k = (int)(s - (int64_t)t * K); s < send; ++s, ++k) {
                // the stage's activation scales (bulk-copied by the producer)
                qwait(&bars->xfull[xslot], xph, err, DEV_TIMEOUT_FULL, abort_flag);
                const float* xst = xring + xslot * (Lay::kXsEntry / 4);
                for (int gl = 0; gl < gst; ++gl, ++gc) {
                    const int g = k * gst + gl;
                    if ((g >> 2) != qi) {
                        qi = g >> 2;
#pragma unroll
                        for (int m = 0; m < MULT; ++m) {
                            wcur[m] = wnext[m];
                            wnext[m] = 4 * qi + 4 < ng ? __ldg(wsq[m] + qi + 1) : make_float4(0.f, 0.f, 0.f, 0.f);
                        }
                    }
                    float wsv[MULT];
#pragma unroll
                    for (int m = 0; m < MULT; ++m) {
                        const int e = g & 3;
                        wsv[m] = e == 0 ? wcur[m].x : e == 1 ? wcur[m].y : e == 2 ? wcur[m].z : wcur[m].w;
                    }
                    const float2* xp = reinterpret_cast<const float2*>(xst + gl * N + c0);
                    qwait(&bars->tfull[buf], bph, err, DEV_TIMEOUT_TFULL, abort_flag);
                    __syncwarp();
                    tc_fence_after();
#pragma unroll
                    for (int m = 0; m < MULT; ++m) {
                        // one tensor at a time: its NC dots of this group, then the fp32 update
                        int d[NC];
                        tmem_ld<NC>(tl + (uint32_t)(buf * N * MULT + m * N + c0), d);
                        tmem_ld_wait();
                        const uint64_t w2 = f2_pack(wsv[m], wsv[m]);
#pragma unroll
                        for (int j = 0; j < NC; j += 2) {
                            // (float)D exactly: the bits of 1.5*2^23 + D, minus 1.5*2^23
                            const uint64_t df = f2_add(f2_pack(__int_as_float(d[j] + 0x4B400000),
                                                               __int_as_float(d[j + 1] + 0x4B400000)),
                                                       f2_pack(-12582912.0f, -12582912.0f));
                            const float2 xv = xp[j >> 1];
                            const uint64_t f = f2_mul(w2, f2_pack(xv.x, xv.y));
                            const uint64_t r = f2_fma(f, df, f2_pack(acc[m][j], acc[m][j + 1]));
                            acc[m][j] = f2_lo(r);
                            acc[m][j + 1] = f2_hi(r);
                        }
                    }
                    tc_fence_before();
                    __syncwarp();
                    if (lane == 0) mbar_arrive(&bars->tempty[buf]);
                    if (++buf == kNBuf) {
                        buf = 0;
                        bph ^= 1u;
                    }
                }
                __syncwarp();
                if (lane == 0) mbar_arrive(&bars->xempty[xslot]);
                if (++xslot == kXsStages) {
                    xslot = 0;
                    xph ^= 1u;
                }
            }
            // piece of tile t done: stages [max(s0, tK), send)
            const int64_t tk0 = (int64_t)t * K;
            const int first = sk_owner(tk0, W, G), lastc = sk_owner(tk0 + K - 1, W, G);
            const int P = lastc - first + 1;
            bool finish = true;
            if (P > 1) {
                const int pslot0 = s0 >= tk0 ? 0 : 1;
                float* pb = a.part + (((size_t)blockIdx.x * 2 + pslot0) * MULT) * N * kTileRows;
#pragma unroll
                for (int m = 0; m < MULT; ++m)
#pragma unroll
                    for (int j = 0; j < NC; ++j) pb[((size_t)m * N + c0 + j) * kTileRows + rr] = acc[m][j];
                __threadfence();
                named_bar_sync(1, kEpiWarps * 32);
                if (threadIdx.x == kEpiWarp0 * 32) {
                    const int old = atomicAdd(a.cnt + t, 1);
                    const int last = old == P - 1;
                    if (last) a.cnt[t] = 0;  // re-arm for the next launch
                    bars->last_flag = last;
                }
                named_bar_sync(1, kEpiWarps * 32);
                finish = bars->last_flag != 0;
                named_bar_sync(1, kEpiWarps * 32);  // last_flag is rewritten by the next piece
                if (finish) {
                    __threadfence();
                    for (int p = 0; p < P; ++p) {
                        const int cta = first + p;
                        const int pslot = sk_start(cta, W, G) >= tk0 ? 0 : 1;
                        const float* qb = a.part + (((size_t)cta * 2 + pslot) * MULT) * N * kTileRows;
#pragma unroll
                        for (int m = 0; m < MULT; ++m)
#pragma unroll
                            for (int j = 0; j < NC; ++j) {
                                const float v = __ldcg(qb + ((size_t)m * N + c0 + j) * kTileRows + rr);
                                acc[m][j] = p == 0 ? v : acc[m][j] + v;
                            }
                    }
                }
            }
            if (finish) {
#pragma unroll
                for (int j = 0; j < NC; ++j) {
                    const float v0 = acc[0][j], v1 = __shfl_xor_sync(0xffffffffu, v0, 1);
                    const float u0 = acc[MULT - 1][j], u1 = __shfl_xor_sync(0xffffffffu, u0, 1);
                    if ((lane & 1) == 0) finish_pair(a.ep, sg, c0 + j, rloc, v0, v1, u0, u1);
                }
            }
        }
    }

    tc_fence_before();
    __syncthreads();
    kt_end_cta(a.ep.kt);
    if (warp == kMmaWarp0) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kCols) : "memory");
    }
}

__global__ void scales_t_kernel(const float* __restrict__ xs, int rows, int ng, int ld, float mul,
                                float* __restrict__ xs_t) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;  // over ng * ld
    if (i >= ng * ld) return;
    const int g = i / ld, b = i - g * ld;
    xs_t[i] = b < rows ? xs[(size_t)b * ng + g] * mul : 0.0f;
}

// ---- host ----------------------------------------------------------------

PFN_cuTensorMapEncodeTiled_v12000 g_encode = nullptr;

bool get_encoder() {
    if (g_encode) return true;
    void* fn = nullptr;
    cudaDriverEntryPointQueryResult qr;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &qr) != cudaSuccess ||
        qr != cudaDriverEntryPointSuccess || !fn) {
        cudaGetLastError();
        return false;
    }
    g_encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
    return true;
}

// 2-D map over a row-major byte matrix [rows][pitch]
bool make_map(CUtensorMap* m, const void* base, uint64_t inner, uint64_t rows, uint64_t pitch, uint32_t box_inner,
              uint32_t box_rows, CUtensorMapSwizzle swz) {
    cuuint64_t dims[2] = {inner, rows};
    cuuint64_t strides[1] = {pitch};
    cuuint32_t box[2] = {box_inner, box_rows};
    cuuint32_t es[2] = {1, 1};
    CUresult r = g_encode(m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(base), dims, strides, box, es,
                          CU_TENSOR_MAP_INTERLEAVE_NONE, swz, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                          CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS;
}

int npad_for(int rows) { return rows <= 16 ? 16 : (rows <= 32 ? 32 : 64); }

template <int KIND, int N, int MULT>
cudaError_t launch_t(const QgemmArgs& q, cudaStream_t st, bool pdl, int grid) {
    using Lay = Layout<KIND, N, MULT>;
    const size_t smem = (size_t)q.stages * Lay::kStage + Lay::kXs + sizeof(Bars) + 1024;
    auto kern = qgemm_kernel<KIND, N, MULT>;
    static size_t set = 0;
    if (smem > set) {
        cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        if (e != cudaSuccess) return e;
        set = smem;
    }
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(kQgThreads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, kern, q);
}

template <int KIND, int N, int MULT>
int stages_for() {
    using Lay = Layout<KIND, N, MULT>;
    const int budget = 227 * 1024 - 1024 - (int)sizeof(Bars) - Lay::kXs;
    int s = budget / Lay::kStage;
    return s > 8 ? 8 : s;
}

template <int KIND>
cudaError_t launch_kind(const QgemmArgs& q, int npad, int mult, cudaStream_t st, bool pdl, int grid) {
    QgemmArgs c = q;
#define LQ_QG(NN, MM)                                    \
    if (npad == NN && mult == MM) {                      \
        c.stages = stages_for<KIND, NN, MM>();           \
        if (c.stages < 2) return cudaErrorInvalidValue;  \
        return launch_t<KIND, NN, MM>(c, st, pdl, grid); \
    }
    LQ_QG(16, 1) LQ_QG(32, 1) LQ_QG(64, 1) LQ_QG(16, 2) LQ_QG(32, 2) LQ_QG(64, 2)
#undef LQ_QG
    return cudaErrorInvalidValue;
}

}  // namespace

bool qgemm_ok(const GemvArgs& a, int kind, int rows) {
    if (kind != 8 && kind != 4) return false;
    if (rows < 1 || rows > 64) return false;
    if (!(a.gs == 32 || a.gs == 64 || a.gs == 128)) return false;
    if (a.cols % kStageK || a.in_mode != IN_QUANT || !a.xq) return false;
    if ((a.cols / a.gs) % 4) return false;  // weight scales are read four groups at a time
    if (a.nseg < 1 || a.nseg > kMaxSegs) return false;
    for (int i = 0; i < a.nseg; ++i) {
        const GemvSeg& g = a.seg[i];
        if (g.rows % kTileRows || !g.wq || !g.ws) return false;
        if ((reinterpret_cast<uintptr_t>(g.wq) | reinterpret_cast<uintptr_t>(g.ws)) & 15u) return false;
        if (a.paired && (!g.wq2 || !g.ws2 ||
                         ((reinterpret_cast<uintptr_t>(g.wq2) | reinterpret_cast<uintptr_t>(g.ws2)) & 15u)))
            return false;
    }
    if (reinterpret_cast<uintptr_t>(a.xq) & 15u) return false;
    return get_encoder();
}

int qgemm_npad(int rows) { return npad_for(rows); }

size_t qgemm_part_floats(int num_sms) { return (size_t)num_sms * 2 * 2 * 64 * kTileRows; }

int qgemm_max_tiles(const GemvArgs& a) {
    int t = 0;
    for (int i = 0; i < a.nseg; ++i) t += a.seg[i].rows / kTileRows;
    return t;
}

cudaError_t qgemm_scales_launch(const float* xs, int rows, int ng, int ld, float mul, float* xs_t,
                                cudaStream_t st) {
    const int n = ng * ld;
    scales_t_kernel<<<(n + 255) / 256, 256, 0, st>>>(xs, rows, ng, ld, mul, xs_t);
    return cudaGetLastError();
}

cudaError_t qgemm_launch(const GemvArgs& a, int kind, const float* xs_t, int xs_ld, float* part, int* cnt,
                         cudaStream_t st, bool pdl, int num_sms) {
    const int rows = a.nvalid > 0 ? a.nvalid : a.nb;
    if (!qgemm_ok(a, kind, rows) || !xs_t || !part || !cnt) return cudaErrorInvalidValue;
    const int npad = npad_for(rows);
    // the scales of a stage's groups are one contiguous run: row pitch = npad
    if (xs_ld != npad || (reinterpret_cast<uintptr_t>(xs_t) & 15u)) return cudaErrorInvalidValue;
    QgemmArgs q;
    memset(&q, 0, sizeof(q));
    q.ep = a;
    q.ep.nb = npad;
    q.ep.nvalid = rows;
    q.xs_t = xs_t;
    q.xs_ld = xs_ld;
    q.part = part;
    q.cnt = cnt;
    const int mult = a.paired ? 2 : 1;
    const uint64_t kbytes = kind == 8 ? (uint64_t)a.cols : (uint64_t)a.cols / 2;
    int tiles = 0;
    for (int i = 0; i < a.nseg; ++i) {
        const GemvSeg& g = a.seg[i];
        q.tile_start[i] = tiles;
        tiles += g.rows / kTileRows;
        const CUtensorMapSwizzle swz = kind == 8 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_NONE;
        const uint32_t box = kind == 8 ? kStageK : kStageK / 2;
        if (!make_map(&q.wmap[i][0], g.wq, kbytes, (uint64_t)g.rows, kbytes, box, kTileRows, swz))
            return cudaErrorInvalidValue;
        if (mult == 2 && !make_map(&q.wmap[i][1], g.wq2, kbytes, (uint64_t)g.rows, kbytes, box, kTileRows, swz))
            return cudaErrorInvalidValue;
    }
    q.tile_start[a.nseg] = tiles;
    q.tiles = tiles;
    q.kst = a.cols / kStageK;
    // rows beyond the real ones read as zeros (out-of-range box rows)
    if (!make_map(&q.xmap, a.xq, (uint64_t)a.cols, (uint64_t)rows, (uint64_t)a.cols, kStageK, (uint32_t)npad,
                  CU_TENSOR_MAP_SWIZZLE_128B))
        return cudaErrorInvalidValue;
    const int64_t W = (int64_t)tiles * q.kst;
    const int grid = (int)(W < num_sms ? W : num_sms);
    return kind == 8 ? launch_kind<8>(q, npad, mult, st, pdl, grid) : launch_kind<4>(q, npad, mult, st, pdl, grid);
}

bool kv_tensor_map(CUtensorMap* m, const float* kcache, int head_size, uint64_t rows) {
    if (!get_encoder()) return false;
    const uint64_t row = (uint64_t)head_size * sizeof(float);
    return make_map(m, kcache, row, rows, row, 128, kChunk, CU_TENSOR_MAP_SWIZZLE_128B);
}

}  // namespace lq
