// Device helpers for sm_100a: mbarriers, 1-D bulk (TMA) copies, programmatic
// dependent launch, bounded waits.  Inline PTX from the public PTX ISA.
#pragma once
#include <cstdint>
#include <cuda.h>
#include <cuda_runtime.h>

namespace lq {

// Device-side error word codes (written with atomicCAS, first error wins).
enum : int {
    DEV_OK = 0,
    DEV_TIMEOUT_FULL = 0x101,   // consumer waited too long for a stage to land
    DEV_TIMEOUT_EMPTY = 0x102,  // producer waited too long for a stage to drain
    DEV_TIMEOUT_DRAIN = 0x103,  // producer could not confirm its copies after an error
    DEV_TIMEOUT_PEER = 0x104,   // a tensor-parallel peer did not publish its partial in time
    DEV_BAD_ARG = 0x201,        // a launch argument failed a device-side check
};

// Every wait gives up after this long; a healthy wait here lasts microseconds.
constexpr uint64_t kWaitLimitNs = 2000000000ull;

__device__ __forceinline__ uint32_t smem_addr(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ uint64_t globaltimer() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(bar)), "r"(count));
}

__device__ __forceinline__ void fence_mbar_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_addr(bar)),
                 "r"(bytes)
                 : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_addr(bar)) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n"
        " selp.u32 %0, 1, 0, p;\n}\n"
        : "=r"(ok)
        : "r"(smem_addr(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}

// Bounded wait on an mbarrier phase.  Returns false (and records `code` in
// *err) when the wait limit passes.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, int* err, int code) {
    if (mbar_try_wait(bar, parity)) return true;
    const uint64_t t0 = globaltimer();
    for (uint32_t i = 1;; ++i) {
        if (mbar_try_wait(bar, parity)) return true;
        if ((i & 63u) == 0 && globaltimer() - t0 > kWaitLimitNs) {
            if (err) atomicCAS(err, 0, code);
            return false;
        }
    }
}

__device__ __forceinline__ uint64_t l2_evict_first_policy() {
    uint64_t p;
    asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
    return p;
}

// 1-D bulk copy global -> shared (TMA unit).  dst, src 16-byte aligned and
// bytes a multiple of 16.  Completion is signalled on `bar` as tx bytes.
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar,
                                         uint64_t policy) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint"
        " [%0], [%1], %2, [%3], %4;" ::"r"(smem_addr(dst)),
        "l"(src), "r"(bytes), "r"(smem_addr(bar)), "l"(policy)
        : "memory");
}

// 2-D tiled tensor copy global -> shared (TMA): the box at (x, y) of the
// tensor map, completion signalled on `bar` as tx bytes.  x * element size
// must be a multiple of 16 bytes.
__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, int x, int y, uint64_t* bar,
                                            uint64_t policy) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes.L2::cache_hint"
        " [%0], [%1, {%2, %3}], [%4], %5;" ::"r"(smem_addr(dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_addr(bar)), "l"(policy)
        : "memory");
}

// Programmatic dependent launch (PTX griddepcontrol).
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() {
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

__device__ __forceinline__ void named_bar_sync(int id, int nthreads) {
    asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(nthreads) : "memory");
}

// 4-way byte dot product: unsigned bytes of a times signed bytes of b, plus c.
__device__ __forceinline__ int dp4a_us(uint32_t a, uint32_t b, int c) {
    int d;
    asm("dp4a.u32.s32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
    return d;
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

// the xor butterfly levels o, o/2, ..., 1 of a warp sum
__device__ __forceinline__ float warp_sum_below(float v, int o) {
#pragma unroll
    for (; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

// System-scope accesses for flags and data shared with peer GPUs.
__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
    uint32_t v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

__device__ __forceinline__ void st_release_sys(uint32_t* p, uint32_t v) {
    asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

// 64-bit words of the low-latency all-reduce: relaxed system-scope accesses
// (each aligned 64-bit element is single-copy atomic)
__device__ __forceinline__ void st_relaxed_sys_u64(uint64_t* p, uint64_t v) {
    asm volatile("st.relaxed.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ void st_relaxed_sys_v2(uint64_t* p, uint64_t a, uint64_t b) {
    asm volatile("st.relaxed.sys.global.v2.u64 [%0], {%1, %2};" ::"l"(p), "l"(a), "l"(b) : "memory");
}
__device__ __forceinline__ void ld_relaxed_sys_v2(const uint64_t* p, uint64_t& a, uint64_t& b) {
    asm volatile("ld.relaxed.sys.global.v2.u64 {%0, %1}, [%2];" : "=l"(a), "=l"(b) : "l"(p) : "memory");
}

__device__ __forceinline__ void fence_acq_rel_sys() { asm volatile("fence.acq_rel.sys;" ::: "memory"); }

__device__ __forceinline__ float4 ld_volatile_f4(const float* p) {
    float4 v;
    asm volatile("ld.volatile.global.v4.f32 {%0, %1, %2, %3}, [%4];"
                 : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
                 : "l"(p)
                 : "memory");
    return v;
}

__device__ __forceinline__ void set_err(int* err, int code) {
    if (err) atomicCAS(err, 0, code);
}

// Step trace (profiling; kt == nullptr: off).  kt holds this kernel's
// stamps (globaltimer ns) in 3 x kKtSlots words, each reduced over the CTAs
// that share a slot (blockIdx.x % kKtSlots) with atomicMin from an all-ones
// reset, so that no single word takes every CTA's atomic:
// [0, S) start of a CTA, [S, 2S) a CTA past its dependency wait, [2S, 3S) the
// bitwise complement of a CTA's end.  One thread per CTA stamps each.
constexpr int kKtSlots = 32;
__device__ __forceinline__ void kt_stamp(uint64_t* kt, int which, uint64_t v) {
    atomicMin(reinterpret_cast<unsigned long long*>(kt) + which * kKtSlots + (blockIdx.x % kKtSlots),
              (unsigned long long)v);
}
__device__ __forceinline__ void kt_start(uint64_t* kt) {
    if (kt && threadIdx.x == 0) kt_stamp(kt, 0, globaltimer());
}
__device__ __forceinline__ void kt_waited(uint64_t* kt) {
    if (kt && threadIdx.x == 0) kt_stamp(kt, 1, globaltimer());
}
// at a point every thread of the CTA reaches (it synchronizes the CTA)
__device__ __forceinline__ void kt_end_cta(uint64_t* kt) {
    if (kt) {
        __syncthreads();
        if (threadIdx.x == 0) kt_stamp(kt, 2, ~globaltimer());
    }
}

}  // namespace lq
