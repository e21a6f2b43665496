// matmul_f32_noalloc: the fp32-input GEMV (quantize x, then the group-
// quantized product) for callers that must not allocate device memory.
//
// Some callers cannot call cudaMalloc at the moment they need this product:
// a host framework that owns every device allocation and forbids plugins
// from allocating while a request is being served, or a latency-bound loop
// where a first-use allocation (which may synchronize the device, and may
// fail when memory is exhausted) is not acceptable.  This entry point uses
// no allocation of any kind: its scratch (the int8 activation, its group
// scales and group sums, and an error word) is a fixed array in device
// memory, defined below, that exists on every GPU that loads the library
// until the process exits.
//
// Limits and sharing:
//  * n may be at most kNoAllocMaxN (32768) and the group size at least 32;
//    larger requests are rejected with LQ_EINVAL.
//  * Every call on a device uses the same array and leaves its contents in
//    place for the next call.  Two calls whose kernels overlap on the GPU
//    (different streams, or different host threads) race on the array.
//  * The first call on each device looks up the array's device address
//    (cudaGetSymbolAddress) with that device current; make that first call
//    before any stream capture.
//  * A device-side wait that gives up inside one of these calls sets the
//    array's error word; lq_sync reports it (LQ_ETIMEOUT) and clears it.
#include <cstdint>
#include <cstdio>

#include "lq_ctx.h"
#include "lq_host.h"
#include "lq_kernels.h"

namespace {

constexpr int kNoAllocMaxN = 32768;
constexpr int kNoAllocMinGs = 32;
constexpr size_t kXqBytes = kNoAllocMaxN;                                  // int8 activation
constexpr size_t kGroupBytes = (size_t)kNoAllocMaxN / kNoAllocMinGs * 4;  // fp32 scales / int32 sums
constexpr size_t kErrOff = kXqBytes + 2 * kGroupBytes;
constexpr size_t kScratchBytes = kErrOff + 256;  // 40 KB in all

void* g_noalloc_addr[64] = {nullptr};  // device address of the array, per device

bool on_device(const void* p) {
    cudaPointerAttributes at;
    if (cudaPointerGetAttributes(&at, p) != cudaSuccess) {
        cudaGetLastError();
        return false;
    }
    return at.type == cudaMemoryTypeDevice || at.type == cudaMemoryTypeManaged;
}

}  // namespace

// The fixed scratch: one copy per device, for the life of the process.
static __device__ __align__(256) unsigned char g_noalloc_scratch[kScratchBytes];

extern "C" int matmul_f32_noalloc(float* xout, const float* x, const QuantizedTensor* w, int n, int d) {
    if (!xout || !x || !w || !w->q || !w->s) return lq_fail(LQ_EINVAL, "matmul_f32_noalloc: null argument");
    if (w->kind != LQ_KIND_INT8 && w->kind != LQ_KIND_INT4)
        return lq_fail(LQ_EINVAL, "matmul_f32_noalloc: weight kind must be LQ_KIND_INT8 or LQ_KIND_INT4");
    const int gs = w->group_size;
    if (!(gs == 32 || gs == 64 || gs == 128 || gs == 256))
        return lq_fail(LQ_EUNSUPPORTED, "matmul_f32_noalloc: group size %d not supported", gs);
    if (n <= 0 || d <= 0 || w->cols != n || w->rows != d || n % gs)
        return lq_fail(LQ_EINVAL, "matmul_f32_noalloc: shape mismatch (w is %lld x %lld, n=%d d=%d)",
                       (long long)w->rows, (long long)w->cols, n, d);
    if (n > kNoAllocMaxN)
        return lq_fail(LQ_EINVAL, "matmul_f32_noalloc: n=%d exceeds the fixed scratch limit of %d", n, kNoAllocMaxN);
    if ((reinterpret_cast<uintptr_t>(w->q) | reinterpret_cast<uintptr_t>(w->s) | reinterpret_cast<uintptr_t>(x)) & 15u)
        return lq_fail(LQ_EINVAL, "matmul_f32_noalloc: x, w->q and w->s must be 16-byte aligned");
    if (!on_device(x) || !on_device(xout))
        return lq_fail(LQ_EINVAL, "matmul_f32_noalloc: x and xout must be device memory");
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess || dev < 0 || dev >= 64) return lq_fail(LQ_ECUDA, "matmul_f32_noalloc: no CUDA device");
    if (!g_noalloc_addr[dev]) {
        // set-up, once per device, with that device current
        void* p = nullptr;
        e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
        if (e != cudaSuccess || !p) return lq::cuda_fail(e, "matmul_f32_noalloc: scratch address lookup");
        g_noalloc_addr[dev] = p;
    }
    int num_sms = 148;
    cudaDeviceGetAttribute(&num_sms, cudaDevAttrMultiProcessorCount, dev);
    unsigned char* base = static_cast<unsigned char*>(g_noalloc_addr[dev]);
    int8_t* xq = reinterpret_cast<int8_t*>(base);
    float* xs = reinterpret_cast<float*>(base + kXqBytes);
    int* xsum = reinterpret_cast<int*>(base + kXqBytes + kGroupBytes);
    int* err = reinterpret_cast<int*>(base + kErrOff);
    cudaStream_t st = lq::stream();
    // The activation, scales and sums are fully rewritten by the quantizer
    // before the GEMV reads them.  The error word starts at zero (static
    // device memory is zero-initialised) and goes back to zero whenever
    // lq_sync reports it, so a device-side error of any call stays recorded
    // until the next lq_sync.
    return lq::matmul_f32_device(xout, x, w, n, d, xq, xs, xsum, err, st, lq::launch_flags() & LQ_LAUNCH_PDL, num_sms,
                                 lq::trace_buffer());
}

namespace lq {

// Report (and clear) the error word of the fixed scratch on the current
// device, if matmul_f32_noalloc has been used there.  Called by lq_sync.
int noalloc_check_error(cudaStream_t st) {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64 || !g_noalloc_addr[dev]) return LQ_OK;
    int* err = reinterpret_cast<int*>(static_cast<unsigned char*>(g_noalloc_addr[dev]) + kErrOff);
    return check_device_error(err, st);
}

}  // namespace lq
