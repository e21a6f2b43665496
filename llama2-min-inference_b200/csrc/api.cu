// C-ABI: error reporting, stream, and the operator entry points
// (quantize / matmul / matmul_f32).
#include <cstdarg>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <mutex>

#include "lq_ctx.h"
#include "lq_host.h"
#include "lq_kernels.h"
#include "lq_ops.h"

namespace {

thread_local char g_err[1024] = "";
cudaStream_t g_stream = nullptr;
int g_launch_flags = 0;
uint64_t* g_trace = nullptr;  // device buffer for per-CTA GEMV phase timestamps (lq_set_trace)
std::mutex g_ctx_mu;
lq::DevCtx* g_ctx[64] = {nullptr};

// page-locked (registered or cudaHostAlloc'd) host memory
bool is_pinned_host_ptr(const void* p) {
    cudaPointerAttributes at;
    if (cudaPointerGetAttributes(&at, p) != cudaSuccess) {
        cudaGetLastError();
        return false;
    }
    return at.type == cudaMemoryTypeHost;
}

bool is_device_ptr(const void* p) {
    cudaPointerAttributes at;
    if (cudaPointerGetAttributes(&at, p) != cudaSuccess) {
        cudaGetLastError();
        return false;
    }
    return at.type == cudaMemoryTypeDevice || at.type == cudaMemoryTypeManaged;
}

}  // namespace

extern "C" int lq_fail(int code, const char* fmt, ...) {
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(g_err, sizeof(g_err), fmt, ap);
    va_end(ap);
    return code;
}

namespace lq {

int cuda_fail(cudaError_t e, const char* what) {
    return lq_fail(e == cudaErrorMemoryAllocation ? LQ_ENOMEM : LQ_ECUDA, "%s: %s", what, cudaGetErrorString(e));
}

DevCtx* ctx() {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return nullptr;
    std::lock_guard<std::mutex> lk(g_ctx_mu);
    if (!g_ctx[dev]) {
        DevCtx* c = new DevCtx();
        c->dev = dev;
        if (cudaDeviceGetAttribute(&c->num_sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess ||
            cudaMalloc(&c->err, sizeof(int)) != cudaSuccess || cudaMemset(c->err, 0, sizeof(int)) != cudaSuccess) {
            cudaGetLastError();
            delete c;
            return nullptr;
        }
        g_ctx[dev] = c;
    }
    return g_ctx[dev];
}

int ensure_scratch(DevCtx* c, size_t bytes) {
    if (c->scratch_bytes >= bytes) return LQ_OK;
    cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
    if (cudaStreamIsCapturing(g_stream, &cs) == cudaSuccess && cs != cudaStreamCaptureStatusNone)
        return lq_fail(LQ_EINVAL,
                       "scratch of %zu bytes needed inside a graph capture: make one call of this size before capturing",
                       bytes);
    // the cached call graphs point into the old scratch
    for (auto& g : c->graphs)
        if (g.exec) cudaGraphExecDestroy(g.exec);
    c->graphs.clear();
    if (c->scratch) cudaFree(c->scratch);
    c->scratch = nullptr;
    c->scratch_bytes = 0;
    cudaError_t e = cudaMalloc(&c->scratch, bytes);
    if (e != cudaSuccess) return cuda_fail(e, "scratch allocation");
    c->scratch_bytes = bytes;
    return LQ_OK;
}

int check_device_error(int* err_dev, cudaStream_t st) {
    int h = 0;
    cudaError_t e = cudaMemcpyAsync(&h, err_dev, sizeof(int), cudaMemcpyDeviceToHost, st);
    if (e == cudaSuccess) e = cudaStreamSynchronize(st);
    if (e != cudaSuccess) return cuda_fail(e, "device error check");
    if (h != 0) {
        cudaMemsetAsync(err_dev, 0, sizeof(int), st);
        cudaStreamSynchronize(st);
        return lq_fail(LQ_ETIMEOUT, "device-side wait gave up (code 0x%x)", h);
    }
    return LQ_OK;
}

cudaStream_t stream() { return g_stream; }
int launch_flags() { return g_launch_flags; }
uint64_t* trace_buffer() { return g_trace; }

// quantize x into (xq, xs, xsum), then the GEMV from the pre-quantized
// activation; the GEMV may start streaming weights while the quantizer runs
int matmul_f32_device(float* yd, const float* xd, const QuantizedTensor* w, int n, int d, int8_t* xq, float* xs,
                      int* xsum, int* err, cudaStream_t st, bool pdl_first, int num_sms, uint64_t* trace) {
    ActQuantArgs q = {};
    q.mode = IN_F32;
    q.n = n;
    q.gs = w->group_size;
    q.nb = 1;
    q.x = xd;
    q.xq = xq;
    q.xs = xs;
    q.xsum = xsum;
    cudaError_t e = act_quant_launch(q, st, pdl_first);
    if (e != cudaSuccess) return cuda_fail(e, "matmul_f32: quantize launch");
    GemvArgs a = {};
    a.seg[0] = {static_cast<const uint8_t*>(w->q), w->s, yd, d, EPI_STORE};
    a.nseg = 1;
    a.cols = n;
    a.gs = w->group_size;
    a.nb = 1;
    a.in_mode = IN_QUANT;
    a.xq = xq;
    a.xs = xs;
    a.xsum_in = xsum;
    a.y_stride = d;
    a.err = err;
    a.trace = trace;
    // the quantizer does not write the weights, so the GEMV may prefetch them
    e = gemv_launch(a, w->kind, st, true, num_sms);
    if (e != cudaSuccess) return cuda_fail(e, "matmul_f32 launch");
    return LQ_OK;
}

}  // namespace lq

using namespace lq;

extern "C" {

const char* lq_last_error(void) { return g_err; }

int lq_select_device(int device) {
    int n = 0;
    cudaError_t e = cudaGetDeviceCount(&n);
    if (e != cudaSuccess || n == 0) return lq_fail(LQ_ECUDA, "no CUDA device context (no device, or first use inside a graph capture)");
    if (device >= n) return lq_fail(LQ_EINVAL, "device %d out of range (%d devices)", device, n);
    if (device < 0) {
        size_t best = 0;
        for (int i = 0; i < n; ++i) {
            size_t f = 0, t = 0;
            if (cudaSetDevice(i) == cudaSuccess && cudaMemGetInfo(&f, &t) == cudaSuccess && f > best) {
                best = f;
                device = i;
            }
            cudaGetLastError();
        }
        if (device < 0) return lq_fail(LQ_ECUDA, "no usable CUDA device");
    }
    e = cudaSetDevice(device);
    if (e != cudaSuccess) return cuda_fail(e, "cudaSetDevice");
    size_t f = 0, t = 0;
    cudaMemGetInfo(&f, &t);
    fprintf(stderr, "using GPU %d (%.1f GB free / %.1f GB)\n", device, f / 1073741824.0, t / 1073741824.0);
    return LQ_OK;
}

int lq_set_stream(void* s) {
    g_stream = static_cast<cudaStream_t>(s);
    // create the device context now: its allocation is not allowed while
    // the stream is being captured into a graph
    if (!ctx()) return lq_fail(LQ_ECUDA, "CUDA device context could not be created");
    return LQ_OK;
}

void* lq_get_stream(void) { return g_stream; }

int lq_sync(void) {
    DevCtx* c = ctx();
    if (!c) return lq_fail(LQ_ECUDA, "no CUDA device context (no device, or first use inside a graph capture)");
    const int a = check_device_error(c->err, g_stream);
    const int b = noalloc_check_error(g_stream);  // always read (and clear) both words
    return a ? a : b;
}

int lq_set_launch_flags(int flags) {
    if (flags & ~LQ_LAUNCH_PDL) return lq_fail(LQ_EINVAL, "unknown launch flags 0x%x", flags);
    g_launch_flags = flags;
    return LQ_OK;
}

int lq_set_trace(void* device_buffer) {
    g_trace = static_cast<uint64_t*>(device_buffer);
    return LQ_OK;
}

int lq_graph_begin(void) {
    if (!g_stream) return lq_fail(LQ_EINVAL, "lq_graph_begin: set a non-default stream first");
    if (!ctx()) return lq_fail(LQ_ECUDA, "CUDA device context could not be created");
    cudaError_t e = cudaStreamBeginCapture(g_stream, cudaStreamCaptureModeThreadLocal);
    return e == cudaSuccess ? LQ_OK : cuda_fail(e, "begin capture");
}

int lq_graph_end(void** exec) {
    if (!exec) return lq_fail(LQ_EINVAL, "lq_graph_end: null argument");
    cudaGraph_t g = nullptr;
    cudaError_t e = cudaStreamEndCapture(g_stream, &g);
    if (e != cudaSuccess) return cuda_fail(e, "end capture");
    cudaGraphExec_t x = nullptr;
    e = cudaGraphInstantiate(&x, g, 0);
    cudaGraphDestroy(g);
    if (e != cudaSuccess) return cuda_fail(e, "graph instantiate");
    *exec = x;
    return LQ_OK;
}

int lq_graph_launch(void* exec) {
    cudaError_t e = cudaGraphLaunch(static_cast<cudaGraphExec_t>(exec), g_stream);
    return e == cudaSuccess ? LQ_OK : cuda_fail(e, "graph launch");
}

void lq_graph_destroy(void* exec) {
    if (exec) cudaGraphExecDestroy(static_cast<cudaGraphExec_t>(exec));
}

int lq_synth_tensor(QuantizedTensor* w, uint64_t seed, int tensor_id, float std) {
    if (!w || !w->q || !w->s || w->rows <= 0 || w->cols <= 0)
        return lq_fail(LQ_EINVAL, "lq_synth_tensor: tensor not allocated");
    if (w->kind != LQ_KIND_INT8 && w->kind != LQ_KIND_INT4) return lq_fail(LQ_EINVAL, "lq_synth_tensor: kind");
    const int gs = w->group_size;
    if (!(gs == 32 || gs == 64 || gs == 128 || gs == 256) || w->cols % gs)
        return lq_fail(LQ_EINVAL, "lq_synth_tensor: group size");
    cudaError_t e = synth_quant_launch(static_cast<uint8_t*>(w->q), w->s, w->rows, w->cols, gs, w->kind, seed,
                                       tensor_id, std, 0, g_stream);
    return e == cudaSuccess ? LQ_OK : cuda_fail(e, "lq_synth_tensor");
}

int quantize(QuantizedTensor* out, const float* x, int n) {
    if (!out || !x || n <= 0) return lq_fail(LQ_EINVAL, "quantize: null argument or n <= 0");
    const int gs = out->group_size;
    if (gs <= 0 || gs % 32 || gs > 256 || n % gs)
        return lq_fail(LQ_EINVAL, "quantize: n=%d must be a multiple of group_size=%d (multiple of 32, <= 256)", n, gs);
    if (out->rows <= 0) out->rows = 1;
    if (!out->q || !out->s) return lq_fail(LQ_EINVAL, "quantize: out->q / out->s not allocated");
    DevCtx* c = ctx();
    if (!c) return lq_fail(LQ_ECUDA, "no CUDA device context (no device, or first use inside a graph capture)");
    const float* xd = x;
    const size_t bytes = (size_t)out->rows * n * sizeof(float);
    if (!is_device_ptr(x)) {
        int rc = ensure_scratch(c, bytes);
        if (rc) return rc;
        cudaError_t e = cudaMemcpyAsync(c->scratch, x, bytes, cudaMemcpyHostToDevice, g_stream);
        if (e != cudaSuccess) return cuda_fail(e, "quantize: copy of x");
        xd = static_cast<const float*>(c->scratch);
    }
    cudaError_t e = quantize_act_launch(xd, out->rows, n, gs, static_cast<int8_t*>(out->q), out->s, g_stream);
    if (e != cudaSuccess) return cuda_fail(e, "quantize launch");
    if (xd != x) {
        e = cudaStreamSynchronize(g_stream);  // the scratch copy must finish before reuse
        if (e != cudaSuccess) return cuda_fail(e, "quantize");
    }
    out->cols = n;
    out->kind = LQ_KIND_ACT8;
    return LQ_OK;
}

constexpr int kQgMaxTiles = 4096;

static int mma_min_rows() {
    static int v = -1;
    if (v < 0) {
        const char* e = getenv("LQ_MMA_MIN_ROWS");
        v = e ? atoi(e) : 16;
        if (v < 1) v = 1 << 30;  // 0 or negative: never
    }
    return v;
}

// workspace of the tensor-core GEMM (allocated outside graph capture)
static int ensure_qgemm(DevCtx* c, int ng) {
    cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
    const bool capturing = cudaStreamIsCapturing(g_stream, &cs) == cudaSuccess && cs != cudaStreamCaptureStatusNone;
    const size_t xst = (size_t)ng * 64;
    if (c->qg_part && c->qg_xst_floats >= xst) return LQ_OK;
    if (capturing)
        return lq_fail(LQ_EINVAL, "matmul: tensor-core workspace needed inside a graph capture: make one call first");
    cudaError_t e = cudaSuccess;
    if (!c->qg_part) {
        e = cudaMalloc(&c->qg_part, qgemm_part_floats(c->num_sms) * sizeof(float));
        if (e == cudaSuccess) e = cudaMalloc(&c->qg_cnt, kQgMaxTiles * sizeof(int));
        if (e == cudaSuccess) e = cudaMemset(c->qg_cnt, 0, kQgMaxTiles * sizeof(int));
    }
    if (e == cudaSuccess && c->qg_xst_floats < xst) {
        if (c->qg_xst) cudaFree(c->qg_xst);
        c->qg_xst = nullptr;
        c->qg_xst_floats = 0;
        e = cudaMalloc(&c->qg_xst, xst * sizeof(float));
        if (e == cudaSuccess) c->qg_xst_floats = xst;
    }
    return e == cudaSuccess ? LQ_OK : cuda_fail(e, "tensor-core GEMM workspace");
}

static int check_weight(const QuantizedTensor* w, int n, int d, const char* fn) {
    if (!w || !w->q || !w->s) return lq_fail(LQ_EINVAL, "%s: weight tensor not set", fn);
    if (w->kind != LQ_KIND_INT8 && w->kind != LQ_KIND_INT4)
        return lq_fail(LQ_EINVAL, "%s: weight kind must be LQ_KIND_INT8 or LQ_KIND_INT4", fn);
    const int gs = w->group_size;
    if (!(gs == 32 || gs == 64 || gs == 128 || gs == 256))
        return lq_fail(LQ_EUNSUPPORTED, "%s: group size %d not supported (32, 64, 128, 256)", fn, gs);
    if (n <= 0 || d <= 0 || w->cols != n || w->rows != d || n % gs)
        return lq_fail(LQ_EINVAL, "%s: shape mismatch (w is %lld x %lld, n=%d d=%d, gs=%d)", fn,
                       (long long)w->rows, (long long)w->cols, n, d, gs);
    if ((reinterpret_cast<uintptr_t>(w->q) | reinterpret_cast<uintptr_t>(w->s)) & 15u)
        return lq_fail(LQ_EINVAL, "%s: w->q and w->s must be 16-byte aligned", fn);
    return LQ_OK;
}

int matmul(float* xout, const QuantizedTensor* x, const QuantizedTensor* w, int n, int d) {
    int rc = check_weight(w, n, d, "matmul");
    if (rc) return rc;
    if (!xout || !x || !x->q || !x->s) return lq_fail(LQ_EINVAL, "matmul: null argument");
    if (x->kind != LQ_KIND_ACT8 || x->cols != n || x->group_size != w->group_size || x->rows <= 0)
        return lq_fail(LQ_EINVAL, "matmul: x must be an ACT8 tensor [B, n] with the weight's group size");
    if (reinterpret_cast<uintptr_t>(x->q) & 7u) return lq_fail(LQ_EINVAL, "matmul: x->q must be 8-byte aligned");
    DevCtx* c = ctx();
    if (!c) return lq_fail(LQ_ECUDA, "no CUDA device context (no device, or first use inside a graph capture)");
    const int ng = n / w->group_size;
    int64_t done = 0;
    if (x->rows >= mma_min_rows()) {
        // tensor cores: up to 64 activation rows per launch
        GemvArgs a = {};
        a.seg[0] = {static_cast<const uint8_t*>(w->q), w->s, xout, d, EPI_STORE};
        a.nseg = 1;
        a.cols = n;
        a.gs = w->group_size;
        a.in_mode = IN_QUANT;
        a.xq = static_cast<const int8_t*>(x->q);
        a.y_stride = d;
        a.err = c->err;
        a.nb = a.nvalid = 16;
        if (qgemm_ok(a, w->kind, 16) && d / 128 <= kQgMaxTiles) {
            rc = ensure_qgemm(c, ng);
            if (rc) return rc;
            const float mul = w->kind == LQ_KIND_INT4 ? 0.0625f : 1.0f;
            while (done < x->rows) {
                const int rows = (int)(x->rows - done < 64 ? x->rows - done : 64);
                const int npad = qgemm_npad(rows);
                cudaError_t e = qgemm_scales_launch(x->s + done * ng, rows, ng, npad, mul, c->qg_xst, g_stream);
                a.seg[0].y = xout + done * d;
                a.xq = static_cast<const int8_t*>(x->q) + done * n;
                a.nb = a.nvalid = rows;
                if (e == cudaSuccess)
                    e = qgemm_launch(a, w->kind, c->qg_xst, npad, c->qg_part, c->qg_cnt, g_stream,
                                     g_launch_flags & LQ_LAUNCH_PDL, c->num_sms);
                if (e != cudaSuccess) return cuda_fail(e, "matmul (tensor cores) launch");
                done += rows;
            }
            return LQ_OK;
        }
    }
    while (done < x->rows) {
        const int64_t left = x->rows - done;
        const int nb = left >= 8 ? 8 : left >= 4 ? 4 : left >= 2 ? 2 : 1;
        GemvArgs a = {};
        a.seg[0] = {static_cast<const uint8_t*>(w->q), w->s, xout + done * d, d, EPI_STORE};
        a.nseg = 1;
        a.cols = n;
        a.gs = w->group_size;
        a.nb = nb;
        a.in_mode = IN_QUANT;
        a.xq = static_cast<const int8_t*>(x->q) + done * n;
        a.xs = x->s + done * ng;
        a.y_stride = d;
        a.err = c->err;
        a.trace = g_trace;
        cudaError_t e = gemv_launch(a, w->kind, g_stream, g_launch_flags & LQ_LAUNCH_PDL, c->num_sms);
        if (e != cudaSuccess) return cuda_fail(e, "matmul launch");
        done += nb;
    }
    return LQ_OK;
}

int matmul_f32(float* xout, const float* x, const QuantizedTensor* w, int n, int d) {
    int rc = check_weight(w, n, d, "matmul_f32");
    if (rc) return rc;
    if (!xout || !x) return lq_fail(LQ_EINVAL, "matmul_f32: null argument");
    DevCtx* c = ctx();
    if (!c) return lq_fail(LQ_ECUDA, "no CUDA device context (no device, or first use inside a graph capture)");
    const bool xdev = is_device_ptr(x), ydev = is_device_ptr(xout);
    if ((reinterpret_cast<uintptr_t>(x) & 15u) && xdev)
        return lq_fail(LQ_EINVAL, "matmul_f32: device x must be 16-byte aligned");
    const int ng = n / w->group_size;
    auto up = [](size_t v) { return (v + 255) / 256 * 256; };
    // scratch: [fp32 x (host input only)] [fp32 y (host output only)] [int8 xq] [fp32 xs] [int32 xsum]
    const size_t off_y = xdev ? 0 : up((size_t)n * 4);
    const size_t off_xq = off_y + (ydev ? 0 : up((size_t)d * 4));
    const size_t off_xs = off_xq + up((size_t)n), off_xsum = off_xs + up((size_t)ng * 4);
    rc = ensure_scratch(c, off_xsum + up((size_t)ng * 4));
    if (rc) return rc;
    char* sc = static_cast<char*>(c->scratch);
    float* yd = ydev ? xout : reinterpret_cast<float*>(sc + off_y);
    // the call's work on stream st: copy x in (host x), the activation
    // quantizer (quantize_act, runq.c:117-139), then the GEMV from the int8
    // activation (it streams its first weights while the quantizer runs),
    // copy y out (host y)
    auto enqueue = [&](cudaStream_t st, bool pdl_first) -> int {
        const float* xd = x;
        if (!xdev) {
            cudaError_t e = cudaMemcpyAsync(sc, x, (size_t)n * 4, cudaMemcpyHostToDevice, st);
            if (e != cudaSuccess) return cuda_fail(e, "matmul_f32: copy of x");
            xd = reinterpret_cast<const float*>(sc);
        }
        int r = lq::matmul_f32_device(yd, xd, w, n, d, reinterpret_cast<int8_t*>(sc + off_xq),
                                      reinterpret_cast<float*>(sc + off_xs), reinterpret_cast<int*>(sc + off_xsum),
                                      c->err, st, pdl_first, c->num_sms, g_trace);
        if (r) return r;
        if (!ydev) {
            cudaError_t e = cudaMemcpyAsync(xout, yd, (size_t)d * 4, cudaMemcpyDeviceToHost, st);
            if (e != cudaSuccess) return cuda_fail(e, "matmul_f32: copy of y");
        }
        return LQ_OK;
    };
    auto finish = [&]() -> int {
        if (xdev && ydev) return LQ_OK;  // device buffers: asynchronous like matmul
        cudaError_t e = cudaStreamSynchronize(g_stream);
        return e == cudaSuccess ? LQ_OK : cuda_fail(e, "matmul_f32");
    };
    // page-locked host x and y: one graph launch per call from the second
    // call with the same buffers, weight and shape on
    cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
    const bool graphable = !xdev && !ydev && !g_trace && is_pinned_host_ptr(x) && is_pinned_host_ptr(xout) &&
                           cudaStreamIsCapturing(g_stream, &cs) == cudaSuccess && cs == cudaStreamCaptureStatusNone;
    if (graphable) {
        DevCtx::CallGraph* g = nullptr;
        for (auto& k : c->graphs)
            if (k.x == x && k.y == xout && k.wq == w->q && k.ws == w->s && k.kind == w->kind &&
                k.gs == w->group_size && k.n == n && k.d == d && k.flags == g_launch_flags) {
                g = &k;
                break;
            }
        if (g && g->exec) {
            g->used = ++c->tick;
            cudaError_t e = cudaGraphLaunch(g->exec, g_stream);
            if (e != cudaSuccess) return cuda_fail(e, "matmul_f32: graph launch");
            return finish();
        }
        if (g && !g->failed) {
            // second call with this key: capture the call on the private stream
            if (!c->capture && cudaStreamCreateWithFlags(&c->capture, cudaStreamNonBlocking) != cudaSuccess) {
                cudaGetLastError();
                c->capture = nullptr;
            }
            cudaGraph_t graph = nullptr;
            cudaGraphExec_t exec = nullptr;
            bool ok = c->capture && cudaStreamBeginCapture(c->capture, cudaStreamCaptureModeThreadLocal) == cudaSuccess;
            if (ok) {
                ok = enqueue(c->capture, false) == LQ_OK;
                ok = cudaStreamEndCapture(c->capture, &graph) == cudaSuccess && ok;
            }
            ok = ok && cudaGraphInstantiate(&exec, graph, 0) == cudaSuccess;
            if (graph) cudaGraphDestroy(graph);
            if (!ok) {
                cudaGetLastError();
                if (exec) cudaGraphExecDestroy(exec);
                g->failed = true;  // this key runs call by call from now on
            } else {
                g->exec = exec;
                g->used = ++c->tick;
                cudaError_t e = cudaGraphLaunch(exec, g_stream);
                if (e != cudaSuccess) return cuda_fail(e, "matmul_f32: graph launch");
                return finish();
            }
        } else if (!g) {
            // first call with this key: remember it (64 keys, least recently used dropped)
            if (c->graphs.size() >= 64) {
                auto old = c->graphs.begin();
                for (auto it = c->graphs.begin(); it != c->graphs.end(); ++it)
                    if (it->used < old->used) old = it;
                if (old->exec) cudaGraphExecDestroy(old->exec);
                c->graphs.erase(old);
            }
            c->graphs.push_back({x, xout, w->q, w->s, w->kind, w->group_size, n, d, g_launch_flags, nullptr, false,
                                 ++c->tick});
        }
    }
    rc = enqueue(g_stream, g_launch_flags & LQ_LAUNCH_PDL);
    if (rc) return rc;
    return finish();
}

}  // extern "C"
