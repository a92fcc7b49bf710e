// runtime.cu — the C ABI declared in include/lightx2v_cuda.h: contexts,
// activation buffers, weight upload into the device layout, linear dispatch,
// errors and per-op profiling.
#include <cuda.h>
#include <cuda_runtime.h>
#include <cudaTypedefs.h>
#include <cuda_fp16.h>
#include <dlfcn.h>
#include <nccl.h>

#include <algorithm>
#include <chrono>
#include <climits>
#include <cmath>
#include <cstdarg>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <initializer_list>
#include <map>
#include <mutex>
#include <string>
#include <vector>
#include <limits>

#include "../../include/lightx2v_cuda.h"
#include "dequant.cuh"
#include "gemm.h"
#include "attention.h"
#include "kvcache.h"
#include "dit_ops.h"
#include "peer.h"
#include "sparse.h"

using namespace lx2v;

struct ProfEntry {
    uint64_t calls = 0;
    double ms = 0.0;
};
struct PendingEvent {
    std::string op;
    cudaEvent_t a, b;
};

struct lx2v_ctx {
    int dev = 0;
    ncclComm_t comm = nullptr;   // tensor-parallel group (lx2v_comm_init)
    int comm_rank = 0, comm_world = 1;
    int num_sms = 0;
    cudaStream_t stream = nullptr;
    int *err_dev = nullptr;
    uint64_t wait_limit_ns = 2000000000ull;
    int path = 0;
    int token_tile = 0;
    int split_mode = 0;          // 0 automatic, 1 whole tiles, 2 stream-K
    void *sk_ws = nullptr;       // stream-K workspace: partial tiles + flags
    size_t sk_ws_bytes = 0;
    int sk_epoch = 0;
    float *gemv_ws = nullptr;    // few-token kernel: split-K partials + arrival counters
    // Two-pass linear: the weight decoded to bf16, in two buffers used in
    // turn (a call's decode runs while the previous call's GEMM still reads
    // the other one).
    void *dq_ws[2] = {nullptr, nullptr};
    size_t dq_ws_bytes = 0;
    int dq_next = 0;
    size_t gemv_ws_floats = 0;
    int *gemv_arrivals = nullptr;
    size_t gemv_tiles = 0;
    void *att_ws = nullptr;      // attention: mask bits / temporal indices
    size_t att_ws_bytes = 0;
    void *kv_tmp = nullptr;      // KV cache: staging of row moves (splice / evict)
    size_t kv_tmp_bytes = 0;
    void *att_host = nullptr;    // page-locked staging of the mask data (reused once its copy is done)
    size_t att_host_bytes = 0;
    cudaEvent_t att_host_ev = nullptr;
    uint64_t launches = 0;
    bool profile = false;
    std::map<std::string, ProfEntry> prof;
    std::vector<PendingEvent> pending;
    std::vector<cudaEvent_t> event_pool;
    void *staging = nullptr;
    size_t staging_bytes = 0;
    // Host -> device copies of lx2v_buf_write_f32 / upload run on their own
    // stream, so that they overlap kernels queued before them: each copy
    // waits only for the last kernel that used its destination, and the
    // compute stream waits for the copy before anything queued after it.
    cudaStream_t h2d = nullptr;
    void *wstage = nullptr;            // f32 landing area of writes into bf16 buffers
    size_t wstage_bytes = 0;
    cudaEvent_t wstage_ev = nullptr;   // the last convert that read wstage
    bool wstage_used = false;
    std::string last_err;
    PFN_cuTensorMapEncodeTiled_v12000 encode = nullptr;
};

struct lx2v_buf {
    void *ptr = nullptr;
    size_t len = 0;
    int dtype = LX2V_BF16;
    cudaEvent_t last_use = nullptr;  // recorded on the compute stream after each op that touches the buffer
    bool ipc = false;                // a peer's buffer mapped by CUDA IPC (closed, not freed)
};

struct lx2v_weight {
    int fmt = LX2V_W_BF16;
    size_t rows = 0, cols = 0, group = 0;
    void *codes = nullptr;
    float *scales_t = nullptr;
    uint32_t *sz_t = nullptr;
    uint8_t *flags = nullptr;  // FP8: [ceil(cols/32)][rows] blocks needing the fix-up / reference formula
};

static thread_local std::string g_init_err;

static lx2v_status fail(lx2v_ctx *ctx, lx2v_status code, const char *fmt, ...) {
    char buf[512];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof buf, fmt, ap);
    va_end(ap);
    if (ctx) ctx->last_err = buf;
    else g_init_err = buf;
    return code;
}

#define CUDA_TRY(ctx, expr)                                                                       \
    do {                                                                                          \
        cudaError_t e_ = (expr);                                                                  \
        if (e_ != cudaSuccess)                                                                    \
            return fail(ctx, e_ == cudaErrorMemoryAllocation ? LX2V_ERR_OOM : LX2V_ERR_CUDA,     \
                        "%s: %s (%s:%d)", #expr, cudaGetErrorString(e_), __FILE__, __LINE__);     \
    } while (0)

static size_t esize(int dtype) { return dtype == LX2V_F32 ? 4 : 2; }

// Record that work just queued on the compute stream reads or writes `b`
// (a later host -> device copy into `b` waits for this point).
static cudaError_t note_use(lx2v_ctx *ctx, const lx2v_buf *b) {
    if (!b) return cudaSuccess;
    lx2v_buf *m = const_cast<lx2v_buf *>(b);
    if (!m->last_use) {
        cudaError_t e = cudaEventCreateWithFlags(&m->last_use, cudaEventDisableTiming);
        if (e != cudaSuccess) return e;
    }
    return cudaEventRecord(m->last_use, ctx->stream);
}
static cudaError_t note_uses(lx2v_ctx *ctx, std::initializer_list<const lx2v_buf *> bufs) {
    for (const lx2v_buf *b : bufs) {
        cudaError_t e = note_use(ctx, b);
        if (e != cudaSuccess) return e;
    }
    return cudaSuccess;
}

static lx2v_status enter(lx2v_ctx *ctx) {
    if (!ctx) return fail(nullptr, LX2V_ERR_INVALID, "null context");
    ctx->last_err.clear();
    CUDA_TRY(ctx, cudaSetDevice(ctx->dev));
    return LX2V_OK;
}

// ---- profiling ---------------------------------------------------------------
struct OpScope {
    lx2v_ctx *ctx;
    const char *op;
    cudaEvent_t a = nullptr;
    OpScope(lx2v_ctx *c, const char *name) : ctx(c), op(name) {
        if (!ctx->profile) return;
        a = take();
        cudaEventRecord(a, ctx->stream);
    }
    cudaEvent_t take() {
        if (!ctx->event_pool.empty()) {
            cudaEvent_t e = ctx->event_pool.back();
            ctx->event_pool.pop_back();
            return e;
        }
        cudaEvent_t e = nullptr;
        cudaEventCreate(&e);
        return e;
    }
    ~OpScope() {
        if (!ctx->profile || !a) return;
        cudaEvent_t b = take();
        cudaEventRecord(b, ctx->stream);
        ctx->pending.push_back({op, a, b});
    }
};

static void resolve_profile(lx2v_ctx *ctx) {
    if (ctx->pending.empty()) return;
    cudaStreamSynchronize(ctx->stream);
    for (auto &p : ctx->pending) {
        float ms = 0.0f;
        cudaEventElapsedTime(&ms, p.a, p.b);
        auto &e = ctx->prof[p.op];
        e.calls += 1;
        e.ms += ms;
        ctx->event_pool.push_back(p.a);
        ctx->event_pool.push_back(p.b);
    }
    ctx->pending.clear();
}

// Stream-K workspace: `pairs` x 2 partial tiles of 128 x bt f32, then the
// pairs x 2 publication flags (zeroed when the workspace is allocated; they
// hold launch epochs, so they never need clearing afterwards).
static lx2v_status ensure_sk_workspace(lx2v_ctx *ctx, int pairs, int bt, float **partials, int **flags) {
    // >= pairs x 2 CTAs x 8 flags (the two-pass kernel has one per epilogue warp)
    const size_t flag_bytes = (size_t)ctx->num_sms * 2 * 8 * sizeof(int);
    const size_t part_bytes = (size_t)pairs * 2 * 128 * bt * sizeof(float);
    if (ctx->sk_ws_bytes < part_bytes + flag_bytes) {
        if (ctx->sk_ws) {
            CUDA_TRY(ctx, cudaStreamSynchronize(ctx->stream));
            cudaFree(ctx->sk_ws);
            ctx->sk_ws = nullptr;
            ctx->sk_ws_bytes = 0;
        }
        // sized for the largest tile (256 tokens) on every SM pair at once
        const size_t dflt = (size_t)((ctx->num_sms + 1) / 2) * 2 * 128 * 256 * sizeof(float);
        const size_t bytes = (dflt > part_bytes ? dflt : part_bytes) + flag_bytes;
        CUDA_TRY(ctx, cudaMalloc(&ctx->sk_ws, bytes));
        CUDA_TRY(ctx, cudaMemsetAsync(ctx->sk_ws, 0, bytes, ctx->stream));
        ctx->sk_ws_bytes = bytes;
    }
    *partials = (float *)ctx->sk_ws;
    *flags = (int *)((char *)ctx->sk_ws + (ctx->sk_ws_bytes - flag_bytes));
    return LX2V_OK;
}

// Few-token kernel workspace for an output width N: partial tiles, then one
// arrival counter per 64-row tile (zeroed here; the kernel leaves them zero).
static lx2v_status ensure_gemv_workspace(lx2v_ctx *ctx, int N, int K) {
    const size_t floats = gemv_workspace_floats(N, K, ctx->num_sms);
    const size_t tiles = (size_t)(N + 63) / 64;
    if (ctx->gemv_ws_floats >= floats && ctx->gemv_tiles >= tiles) return LX2V_OK;
    if (ctx->gemv_ws) {
        CUDA_TRY(ctx, cudaStreamSynchronize(ctx->stream));
        cudaFree(ctx->gemv_ws);
        ctx->gemv_ws = nullptr;
    }
    const size_t f = floats > ctx->gemv_ws_floats ? floats : ctx->gemv_ws_floats;
    const size_t t = tiles > ctx->gemv_tiles ? tiles : ctx->gemv_tiles;
    const size_t bytes = f * sizeof(float) + t * sizeof(int);
    CUDA_TRY(ctx, cudaMalloc(&ctx->gemv_ws, bytes));
    CUDA_TRY(ctx, cudaMemsetAsync(ctx->gemv_ws, 0, bytes, ctx->stream));
    ctx->gemv_ws_floats = f;
    ctx->gemv_tiles = t;
    ctx->gemv_arrivals = (int *)(ctx->gemv_ws + f);
    return LX2V_OK;
}

// Two-pass linear workspace: two bf16 [N][K] buffers (grow-only). The
// decode of call n writes buffer n % 2 while the GEMM of call n - 1 may
// still read the other; the GEMM of call n - 2, the last reader of buffer
// n % 2, has completed by then (each decode waits for its predecessor in the
// stream before it exits, and each GEMM for its decode before it lets the
// next kernel start).
static lx2v_status ensure_dq_workspace(lx2v_ctx *ctx, size_t bytes) {
    if (ctx->dq_ws_bytes >= bytes) return LX2V_OK;
    if (ctx->dq_ws[0] || ctx->dq_ws[1]) {
        CUDA_TRY(ctx, cudaStreamSynchronize(ctx->stream));
        for (void *&b : ctx->dq_ws) {
            if (b) cudaFree(b);
            b = nullptr;
        }
        ctx->dq_ws_bytes = 0;
    }
    CUDA_TRY(ctx, cudaMalloc(&ctx->dq_ws[0], bytes));
    CUDA_TRY(ctx, cudaMalloc(&ctx->dq_ws[1], bytes));
    ctx->dq_ws_bytes = bytes;
    return LX2V_OK;
}

static lx2v_status ensure_staging(lx2v_ctx *ctx, size_t bytes) {
    if (ctx->staging_bytes >= bytes) return LX2V_OK;
    if (ctx->staging) {
        CUDA_TRY(ctx, cudaStreamSynchronize(ctx->stream));
        cudaFree(ctx->staging);
        ctx->staging = nullptr;
        ctx->staging_bytes = 0;
    }
    size_t want = bytes < (1u << 20) ? (1u << 20) : bytes;
    CUDA_TRY(ctx, cudaMalloc(&ctx->staging, want));
    ctx->staging_bytes = want;
    return LX2V_OK;
}

// Workspaces a linear on an N x K weight may need, sized when the weight is
// uploaded (a blocking call) so that no linear allocates or synchronises:
// the two-pass decode buffers, the few-token split-K partials and the
// stream-K partial tiles. They only grow; lx2v_linear still grows them if a
// caller forces a path or tile the upload did not plan for.
static lx2v_status plan_workspaces(lx2v_ctx *ctx, int fmt, size_t rows, size_t cols) {
    lx2v_status s = LX2V_OK;
    if (fmt != LX2V_W_BF16 && (s = ensure_dq_workspace(ctx, rows * cols * 2))) return s;
    if (cols % 64 == 0 && (s = ensure_gemv_workspace(ctx, (int)rows, (int)cols))) return s;
    float *partials = nullptr;
    int *flags = nullptr;
    return ensure_sk_workspace(ctx, ctx->num_sms / 2, 256, &partials, &flags);
}

// ---- context -------------------------------------------------------------------
extern "C" lx2v_status lx2v_init(int device, lx2v_ctx **out) {
    if (!out) return fail(nullptr, LX2V_ERR_INVALID, "null output pointer");
    *out = nullptr;
    int n = 0;
    if (cudaGetDeviceCount(&n) != cudaSuccess || n == 0)
        return fail(nullptr, LX2V_ERR_NO_DEVICE, "no CUDA device is visible");
    if (device < 0 || device >= n)
        return fail(nullptr, LX2V_ERR_NO_DEVICE, "device %d out of range (%d visible)", device, n);
    cudaDeviceProp prop;
    if (cudaGetDeviceProperties(&prop, device) != cudaSuccess)
        return fail(nullptr, LX2V_ERR_NO_DEVICE, "cannot query device %d", device);
    if (prop.major != 10)
        return fail(nullptr, LX2V_ERR_NO_DEVICE,
                    "device %d is sm_%d%d; this library is built for sm_100a (B200)", device,
                    prop.major, prop.minor);
    auto *ctx = new lx2v_ctx();
    ctx->dev = device;
    ctx->num_sms = prop.multiProcessorCount;
    cudaError_t e = cudaSetDevice(device);
    if (e == cudaSuccess) e = cudaStreamCreateWithFlags(&ctx->stream, cudaStreamNonBlocking);
    if (e == cudaSuccess) e = cudaStreamCreateWithFlags(&ctx->h2d, cudaStreamNonBlocking);
    if (e == cudaSuccess) e = cudaEventCreateWithFlags(&ctx->wstage_ev, cudaEventDisableTiming);
    if (e == cudaSuccess) e = cudaMalloc(&ctx->err_dev, sizeof(int));
    if (e == cudaSuccess) e = cudaMemset(ctx->err_dev, 0, sizeof(int));
    if (e != cudaSuccess) {
        lx2v_status st = fail(nullptr, LX2V_ERR_CUDA, "context setup: %s", cudaGetErrorString(e));
        lx2v_free_ctx(ctx);
        return st;
    }
    void *fn = nullptr;
    cudaDriverEntryPointQueryResult q;
    e = cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q);
    if (e != cudaSuccess || q != cudaDriverEntryPointSuccess || !fn) {
        lx2v_free_ctx(ctx);
        return fail(nullptr, LX2V_ERR_CUDA, "cuTensorMapEncodeTiled not available from the driver");
    }
    ctx->encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
    const char *pe = getenv("LIGHTX2V_PROFILE");
    ctx->profile = pe && strcmp(pe, "0") != 0;
    *out = ctx;
    return LX2V_OK;
}

static void comm_destroy(lx2v_ctx *ctx);

extern "C" void lx2v_free_ctx(lx2v_ctx *ctx) {
    if (!ctx) return;
    cudaSetDevice(ctx->dev);
    if (ctx->stream) cudaStreamSynchronize(ctx->stream);
    comm_destroy(ctx);
    for (auto &p : ctx->pending) {
        cudaEventDestroy(p.a);
        cudaEventDestroy(p.b);
    }
    for (auto e : ctx->event_pool) cudaEventDestroy(e);
    if (ctx->h2d) cudaStreamSynchronize(ctx->h2d);
    if (ctx->staging) cudaFree(ctx->staging);
    if (ctx->wstage) cudaFree(ctx->wstage);
    if (ctx->wstage_ev) cudaEventDestroy(ctx->wstage_ev);
    if (ctx->h2d) cudaStreamDestroy(ctx->h2d);
    if (ctx->sk_ws) cudaFree(ctx->sk_ws);
    if (ctx->gemv_ws) cudaFree(ctx->gemv_ws);
    if (ctx->att_ws) cudaFree(ctx->att_ws);
    if (ctx->att_host) cudaFreeHost(ctx->att_host);
    if (ctx->kv_tmp) cudaFree(ctx->kv_tmp);
    if (ctx->att_host_ev) cudaEventDestroy(ctx->att_host_ev);
    for (void *b : ctx->dq_ws)
        if (b) cudaFree(b);
    if (ctx->err_dev) cudaFree(ctx->err_dev);
    if (ctx->stream) cudaStreamDestroy(ctx->stream);
    delete ctx;
}

extern "C" const char *lx2v_last_error(const lx2v_ctx *ctx) {
    return ctx ? ctx->last_err.c_str() : g_init_err.c_str();
}

extern "C" lx2v_status lx2v_name(lx2v_ctx *ctx, char *buf, size_t cap) {
    lx2v_status s = enter(ctx);
    if (s) return s;
    cudaDeviceProp prop;
    CUDA_TRY(ctx, cudaGetDeviceProperties(&prop, ctx->dev));
    char tmp[320];
    snprintf(tmp, sizeof tmp, "cuda:%d (%s, sm_%d%d, %d SMs)", ctx->dev, prop.name, prop.major,
             prop.minor, prop.multiProcessorCount);
    if (!buf || cap == 0) return fail(ctx, LX2V_ERR_INVALID, "null buffer");
    snprintf(buf, cap, "%s", tmp);
    return LX2V_OK;
}

static cudaError_t clear_split_flags(lx2v_ctx *ctx);

static lx2v_status check_device_error(lx2v_ctx *ctx) {
    int h = 0;
    CUDA_TRY(ctx, cudaMemcpyAsync(&h, ctx->err_dev, sizeof(int), cudaMemcpyDeviceToHost, ctx->stream));
    CUDA_TRY(ctx, cudaStreamSynchronize(ctx->stream));
    if (h != 0) {
        // a stopped stream-K launch may have left flags set that no owner
        // consumed; clear them so that no later launch reads stale partials
        CUDA_TRY(ctx, clear_split_flags(ctx));
        CUDA_TRY(ctx, cudaMemsetAsync(ctx->err_dev, 0, sizeof(int), ctx->stream));
        CUDA_TRY(ctx, cudaStreamSynchronize(ctx->stream));
        return fail(ctx, LX2V_ERR_DEVICE,
                    "a kernel stopped: a pipeline wait exceeded the %llu ns limit (code %d)",
                    (unsigned long long)ctx->wait_limit_ns, h);
    }
    return LX2V_OK;
}

extern "C" lx2v_status lx2v_sync(lx2v_ctx *ctx) {
    lx2v_status s = enter(ctx);
    if (s) return s;
    CUDA_TRY(ctx, cudaStreamSynchronize(ctx->stream));
    return check_device_error(ctx);
}

extern "C" void *lx2v_stream(lx2v_ctx *ctx) { return ctx ? (void *)ctx->stream : nullptr; }

// ---- buffers -----------------------------------------------------------------------
static bool valid_dtype(int d) { return d == LX2V_BF16 || d == LX2V_F32; }

extern "C" lx2v_status lx2v_buf_alloc(lx2v_ctx *ctx, size_t len, int dtype, lx2v_buf **out) {
    lx2v_status s = enter(ctx);
    if (s) return s;
    if (!out || !valid_dtype(dtype)) return fail(ctx, LX2V_ERR_INVALID, "bad output or dtype");
    auto *b = new lx2v_buf();
    b->len = len;
    b->dtype = dtype;
    if (len) {
        cudaError_t e = cudaMalloc(&b->ptr, len * esize(dtype));
        if (e == cudaSuccess) e = cudaMemsetAsync(b->ptr, 0, len * esize(dtype), ctx->stream);
        if (e == cudaSuccess) e = note_use(ctx, b);
        if (e != cudaSuccess) {
            if (b->ptr) cudaFree(b->ptr);
            delete b;
            return fail(ctx, e == cudaErrorMemoryAllocation ? LX2V_ERR_OOM : LX2V_ERR_CUDA,
                        "alloc of %zu elements: %s", len, cudaGetErrorString(e));
        }
    }
    *out = b;
    return LX2V_OK;
}

// Host -> device: the copy runs on the h2d stream once the last kernel that
// used its destination is done (so it overlaps any other queued work), and
// the compute stream waits for it before whatever is queued next. bf16
// buffers land in f32 in `wstage` and are converted on the compute stream.
static lx2v_status write_f32(lx2v_ctx *ctx, lx2v_buf *b, const float *data, size_t len) {
    if (len == 0) return LX2V_OK;
    void *dst = b->ptr;
    if (b->dtype != LX2V_F32) {
        if (ctx->wstage_bytes < len * 4) {
            CUDA_TRY(ctx, cudaStreamSynchronize(ctx->stream));
            CUDA_TRY(ctx, cudaStreamSynchronize(ctx->h2d));
            if (ctx->wstage) cudaFree(ctx->wstage);
            ctx->wstage = nullptr;
            ctx->wstage_bytes = 0;
            ctx->wstage_used = false;
            CUDA_TRY(ctx, cudaMalloc(&ctx->wstage, len * 4));
            ctx->wstage_bytes = len * 4;
        }
        if (ctx->wstage_used) CUDA_TRY(ctx, cudaStreamWaitEvent(ctx->h2d, ctx->wstage_ev, 0));
        dst = ctx->wstage;
    } else if (b->last_use) {
        CUDA_TRY(ctx, cudaStreamWaitEvent(ctx->h2d, b->last_use, 0));
    }
    cudaEvent_t done = nullptr;
    CUDA_TRY(ctx, cudaEventCreateWithFlags(&done, cudaEventDisableTiming));
    cudaError_t e = cudaMemcpyAsync(dst, data, len * 4, cudaMemcpyHostToDevice, ctx->h2d);
    if (e == cudaSuccess) e = cudaEventRecord(done, ctx->h2d);
    if (e == cudaSuccess) e = cudaStreamWaitEvent(ctx->stream, done, 0);
    cudaEventDestroy(done);  // released once recorded work completes
    CUDA_TRY(ctx, e);
    if (b->dtype != LX2V_F32) {
        CUDA_TRY(ctx, convert_launch(ctx->wstage, 1, b->ptr, 0, len, ctx->stream));
        ctx->launches++;
        CUDA_TRY(ctx, cudaEventRecord(ctx->wstage_ev, ctx->stream));
        ctx->wstage_used = true;
    }
    CUDA_TRY(ctx, note_use(ctx, b));
    return LX2V_OK;
}

extern "C" lx2v_status lx2v_buf_upload_f32(lx2v_ctx *ctx, const float *data, size_t len, int dtype,
                                           lx2v_buf **out) {
    lx2v_status s = enter(ctx);
    if (s) return s;
    if (!out || (len && !data) || !valid_dtype(dtype)) return fail(ctx, LX2V_ERR_INVALID, "bad arguments");
    OpScope ps(ctx, "upload");
    lx2v_buf *b = nullptr;
    s = lx2v_buf_alloc(ctx, len, dtype, &b);
    if (s) return s;
    s = write_f32(ctx, b, data, len);
    if (s) {
        lx2v_buf_free(ctx, b);
        return s;
    }
    *out = b;
    return LX2V_OK;
}

extern "C" lx2v_status lx2v_buf_write_f32(lx2v_ctx *ctx, lx2v_buf *buf, const float *data, size_t len) {
    lx2v_status s = enter(ctx);
    if (s) return s;
    if (!buf || (len && !data)) return fail(ctx, LX2V_ERR_INVALID, "null buffer or data");
    if (len > buf->len) return fail(ctx, LX2V_ERR_INVALID, "write of %zu elements into a buffer of %zu", len, buf->len);
    OpScope ps(ctx, "write");
    return write_f32(ctx, buf, data, len);
}

// Device -> host on the compute stream (after everything queued before).
static lx2v_status queue_download(lx2v_ctx *ctx, const lx2v_buf *buf, float *out, size_t len) {
    if (len == 0) return LX2V_OK;
    if (buf->dtype == LX2V_F32) {
        CUDA_TRY(ctx, cudaMemcpyAsync(out, buf->ptr, len * 4, cudaMemcpyDeviceToHost, ctx->stream));
    } else {
        lx2v_status s = ensure_staging(ctx, len * 4);
        if (s) return s;
        CUDA_TRY(ctx, convert_launch(buf->ptr, 0, ctx->staging, 1, len, ctx->stream));
        ctx->launches++;
        CUDA_TRY(ctx, cudaMemcpyAsync(out, ctx->staging, len * 4, cudaMemcpyDeviceToHost, ctx->stream));
    }
    CUDA_TRY(ctx, note_use(ctx, buf));
    return LX2V_OK;
}

extern "C" lx2v_status lx2v_buf_download_f32(lx2v_ctx *ctx, const lx2v_buf *buf, float *out, size_t len) {
    lx2v_status s = enter(ctx);
    if (s) return s;
    if (!buf || (len && !out)) return fail(ctx, LX2V_ERR_INVALID, "null buffer or output");
    if (len > buf->len) return fail(ctx, LX2V_ERR_INVALID, "download of %zu elements from a buffer of %zu", len, buf->len);
    {
        OpScope ps(ctx, "download");
        s = queue_download(ctx, buf, out, len);
        if (s) return s;
    }
    CUDA_TRY(ctx, cudaStreamSynchronize(ctx->stream));
    return check_device_error(ctx);
}

extern "C" lx2v_status lx2v_buf_download_f32_async(lx2v_ctx *ctx, const lx2v_buf *buf, float *out, size_t len) {
    lx2v_status s = enter(ctx);
    if (s) return s;
    if (!buf || (len && !out)) return fail(ctx, LX2V_ERR_INVALID, "null buffer or output");
    if (len > buf->len) return fail(ctx, LX2V_ERR_INVALID, "download of %zu elements from a buffer of %zu", len, buf->len);
    OpScope ps(ctx, "download_async");
    return queue_download(ctx, buf, out, len);
}

extern "C" lx2v_status lx2v_buf_len(lx2v_ctx *ctx, const lx2v_buf *buf, size_t *len) {
    if (!ctx) return fail(nullptr, LX2V_ERR_INVALID, "null context");
    if (!buf || !len) return fail(ctx, LX2V_ERR_INVALID, "null buffer or output");
    *len = buf->len;
    return LX2V_OK;
}

extern "C" lx2v_status lx2v_buf_info(lx2v_ctx *ctx, const lx2v_buf *buf, int *dtype, void **dev_ptr) {
    if (!ctx) return fail(nullptr, LX2V_ERR_INVALID, "null context");
    if (!buf) return fail(ctx, LX2V_ERR_INVALID, "null buffer");
    if (dtype) *dtype = buf->dtype;
    if (dev_ptr) *dev_ptr = buf->ptr;
    return LX2V_OK;
}

extern "C" lx2v_status lx2v_buf_copy(lx2v_ctx *ctx, const lx2v_buf *src, size_t src_off, lx2v_buf *dst,
                                     size_t dst_off, size_t len) {
    lx2v_status s = enter(ctx);
    if (s) return s;
    if (!src || !dst) return fail(ctx, LX2V_ERR_INVALID, "null buffer");
    if (src_off + len > src->len || dst_off + len > dst->len)
        return fail(ctx, LX2V_ERR_INVALID, "copy range out of bounds");
    if (len == 0) return LX2V_OK;
    OpScope ps(ctx, "copy");
    const char *sp = (const char *)src->ptr + src_off * esize(src->dtype);
    char *dp = (char *)dst->ptr + dst_off * esize(dst->dtype);
    if (src->dtype == dst->dtype) {
        CUDA_TRY(ctx, cudaMemcpyAsync(dp, sp, len * esize(src->dtype), cudaMemcpyDeviceToDevice, ctx->stream));
    } else {
        CUDA_TRY(ctx, convert_launch(sp, src->dtype == LX2V_F32, dp, dst->dtype == LX2V_F32, len, ctx->stream));
        ctx->launches++;
    }
    CUDA_TRY(ctx, note_uses(ctx, {src, dst}));
    return LX2V_OK;
}

extern "C" void lx2v_buf_free(lx2v_ctx *ctx, lx2v_buf *buf) {
    if (!buf) return;
    if (ctx) {
        cudaSetDevice(ctx->dev);
        cudaStreamSynchronize(ctx->stream);
    }
    if (buf->ptr) {
        if (buf->ipc) cudaIpcCloseMemHandle(buf->ptr);
        else cudaFree(buf->ptr);
    }
    if (buf->last_use) cudaEventDestroy(buf->last_use);
    delete buf;
}

// ---- weights -------------------------------------------------------------------------
static void weight_release(lx2v_weight *w) {
    if (!w) return;
    if (w->codes) cudaFree(w->codes);
    if (w->scales_t) cudaFree(w->scales_t);
    if (w->sz_t) cudaFree(w->sz_t);
    if (w->flags) cudaFree(w->flags);
    delete w;
}

static lx2v_status check_shape(lx2v_ctx *ctx, size_t rows, size_t cols, size_t group) {
    if (rows == 0 || cols == 0) return fail(ctx, LX2V_ERR_INVALID, "empty weight %zux%zu", rows, cols);
    if (rows > (1u << 30) || cols > (1u << 30)) return fail(ctx, LX2V_ERR_UNSUPPORTED, "weight too large");
    if (group == 0 || cols % group != 0)
        return fail(ctx, LX2V_ERR_INVALID, "group %zu does not divide cols %zu", group, cols);
    return LX2V_OK;
}

// Scales [rows, G] -> device [G, rows].
static std::vector<float> transpose_scales(const float *s, size_t rows, size_t G) {
    std::vector<float> t(rows * G);
    for (size_t r = 0; r < rows; ++r)
        for (size_t g = 0; g < G; ++g) t[g * rows + r] = s[r * G + g];
    return t;
}

extern "C" lx2v_status lx2v_weight_f32(lx2v_ctx *ctx, const float *data, size_t rows, size_t cols,
                                       lx2v_weight **out) {
    lx2v_status s = enter(ctx);
    if (s) return s;
    if (!out || !data) return fail(ctx, LX2V_ERR_INVALID, "null data or output");
    if ((s = check_shape(ctx, rows, cols, cols))) return s;
    OpScope ps(ctx, "weight");
    auto *w = new lx2v_weight();
    w->fmt = LX2V_W_BF16;
    w->rows = rows; w->cols = cols; w->group = cols;
    const size_t n = rows * cols;
    cudaError_t e = cudaMalloc(&w->codes, n * 2);
    if (e != cudaSuccess) { weight_release(w); return fail(ctx, LX2V_ERR_OOM, "weight alloc: %s", cudaGetErrorString(e)); }
    if ((s = ensure_staging(ctx, n * 4))) { weight_release(w); return s; }
    e = cudaMemcpyAsync(ctx->staging, data, n * 4, cudaMemcpyHostToDevice, ctx->stream);
    if (e == cudaSuccess) e = convert_launch(ctx->staging, 1, w->codes, 0, n, ctx->stream);
    if (e == cudaSuccess) e = cudaStreamSynchronize(ctx->stream);
    ctx->launches++;
    if (e != cudaSuccess) { weight_release(w); return fail(ctx, LX2V_ERR_CUDA, "weight upload: %s", cudaGetErrorString(e)); }
    if ((s = plan_workspaces(ctx, LX2V_W_BF16, rows, cols))) { weight_release(w); return s; }
    *out = w;
    return LX2V_OK;
}

static lx2v_status upload_codes_scales(lx2v_ctx *ctx, lx2v_weight *w, const void *codes, size_t code_bytes,
                                       const std::vector<float> *scales_t, const std::vector<uint32_t> *sz_t) {
    cudaError_t e = cudaMalloc(&w->codes, code_bytes < 16 ? 16 : code_bytes);
    if (e == cudaSuccess) e = cudaMemcpy(w->codes, codes, code_bytes, cudaMemcpyHostToDevice);
    if (e == cudaSuccess && scales_t) {
        e = cudaMalloc(&w->scales_t, scales_t->size() * 4);
        if (e == cudaSuccess) e = cudaMemcpy(w->scales_t, scales_t->data(), scales_t->size() * 4, cudaMemcpyHostToDevice);
    }
    if (e == cudaSuccess && sz_t) {
        e = cudaMalloc(&w->sz_t, sz_t->size() * 4);
        if (e == cudaSuccess) e = cudaMemcpy(w->sz_t, sz_t->data(), sz_t->size() * 4, cudaMemcpyHostToDevice);
    }
    if (e != cudaSuccess)
        return fail(ctx, e == cudaErrorMemoryAllocation ? LX2V_ERR_OOM : LX2V_ERR_CUDA, "weight upload: %s",
                    cudaGetErrorString(e));
    return LX2V_OK;
}

extern "C" lx2v_status lx2v_weight_q8(lx2v_ctx *ctx, const int8_t *q, const float *scales, size_t rows,
                                      size_t cols, size_t group, lx2v_weight **out) {
    lx2v_status s = enter(ctx);
    if (s) return s;
    if (!out || !q || !scales) return fail(ctx, LX2V_ERR_INVALID, "null codes, scales or output");
    if ((s = check_shape(ctx, rows, cols, group))) return s;
    OpScope ps(ctx, "weight_q8");
    auto *w = new lx2v_weight();
    w->fmt = LX2V_W_Q8; w->rows = rows; w->cols = cols; w->group = group;
    auto st = transpose_scales(scales, rows, cols / group);
    if ((s = upload_codes_scales(ctx, w, q, rows * cols, &st, nullptr))) { weight_release(w); return s; }
    if ((s = plan_workspaces(ctx, LX2V_W_Q8, rows, cols))) { weight_release(w); return s; }
    *out = w;
    return LX2V_OK;
}

extern "C" lx2v_status lx2v_weight_fp8(lx2v_ctx *ctx, const uint8_t *q, const float *scales, size_t rows,
                                       size_t cols, size_t group, lx2v_weight **out) {
    lx2v_status s = enter(ctx);
    if (s) return s;
    if (!out || !q || !scales) return fail(ctx, LX2V_ERR_INVALID, "null codes, scales or output");
    if ((s = check_shape(ctx, rows, cols, group))) return s;
    OpScope ps(ctx, "weight_fp8");
    auto *w = new lx2v_weight();
    w->fmt = LX2V_W_FP8; w->rows = rows; w->cols = cols; w->group = group;
    const size_t G = cols / group;
    // One flag byte per (row, 32-column block): 1 = the block holds a code
    // the fast decode does not cover (fixed up exactly), 2 = a scale outside
    // the fast range (reference formula).
    const size_t ku = (size_t)fp8_flag_cols((int)cols);
    std::vector<uint8_t> flags(rows * ku, 0);
    for (size_t r = 0; r < rows; ++r) {
        for (size_t c = 0; c < cols; ++c) {
            uint8_t &f = flags[(c / 32) * rows + r];
            if (!fp8_scale_fast(scales[r * G + c / group])) f = 2;
            else if (fp8_code_special(q[r * cols + c]) && f == 0) f = 1;
        }
    }
    auto st = transpose_scales(scales, rows, G);
    if ((s = upload_codes_scales(ctx, w, q, rows * cols, &st, nullptr))) { weight_release(w); return s; }
    cudaError_t e = cudaMalloc(&w->flags, flags.size() < 16 ? 16 : flags.size());
    if (e == cudaSuccess) e = cudaMemcpy(w->flags, flags.data(), flags.size(), cudaMemcpyHostToDevice);
    if (e != cudaSuccess) {
        weight_release(w);
        return fail(ctx, e == cudaErrorMemoryAllocation ? LX2V_ERR_OOM : LX2V_ERR_CUDA, "weight upload: %s",
                    cudaGetErrorString(e));
    }
    if ((s = plan_workspaces(ctx, LX2V_W_FP8, rows, cols))) { weight_release(w); return s; }
    *out = w;
    return LX2V_OK;
}

// e4m3 as the OCP FP8 format defines it (NVFP4 block scales): exponent-field-0
// codes are m/8 * 2^-6, 0x7F / 0xFF NaN.
static float e4m3_ocp(uint8_t c) {
    const float sign = (c & 0x80u) ? -1.0f : 1.0f;
    const int e = (c >> 3) & 0xF, m = c & 7;
    if (e == 0xF && m == 7) return std::numeric_limits<float>::quiet_NaN();
    if (e == 0) return sign * ((float)m / 8.0f) * 0x1p-6f;
    return sign * (1.0f + (float)m / 8.0f) * std::ldexp(1.0f, e - 7);
}

extern "C" lx2v_status lx2v_weight_nvfp4(lx2v_ctx *ctx, const uint8_t *packed, const uint8_t *block_scales,
                                         float global_scale, size_t rows, size_t cols, lx2v_weight **out) {
    lx2v_status s = enter(ctx);
    if (s) return s;
    if (!out || !packed || !block_scales) return fail(ctx, LX2V_ERR_INVALID, "null codes, scales or output");
    if ((s = check_shape(ctx, rows, cols, 16))) return s;
    if (cols % 32 != 0) return fail(ctx, LX2V_ERR_UNSUPPORTED, "NVFP4 rows of a multiple of 32 values");
    OpScope ps(ctx, "weight_nvfp4");
    auto *w = new lx2v_weight();
    w->fmt = LX2V_W_NVFP4; w->rows = rows; w->cols = cols; w->group = 16;
    const size_t G = cols / 16;
    std::vector<float> eff(rows * G);  // block scale x global scale, one f32 rounding
    for (size_t i = 0; i < rows * G; ++i) eff[i] = e4m3_ocp(block_scales[i]) * global_scale;
    auto st = transpose_scales(eff.data(), rows, G);
    if ((s = upload_codes_scales(ctx, w, packed, rows * cols / 2, &st, nullptr))) { weight_release(w); return s; }
    if ((s = plan_workspaces(ctx, LX2V_W_NVFP4, rows, cols))) { weight_release(w); return s; }
    *out = w;
    return LX2V_OK;
}

extern "C" lx2v_status lx2v_weight_q4(lx2v_ctx *ctx, const uint8_t *packed, const float *scales,
                                      const float *zeros, size_t rows, size_t cols, size_t group,
                                      lx2v_weight **out) {
    lx2v_status s = enter(ctx);
    if (s) return s;
    if (!out || !packed || !scales || !zeros) return fail(ctx, LX2V_ERR_INVALID, "null codes, scales, zeros or output");
    if ((s = check_shape(ctx, rows, cols, group))) return s;
    OpScope ps(ctx, "weight_q4");
    const size_t G = cols / group;
    std::vector<uint32_t> sz(rows * G);
    for (size_t r = 0; r < rows; ++r) {
        for (size_t g = 0; g < G; ++g) {
            const float sc = scales[r * G + g], ze = zeros[r * G + g];
            const __half hs = __float2half_rn(sc), hz = __float2half_rn(ze);
            const float bs = __half2float(hs), bz = __half2float(hz);
            const bool same = (bs == sc || (std::isnan(bs) && std::isnan(sc))) &&
                              (bz == ze || (std::isnan(bz) && std::isnan(ze)));
            if (!same || (sc == 0.0f && std::signbit(sc) != std::signbit(bs)) ||
                (ze == 0.0f && std::signbit(ze) != std::signbit(bz)))
                return fail(ctx, LX2V_ERR_INVALID,
                            "Q4 scale/zero of row %zu group %zu is not an f16 value (%g, %g)", r, g, sc, ze);
            uint16_t us, uz;
            memcpy(&us, &hs, 2);
            memcpy(&uz, &hz, 2);
            sz[g * rows + r] = (uint32_t)us | ((uint32_t)uz << 16);
        }
    }
    auto *w = new lx2v_weight();
    w->fmt = LX2V_W_Q4; w->rows = rows; w->cols = cols; w->group = group;
    if ((s = upload_codes_scales(ctx, w, packed, (rows * cols + 1) / 2, nullptr, &sz))) { weight_release(w); return s; }
    if ((s = plan_workspaces(ctx, LX2V_W_Q4, rows, cols))) { weight_release(w); return s; }
    *out = w;
    return LX2V_OK;
}

extern "C" void lx2v_weight_free(lx2v_ctx *ctx, lx2v_weight *w) {
    if (!w) return;
    if (ctx) {
        cudaSetDevice(ctx->dev);
        cudaStreamSynchronize(ctx->stream);
    }
    weight_release(w);
}

extern "C" lx2v_status lx2v_weight_info(lx2v_ctx *ctx, const lx2v_weight *w, int *format, size_t *rows,
                                        size_t *cols, size_t *group) {
    if (!ctx) return fail(nullptr, LX2V_ERR_INVALID, "null context");
    if (!w) return fail(ctx, LX2V_ERR_INVALID, "null weight");
    if (format) *format = w->fmt;
    if (rows) *rows = w->rows;
    if (cols) *cols = w->cols;
    if (group) *group = w->group;
    return LX2V_OK;
}

extern "C" lx2v_status lx2v_weight_dequant_f32(lx2v_ctx *ctx, const lx2v_weight *w, float *out) {
    lx2v_status s = enter(ctx);
    if (s) return s;
    if (!w || !out) return fail(ctx, LX2V_ERR_INVALID, "null weight or output");
    const size_t n = w->rows * w->cols;
    if ((s = ensure_staging(ctx, n * 4))) return s;
    CUDA_TRY(ctx, dequant_f32_launch(w->fmt, (const uint8_t *)w->codes, w->scales_t, w->sz_t, w->flags,
                                     (int)w->rows, (int)w->cols, (int)w->group, (float *)ctx->staging,
                                     ctx->stream));
    ctx->launches++;
    CUDA_TRY(ctx, cudaMemcpyAsync(out, ctx->staging, n * 4, cudaMemcpyDeviceToHost, ctx->stream));
    CUDA_TRY(ctx, cudaStreamSynchronize(ctx->stream));
    return LX2V_OK;
}

// ---- linear -----------------------------------------------------------------------------
static lx2v_status make_map(lx2v_ctx *ctx, CUtensorMap *map, const void *base, CUtensorMapDataType dt,
                            size_t esz, uint64_t inner, uint64_t outer, uint32_t box_inner, uint32_t box_outer,
                            CUtensorMapSwizzle sw) {
    cuuint64_t dims[2] = {inner, outer};
    cuuint64_t strides[1] = {inner * esz};
    cuuint32_t box[2] = {box_inner, box_outer};
    cuuint32_t estr[2] = {1, 1};
    CUresult r = ctx->encode(map, dt, 2, const_cast<void *>(base), dims, strides, box, estr,
                             CU_TENSOR_MAP_INTERLEAVE_NONE, sw, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                             CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS)
        return fail(ctx, LX2V_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d) for %llux%llu box %ux%u", (int)r,
                    (unsigned long long)inner, (unsigned long long)outer, box_inner, box_outer);
    return LX2V_OK;
}

// Stream-K pays when whole tiles leave most CTA pairs idle (a grid of fewer
// tiles than pairs, e.g. a few hundred tokens against a long K): it spreads
// the k-blocks over all pairs at the price of one partial tile written and
// read per pair. With several waves of tiles it measured slower than whole
// tiles on B200 (FFN2 of the 1.3B chunk: 762 vs 804 TFLOP/s), so it is only
// taken when it at least shortens the critical path by 40%.
// Stream-K for the two-pass kernel, on request only (lx2v_set_split_mode 2):
// full waves of whole tiles, then the remaining tiles' k-blocks spread evenly
// over all pairs (PairWork::init_split). It would balance the 1.3B chunk's
// N = 1536 linears (114 tiles on 74 pairs) but measured slower on B200 (out
// 423 vs 654, FFN2 1058 vs 1132 TFLOP/s): the partial tiles go through
// per-thread global stores and loads, the traffic the tensor-store epilogue
// avoids, and they sit on the critical path at the end of each pair's work.
// (Splitting every tile into one contiguous range per pair was slower still:
// pairs running at the same time then touch x tiles spread over the whole
// output, which do not fit in L2 together.)
static bool use_streamk_ss(const lx2v_ctx *ctx, int M, int N, int K, int bt, int kgroup) {
    if (ctx->split_mode != 2) return false;
    const int pairs = ctx->num_sms / 2;
    const long long tiles = (long long)((M + bt - 1) / bt) * ((N + 255) / 256);
    const long long kg = ((K + 63) / 64) / kgroup;
    return tiles * kg >= pairs;  // every pair needs at least one group
}

// Rows from which the two-pass linear (decode the weight once to bf16, then a
// GEMM with both operands in shared memory) is the automatic choice for
// quantized weights: below it the one-pass kernel's per-tile decode is
// cheaper than the extra pass over N x K.
static constexpr int TWO_PASS_MIN_ROWS = 1024;
// ... and below that, when the call has so few 256 x 256 output tiles that
// most SMs idle whatever the kernel (measured on B200, K = 8960, N = 1536:
// 135 vs 94 TFLOP/s at 256 rows, 270 vs 226 at 512 rows; with N = 8960 the
// one-pass kernels stay ahead).
static constexpr size_t TWO_PASS_MAX_FEW_TILES = 24;

static bool use_streamk(const lx2v_ctx *ctx, int M, int N, int K, int bt) {
    if (ctx->split_mode == 1) return false;
    const int pairs = ctx->num_sms / 2;
    const long long tiles = (long long)((M + bt - 1) / bt) * ((N + 255) / 256);
    const long long kb = (K + 63) / 64;
    if (tiles * kb < pairs) return false;  // every pair needs at least one k-block
    if (ctx->split_mode == 2) return true;
    const long long waves = (tiles + pairs - 1) / pairs;
    const double whole = (double)waves * kb;                       // k-blocks on the critical path
    const double split = (double)tiles * kb / pairs + 16.0;        // + the partial tile's traffic
    return split < 0.6 * whole;
}

static lx2v_status linear_queue(lx2v_ctx *ctx, const char *opname, const lx2v_buf *x, size_t x_row,
                               size_t rows, const lx2v_weight *w, const lx2v_buf *bias, int act, lx2v_buf *y,
                               size_t y_row, const lx2v_buf *mods, size_t gate) {
    if (!x || !w || !y) return fail(ctx, LX2V_ERR_INVALID, "null x, weight or output");
    if (act != LX2V_ACT_NONE && act != LX2V_ACT_GELU_TANH) return fail(ctx, LX2V_ERR_INVALID, "bad act %d", act);
    if (x == y || (x->ptr && x->ptr == y->ptr)) return fail(ctx, LX2V_ERR_INVALID, "output aliases input");
    const size_t N = w->rows, K = w->cols;
    if ((x_row + rows) * K > x->len)
        return fail(ctx, LX2V_ERR_INVALID, "x has %zu elements, rows [%zu, %zu) x %zu need more", x->len, x_row,
                    x_row + rows, K);
    if ((y_row + rows) * N > y->len)
        return fail(ctx, LX2V_ERR_INVALID, "output has %zu elements, rows [%zu, %zu) x %zu need more", y->len,
                    y_row, y_row + rows, N);
    if (bias && bias->len < N) return fail(ctx, LX2V_ERR_INVALID, "bias has %zu elements, need %zu", bias->len, N);
    if (mods && mods->len < (gate + 1) * N)
        return fail(ctx, LX2V_ERR_INVALID, "mods has %zu elements, gate %zu x %zu needs more", mods->len, gate, N);
    if (rows == 0) return LX2V_OK;
    if (rows > (1u << 30)) return fail(ctx, LX2V_ERR_UNSUPPORTED, "too many rows");
    OpScope ps(ctx, opname);

    const void *gate_ptr = mods ? (const char *)mods->ptr + gate * N * esize(mods->dtype) : nullptr;
    // Tensor-core kernel: 16-byte aligned rows for every TMA map and store,
    // and at most 4 quantization groups per 64-wide k-block.
    const size_t grp = w->group;
    const bool groups_ok = w->fmt == LX2V_W_BF16 || grp % 64 == 0 ||
                           (w->fmt == LX2V_W_Q4 && (grp == 16 || grp == 32));
    const bool tc_ok = x->dtype == LX2V_BF16 && K % 16 == 0 && N % 16 == 0 && groups_ok &&
                       unit_path_ok(w->fmt, (int)K, (int)w->group) && rows >= 16;
    LinearArgs a;
    memset(&a, 0, sizeof a);
    a.fmt = w->fmt; a.codes = (const uint8_t *)w->codes; a.scales_t = w->scales_t; a.sz_t = w->sz_t;
    a.flags = w->flags;
    a.M = (int)rows; a.N = (int)N; a.K = (int)K; a.group = (int)w->group;
    a.x = x->ptr; a.x_f32 = x->dtype == LX2V_F32; a.x_row = (int64_t)x_row;
    a.y = y->ptr; a.y_f32 = y->dtype == LX2V_F32; a.y_row = (int64_t)y_row;
    a.bias = bias ? bias->ptr : nullptr; a.bias_f32 = bias && bias->dtype == LX2V_F32;
    a.gate = gate_ptr; a.gate_f32 = mods && mods->dtype == LX2V_F32;
    a.act = act;
    a.err = ctx->err_dev;
    a.wait_limit_ns = ctx->wait_limit_ns;
    const bool gemv_ok = gemv_supported(a);
    // Two-pass linear (decode once, then both GEMM operands from shared
    // memory): any group size the unit decode takes.
    const bool ss_ok = x->dtype == LX2V_BF16 && K % 16 == 0 && N % 16 == 0 &&
                       unit_path_ok(w->fmt, (int)K, (int)w->group) && rows >= 16;
    int path = ctx->path;
    if (path == 0 && w->fmt == LX2V_W_NVFP4) {
        // NVFP4 runs the two-pass linear (decode to bf16, then the CTA-pair
        // GEMM) at any token count, else the generic kernel
        path = ss_ok && N >= 256 && K % 64 == 0 ? 5 : 3;
    }
    if (path == 0) {
        if (rows <= 16 && gemv_ok) path = 2;
        else if (ss_ok && N >= 256 && K % 64 == 0 &&  // whole 64-wide k-blocks, the shapes it is tested on
                 (rows >= (w->fmt == LX2V_W_BF16 ? 512u : (size_t)TWO_PASS_MIN_ROWS) ||
                  ((rows + 255) / 256) * ((N + 255) / 256) <= TWO_PASS_MAX_FEW_TILES))
            path = 5;
        else if (tc_ok) path = rows >= 512 && N >= 256 ? 4 : 1;
        else path = 3;
    }
    if ((path == 1 || path == 4) && !tc_ok)
        return fail(ctx, LX2V_ERR_UNSUPPORTED, "the tensor-core kernel does not take this shape/dtype");
    if (path == 5 && !ss_ok)
        return fail(ctx, LX2V_ERR_UNSUPPORTED, "the two-pass kernel does not take this shape/dtype");
    if (path == 2) {
        if (!gemv_ok)
            return fail(ctx, LX2V_ERR_UNSUPPORTED,
                        "the few-token kernel takes 1..16 rows, K a multiple of 64 (Q4: 128, or 64 with groups of 64k)");
        lx2v_status s = ensure_gemv_workspace(ctx, (int)N, (int)K);
        if (s) return s;
        CUDA_TRY(ctx, linear_gemv_launch(a, ctx->num_sms, ctx->stream, ctx->gemv_ws, ctx->gemv_arrivals,
                                         ctx->gemv_ws_floats));
        ctx->launches++;
        return LX2V_OK;
    }

    if (path == 5) {
        const void *wa = w->codes;
        if (w->fmt != LX2V_W_BF16) {
            lx2v_status s = ensure_dq_workspace(ctx, N * K * 2);
            if (s) return s;
            void *buf = ctx->dq_ws[ctx->dq_next];
            ctx->dq_next ^= 1;
            CUDA_TRY(ctx, dequant_bf16_launch(w->fmt, (const uint8_t *)w->codes, w->scales_t, w->sz_t, w->flags,
                                              (int)N, (int)K, (int)w->group, (__nv_bfloat16 *)buf, ctx->stream));
            ctx->launches++;
            wa = buf;
        }
        GemmParams p;
        memset(&p, 0, sizeof p);
        const int bt = ctx->token_tile ? ctx->token_tile
                                       : gemm_ss_token_tile((int)rows, (int)N, (int)K, ctx->num_sms / 2);
        lx2v_status s = make_map(ctx, &p.tmap_x, x->ptr, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, K, x_row + rows, 64,
                                 (uint32_t)(bt / 2), CU_TENSOR_MAP_SWIZZLE_128B);
        if (s) return s;
        s = make_map(ctx, &p.tmap_w, wa, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, K, N, 64, 128,
                     CU_TENSOR_MAP_SWIZZLE_128B);
        if (s) return s;
        p.y = y->ptr;
        p.bias = bias ? bias->ptr : nullptr;
        p.bias_f32 = bias && bias->dtype == LX2V_F32;
        p.gate = gate_ptr;
        p.gate_f32 = mods && mods->dtype == LX2V_F32;
        p.err = ctx->err_dev;
        p.wait_limit_ns = ctx->wait_limit_ns;
        p.M = (int)rows; p.N = (int)N; p.K = (int)K; p.group = (int)w->group;
        p.x_row = (int)x_row; p.y_row = (int)y_row;
        p.act = act;
        p.out_f32 = y->dtype == LX2V_F32;
        p.reduce = mods ? 1 : 0;
        p.kgroup = K % 128 == 0 ? 2 : 1;
        // y through TMA tensor stores (reduce-add for an f32 residual); a
        // bf16 residual keeps the kernel's per-element reductions
        if (!(p.reduce && !p.out_f32)) {
            s = make_map(ctx, &p.tmap_y, y->ptr,
                         p.out_f32 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16,
                         p.out_f32 ? 4 : 2, N, y_row + rows, 32, 32, CU_TENSOR_MAP_SWIZZLE_NONE);
            if (s) return s;
            p.tma_y = 1;
        }
        if (use_streamk_ss(ctx, (int)rows, (int)N, (int)K, bt, p.kgroup)) {
            s = ensure_sk_workspace(ctx, ctx->num_sms / 2, bt, &p.partials, &p.flags);
            if (s) return s;
            p.streamk = 1;
            if (++ctx->sk_epoch <= 0) ctx->sk_epoch = 1;
            p.epoch = ctx->sk_epoch;
        } else if (ctx->split_mode == 0 && p.reduce && p.out_f32 && p.tma_y && act == 0) {
            // gated residual into f32 h: k-ranges of a tile reduce-add on their own
            p.ksplit = gemm_ss_ksplit((int)rows, (int)N, (int)K, bt, ctx->num_sms / 2);
            if (p.ksplit > 1 && (long long)((K / 64) / p.kgroup) < p.ksplit) p.ksplit = 1;
        }
        CUDA_TRY(ctx, gemm_ss_pair_launch(bt, p, ctx->num_sms, ctx->stream));
        ctx->launches++;
        return LX2V_OK;
    }

    if (path == 1 || path == 4) {
        const bool pair = path == 4;
        GemmParams p;
        memset(&p, 0, sizeof p);
        const int bt = ctx->token_tile ? ctx->token_tile
                                       : gemm_dq_token_tile((int)rows, (int)N, (int)K, pair ? ctx->num_sms / 2 : ctx->num_sms,
                                                            pair ? 256 : 128);
        lx2v_status s = make_map(ctx, &p.tmap_x, x->ptr, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, K, x_row + rows, 64,
                                 (uint32_t)(pair ? bt / 2 : bt), CU_TENSOR_MAP_SWIZZLE_128B);
        if (s) return s;
        // Code tile of one stage: 128 weight rows x one 64-wide k-block, with
        // the swizzle that makes the dequant threads' row reads conflict free.
        if (w->fmt == LX2V_W_Q4)
            s = make_map(ctx, &p.tmap_w, w->codes, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, K / 2, N, 32, 128,
                         CU_TENSOR_MAP_SWIZZLE_32B);
        else if (w->fmt == LX2V_W_BF16)
            s = make_map(ctx, &p.tmap_w, w->codes, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, K, N, 64, 128,
                         CU_TENSOR_MAP_SWIZZLE_128B);
        else
            s = make_map(ctx, &p.tmap_w, w->codes, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, K, N, 64, 128,
                         CU_TENSOR_MAP_SWIZZLE_64B);
        if (s) return s;
        if (w->fmt != LX2V_W_BF16) {
            const int sgrp = grp % 64 == 0 ? 1 : (int)(64 / grp);
            p.sgrp = sgrp;
            p.gshift = grp % 64 == 0 ? 6 : (grp == 16 ? 4 : 5);
            s = make_map(ctx, &p.tmap_s, w->fmt == LX2V_W_Q4 ? (void *)w->sz_t : (void *)w->scales_t,
                         CU_TENSOR_MAP_DATA_TYPE_UINT32, 4, N, K / grp, 128, (uint32_t)sgrp,
                         CU_TENSOR_MAP_SWIZZLE_NONE);
            if (s) return s;
        }
        if (w->fmt == LX2V_W_FP8) {
            s = make_map(ctx, &p.tmap_f, w->flags, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, N,
                         (size_t)fp8_flag_cols((int)K), 128, 2, CU_TENSOR_MAP_SWIZZLE_NONE);
            if (s) return s;
        }
        p.y = y->ptr;
        p.codes = (const uint8_t *)w->codes;
        p.scales_t = w->scales_t;
        p.sz_t = w->sz_t;
        p.bias = bias ? bias->ptr : nullptr;
        p.bias_f32 = bias && bias->dtype == LX2V_F32;
        p.gate = gate_ptr;
        p.gate_f32 = mods && mods->dtype == LX2V_F32;
        p.err = ctx->err_dev;
        p.wait_limit_ns = ctx->wait_limit_ns;
        p.M = (int)rows; p.N = (int)N; p.K = (int)K; p.group = (int)w->group;
        p.x_row = (int)x_row; p.y_row = (int)y_row;
        p.act = act;
        p.out_f32 = y->dtype == LX2V_F32;
        p.reduce = mods ? 1 : 0;
        p.kgroup = K % 128 == 0 ? 2 : 1;
        if (pair && use_streamk(ctx, (int)rows, (int)N, (int)K, bt)) {
            const int pairs = ctx->num_sms / 2;
            s = ensure_sk_workspace(ctx, pairs, bt, &p.partials, &p.flags);
            if (s) return s;
            p.streamk = 1;
            if (++ctx->sk_epoch <= 0) ctx->sk_epoch = 1;
            p.epoch = ctx->sk_epoch;
        }
        if (pair) CUDA_TRY(ctx, gemm_pair_launch(w->fmt, bt, p, ctx->num_sms, ctx->stream));
        else CUDA_TRY(ctx, gemm_dq_launch(w->fmt, bt, p, ctx->num_sms, ctx->stream));
        ctx->launches++;
        return LX2V_OK;
    }
    CUDA_TRY(ctx, linear_simt_launch(a, ctx->stream));
    ctx->launches++;
    return LX2V_OK;
}

// linear_queue, then the buffers it touched are marked used (for host -> device
// copies queued later).
static lx2v_status linear_impl(lx2v_ctx *ctx, const char *opname, const lx2v_buf *x, size_t x_row,
                               size_t rows, const lx2v_weight *w, const lx2v_buf *bias, int act, lx2v_buf *y,
                               size_t y_row, const lx2v_buf *mods, size_t gate) {
    lx2v_status s = linear_queue(ctx, opname, x, x_row, rows, w, bias, act, y, y_row, mods, gate);
    if (s) return s;
    CUDA_TRY(ctx, note_uses(ctx, {x, bias, y, mods}));
    return LX2V_OK;
}

extern "C" lx2v_status lx2v_linear(lx2v_ctx *ctx, const lx2v_buf *x, size_t x_row, size_t rows,
                                   const lx2v_weight *w, const lx2v_buf *bias, int act, lx2v_buf *y,
                                   size_t y_row) {
    lx2v_status s = enter(ctx);
    if (s) return s;
    return linear_impl(ctx, "linear", x, x_row, rows, w, bias, act, y, y_row, nullptr, 0);
}

extern "C" lx2v_status lx2v_linear_gate_residual(lx2v_ctx *ctx, const lx2v_buf *x, size_t x_row, size_t rows,
                                                 const lx2v_weight *w, const lx2v_buf *bias, int act,
                                                 lx2v_buf *h, size_t h_row, const lx2v_buf *mods, size_t gate) {
    lx2v_status s = enter(ctx);
    if (s) return s;
    if (!mods) return fail(ctx, LX2V_ERR_INVALID, "null mods");
    return linear_impl(ctx, "linear_gate_residual", x, x_row, rows, w, bias, act, h, h_row, mods, gate);
}

extern "C" lx2v_status lx2v_gate_residual(lx2v_ctx *ctx, lx2v_buf *h, const lx2v_buf *a, size_t rows, size_t dim,
                                          const lx2v_buf *mods, size_t gate) {
    lx2v_status s = enter(ctx);
    if (s) return s;
    if (!h || !a || !mods) return fail(ctx, LX2V_ERR_INVALID, "null buffer");
    if (rows * dim > h->len || rows * dim > a->len || (gate + 1) * dim > mods->len)
        return fail(ctx, LX2V_ERR_INVALID, "gate_residual range out of bounds");
    if (rows * dim == 0) return LX2V_OK;
    OpScope ps(ctx, "gate_residual");
    const void *g = (const char *)mods->ptr + gate * dim * esize(mods->dtype);
    CUDA_TRY(ctx, gate_residual_launch(h->ptr, h->dtype == LX2V_F32, a->ptr, a->dtype == LX2V_F32, g,
                                       mods->dtype == LX2V_F32, rows, dim, ctx->stream));
    ctx->launches++;
    CUDA_TRY(ctx, note_uses(ctx, {h, a, mods}));
    return LX2V_OK;
}

// ---- attention (backend.rs:275-307) ------------------------------------------------------
// Grow-only workspace of the attention calls (the mask data).
static lx2v_status ensure_att_workspace(lx2v_ctx *ctx, size_t bytes) {
    if (ctx->att_ws_bytes >= bytes) return LX2V_OK;
    if (ctx->att_ws) {
        CUDA_TRY(ctx, cudaStreamSynchronize(ctx->stream));
        cudaFree(ctx->att_ws);
        ctx->att_ws = nullptr;
        ctx->att_ws_bytes = 0;
    }
    CUDA_TRY(ctx, cudaMalloc(&ctx->att_ws, bytes));
    ctx->att_ws_bytes = bytes;
    return LX2V_OK;
}

static size_t align_up(size_t v, size_t a) { return (v + a - 1) / a * a; }

// Page-locked staging for the mask data of an attention call: the copy from
// it runs asynchronously, and the next call waits for that copy (an event)
// before it writes the staging again.
static lx2v_status att_host_staging(lx2v_ctx *ctx, size_t bytes, void **out) {
    if (!ctx->att_host_ev) CUDA_TRY(ctx, cudaEventCreateWithFlags(&ctx->att_host_ev, cudaEventDisableTiming));
    CUDA_TRY(ctx, cudaEventSynchronize(ctx->att_host_ev));
    if (ctx->att_host_bytes < bytes) {
        if (ctx->att_host) cudaFreeHost(ctx->att_host);
        ctx->att_host = nullptr;
        ctx->att_host_bytes = 0;
        CUDA_TRY(ctx, cudaMallocHost(&ctx->att_host, bytes));
        ctx->att_host_bytes = bytes;
    }
    *out = ctx->att_host;
    return LX2V_OK;
}

// Everything the attention launch needs besides q / k / v / out: which mask,
// and its host data (a row-major bool mask, or the temporal indices).
struct AttnMaskArgs {
    int mode = ATT_MASK_NONE;
    const uint8_t *mask = nullptr;  // [sq][sk] bool, nonzero = allowed
    const int32_t *tq = nullptr;    // [sq]
    const int32_t *tk = nullptr;    // [sk]
    // ATT_MASK_BITS already on the device: [heads][sq][ceil(sk/32)] words
    // (sparse attention's per-head selection), instead of the host bool mask
    const uint32_t *dev_bits = nullptr;
};

// q [heads][q_rows][d] (the first sq rows of each head are the queries),
// k / v [heads][k_rows][d] (the first sk rows are the keys), out [sq][heads*d].
static lx2v_status attention_queue(lx2v_ctx *ctx, const char *opname, const void *q, int q_f32, size_t q_rows,
                                   const void *k, const void *v, int kv_f32, size_t k_rows, size_t heads, size_t sq,
                                   size_t sk, size_t d, const AttnMaskArgs &m, lx2v_buf *out) {
    if (heads == 0 || sq == 0) return LX2V_OK;
    if (sk == 0) return fail(ctx, LX2V_ERR_INVALID, "attention over zero keys");
    if (heads * d > (1u << 20) || sq > (1u << 24) || sk > (1u << 24))
        return fail(ctx, LX2V_ERR_UNSUPPORTED, "attention shape too large");
    OpScope ps(ctx, opname);
    const bool tc = d == 128 && !q_f32 && !kv_f32;
    const size_t sk_pad = align_up(sk, 128);
    const size_t n_qt = (sq + 127) / 128, n_kb = sk_pad / 128;
    // workspace: [mask bits sq*words u32 | tq, tk, tq ranges, tk ranges]
    const size_t words = (sk + 31) / 32;
    size_t mask_bytes = 0;
    if (m.mode == ATT_MASK_BITS && !m.dev_bits) mask_bytes = sq * words * 4;
    else if (m.mode == ATT_MASK_TEMPORAL) mask_bytes = (sq + sk) * 4 + (n_qt + n_kb) * 8 + n_qt * 4;
    lx2v_status s = ensure_att_workspace(ctx, align_up(mask_bytes, 256) + 256);
    if (s) return s;
    char *mws = (char *)ctx->att_ws;
    const uint32_t *bits_dev = nullptr;
    const int *tq_dev = nullptr, *tk_dev = nullptr;
    const int2 *tqr_dev = nullptr, *tkr_dev = nullptr;
    const int *order_dev = nullptr;
    if (m.mode == ATT_MASK_BITS && m.dev_bits) {
        bits_dev = m.dev_bits;
    } else if (m.mode == ATT_MASK_BITS) {
        void *stage = nullptr;
        if ((s = att_host_staging(ctx, mask_bytes, &stage))) return s;
        uint32_t *bits = (uint32_t *)stage;
        memset(bits, 0, mask_bytes);
        for (size_t i = 0; i < sq; ++i)
            for (size_t j = 0; j < sk; ++j)
                if (m.mask[i * sk + j]) bits[i * words + j / 32] |= 1u << (j % 32);
        CUDA_TRY(ctx, cudaMemcpyAsync(mws, bits, mask_bytes, cudaMemcpyHostToDevice, ctx->stream));
        CUDA_TRY(ctx, cudaEventRecord(ctx->att_host_ev, ctx->stream));
        bits_dev = (const uint32_t *)mws;
    } else if (m.mode == ATT_MASK_TEMPORAL) {
        void *stage = nullptr;
        if ((s = att_host_staging(ctx, mask_bytes, &stage))) return s;
        // [tq ranges int2 x n_qt][tk ranges int2 x n_kb][tq x sq][tk x sk]: the
        // int2 arrays first, so that they start on 8-byte boundaries
        int32_t *host = (int32_t *)stage;
        int32_t *tqr = host, *tkr = tqr + 2 * n_qt;
        memcpy(tkr + 2 * n_kb, m.tq, sq * 4);
        memcpy(tkr + 2 * n_kb + sq, m.tk, sk * 4);
        int32_t *order = tkr + 2 * n_kb + sq + sk;
        for (size_t t = 0; t < n_qt; ++t) {
            int32_t lo = INT32_MAX, hi = INT32_MIN;
            for (size_t i = t * 128; i < sq && i < (t + 1) * 128; ++i) {
                lo = std::min(lo, m.tq[i]);
                hi = std::max(hi, m.tq[i]);
            }
            tqr[2 * t] = lo;
            tqr[2 * t + 1] = hi;
        }
        for (size_t b = 0; b < n_kb; ++b) {
            int32_t lo = INT32_MAX, hi = INT32_MIN;
            for (size_t i = b * 128; i < sk && i < (b + 1) * 128; ++i) {
                lo = std::min(lo, m.tk[i]);
                hi = std::max(hi, m.tk[i]);
            }
            tkr[2 * b] = lo;
            tkr[2 * b + 1] = hi;
        }
        // query tiles by the number of key blocks they attend to, most first
        std::vector<std::pair<int, int>> work(n_qt);
        for (size_t t = 0; t < n_qt; ++t) {
            int live = 0;
            for (size_t b = 0; b < n_kb; ++b) live += tkr[2 * b] <= tqr[2 * t + 1];
            work[t] = {-live, (int)t};
        }
        std::stable_sort(work.begin(), work.end());
        for (size_t t = 0; t < n_qt; ++t) order[t] = work[t].second;
        CUDA_TRY(ctx, cudaMemcpyAsync(mws, host, mask_bytes, cudaMemcpyHostToDevice, ctx->stream));
        CUDA_TRY(ctx, cudaEventRecord(ctx->att_host_ev, ctx->stream));
        tqr_dev = (const int2 *)mws;
        tkr_dev = tqr_dev + n_qt;
        tq_dev = (const int *)(tkr_dev + n_kb);
        tk_dev = tq_dev + sq;
        order_dev = tk_dev + sk;
    }
    if (tc) {
        AttnParams p;
        memset(&p, 0, sizeof p);
        if ((s = make_map(ctx, &p.tmap_q, q, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, 128, heads * q_rows, 64, 128,
                          CU_TENSOR_MAP_SWIZZLE_128B)))
            return s;
        if ((s = make_map(ctx, &p.tmap_k, k, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, 128, heads * k_rows, 64, 128,
                          CU_TENSOR_MAP_SWIZZLE_128B)))
            return s;
        // V as stored, [heads][k_rows][128], seen as {128, sk, heads}: the
        // keys of a head past sk are outside the map and load as zeros (their
        // P is 0, and 0 times whatever the cache holds there must stay 0)
        {
            cuuint64_t dims[3] = {128, sk, heads};
            cuuint64_t strides[2] = {128 * 2, (cuuint64_t)k_rows * 128 * 2};
            cuuint32_t box[3] = {64, 128, 1};
            cuuint32_t estr[3] = {1, 1, 1};
            CUresult r = ctx->encode(&p.tmap_v, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void *>(v), dims,
                                     strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                                     CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
            if (r != CUDA_SUCCESS)
                return fail(ctx, LX2V_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d) for V %zux%zux%zu", (int)r,
                            (size_t)128, sk, heads);
        }
        p.out = out->ptr;
        p.out_f32 = out->dtype == LX2V_F32;
        p.heads = (int)heads; p.sq = (int)sq; p.sk = (int)sk;
        p.q_rows = (int)q_rows; p.k_rows = (int)k_rows;
        p.scale_log2 = 1.4426950408889634f / sqrtf(128.0f);
        p.mask_mode = m.mode;
        p.mask_bits = bits_dev; p.mask_words = (int)words;
        p.mask_head_stride = m.dev_bits ? (int64_t)(sq * words) : 0;
        p.tq = tq_dev; p.tk = tk_dev; p.tq_range = tqr_dev; p.tk_range = tkr_dev;
        p.tile_order = order_dev;
        p.err = ctx->err_dev;
        p.wait_limit_ns = ctx->wait_limit_ns;
        CUDA_TRY(ctx, attention_tc_launch(p, ctx->stream));
        ctx->launches++;
        return LX2V_OK;
    }
    if (d > 256) return fail(ctx, LX2V_ERR_UNSUPPORTED, "attention head_dim %zu > 256", d);
    if ((sk + 32) * 4 > 200 * 1024)
        return fail(ctx, LX2V_ERR_UNSUPPORTED, "attention with head_dim != 128 or f32 operands takes at most %d keys",
                    200 * 1024 / 4 - 32);
    AttnSimtParams p;
    memset(&p, 0, sizeof p);
    p.q = q; p.k = k; p.v = v;
    if (q_f32 != kv_f32) return fail(ctx, LX2V_ERR_UNSUPPORTED, "q and k/v must have the same element type");
    p.qkv_f32 = q_f32;
    p.out = out->ptr; p.out_f32 = out->dtype == LX2V_F32;
    p.heads = (int)heads; p.sq = (int)sq; p.sk = (int)sk; p.d = (int)d;
    p.q_rows = (int)q_rows; p.k_rows = (int)k_rows;
    p.mask_mode = m.mode; p.mask_bits = bits_dev; p.mask_words = (int)words;
    p.mask_head_stride = m.dev_bits ? (int64_t)(sq * words) : 0;
    p.tq = tq_dev; p.tk = tk_dev;
    CUDA_TRY(ctx, attention_simt_launch(p, ctx->stream));
    ctx->launches++;
    return LX2V_OK;
}

static lx2v_status attention_buffers(lx2v_ctx *ctx, const char *opname, const lx2v_buf *q, const lx2v_buf *k,
                                     const lx2v_buf *v, size_t heads, size_t sq, size_t sk, size_t d,
                                     const AttnMaskArgs &m, lx2v_buf *out) {
    if (!q || !k || !v || !out) return fail(ctx, LX2V_ERR_INVALID, "null q, k, v or output");
    if (out == q || out == k || out == v) return fail(ctx, LX2V_ERR_INVALID, "output aliases an input");
    if (k->dtype != v->dtype) return fail(ctx, LX2V_ERR_INVALID, "k and v must have the same element type");
    if (heads * sq * d > q->len || heads * sk * d > k->len || heads * sk * d > v->len)
        return fail(ctx, LX2V_ERR_INVALID, "q/k/v hold fewer than heads x rows x head_dim elements");
    if (sq * heads * d > out->len) return fail(ctx, LX2V_ERR_INVALID, "output holds fewer than sq x heads x head_dim");
    if (d == 0) return fail(ctx, LX2V_ERR_INVALID, "head_dim 0");
    lx2v_status s = attention_queue(ctx, opname, q->ptr, q->dtype == LX2V_F32, sq, k->ptr, v->ptr,
                                    k->dtype == LX2V_F32, sk, heads, sq, sk, d, m, out);
    if (s) return s;
    CUDA_TRY(ctx, note_uses(ctx, {q, k, v, out}));
    return LX2V_OK;
}

extern "C" lx2v_status lx2v_attention(lx2v_ctx *ctx, const lx2v_buf *q, const lx2v_buf *k, const lx2v_buf *v,
                                      size_t heads, size_t sq, size_t sk, size_t head_dim, lx2v_buf *out) {
    lx2v_status s = enter(ctx);
    if (s) return s;
    return attention_buffers(ctx, "attention", q, k, v, heads, sq, sk, head_dim, AttnMaskArgs(), out);
}

extern "C" lx2v_status lx2v_causal_attention(lx2v_ctx *ctx, const lx2v_buf *q, const lx2v_buf *k,
                                             const lx2v_buf *v, size_t heads, size_t sq, size_t sk,
                                             size_t head_dim, const uint8_t *mask, lx2v_buf *out) {
    lx2v_status s = enter(ctx);
    if (s) return s;
    AttnMaskArgs m;
    if (mask) {
        m.mode = ATT_MASK_BITS;
        m.mask = mask;
    }
    return attention_buffers(ctx, "causal_attention", q, k, v, heads, sq, sk, head_dim, m, out);
}

extern "C" lx2v_status lx2v_causal_attention_temporal(lx2v_ctx *ctx, const lx2v_buf *q, const lx2v_buf *k,
                                                      const lx2v_buf *v, size_t heads, size_t sq, size_t sk,
                                                      size_t head_dim, const int32_t *tq, const int32_t *tk,
                                                      lx2v_buf *out) {
    lx2v_status s = enter(ctx);
    if (s) return s;
    if (!tq || !tk) return fail(ctx, LX2V_ERR_INVALID, "null temporal indices");
    AttnMaskArgs m;
    m.mode = ATT_MASK_TEMPORAL;
    m.tq = tq;
    m.tk = tk;
    return attention_buffers(ctx, "causal_attention", q, k, v, heads, sq, sk, head_dim, m, out);
}

// ---- KV cache / MemRoPE (backend.rs:334-390) ------------------------------------------------
// The CPU reference (crates/lightx2v-cpu/src/lib.rs:607-806) keeps K and V as
// [rows][heads][head_dim] f32 vectors and splices them. Here the rows live on
// the device as [heads][capacity][head_dim] bf16 (the CUDA backend's
// activation precision), so each head's keys are one matrix the attention
// kernel reads directly; the slot bookkeeping (temporal index and kind per
// row) stays on the host and follows the reference step for step.
enum : uint8_t { SLOT_SINK = 0, SLOT_LONG_EMA = 1, SLOT_SHORT_EMA = 2, SLOT_RECENT = 3, SLOT_NEW = 4 };

struct lx2v_kv_cache {
    size_t heads = 0, head_dim = 0;
    size_t cap = 0;   // rows per head the device arrays hold
    size_t rows = 0;  // rows in use
    __nv_bfloat16 *k = nullptr, *v = nullptr;
    std::vector<size_t> temporal;
    std::vector<uint8_t> kinds;
};

static lx2v_status kv_reserve(lx2v_ctx *ctx, lx2v_kv_cache *c, size_t need) {
    if (need <= c->cap) return LX2V_OK;
    size_t cap = c->cap + c->cap / 2;
    if (cap < need) cap = need;
    cap = align_up(cap, 128);
    const size_t bytes = c->heads * cap * c->head_dim * 2;
    __nv_bfloat16 *nk = nullptr, *nv = nullptr;
    cudaError_t e = cudaMalloc(&nk, bytes);
    if (e == cudaSuccess) e = cudaMalloc(&nv, bytes);
    if (e == cudaSuccess) e = cudaMemsetAsync(nk, 0, bytes, ctx->stream);
    if (e == cudaSuccess) e = cudaMemsetAsync(nv, 0, bytes, ctx->stream);
    if (e == cudaSuccess && c->rows) {
        e = kv_copy_rows_launch(c->k, 0, (int64_t)c->cap, 0, nk, 0, (int64_t)cap, 0, (int64_t)c->rows,
                                (int)c->head_dim, (int)c->heads, ctx->stream);
        if (e == cudaSuccess)
            e = kv_copy_rows_launch(c->v, 0, (int64_t)c->cap, 0, nv, 0, (int64_t)cap, 0, (int64_t)c->rows,
                                    (int)c->head_dim, (int)c->heads, ctx->stream);
        ctx->launches += 2;
    }
    if (e == cudaSuccess) e = cudaStreamSynchronize(ctx->stream);
    if (e != cudaSuccess) {
        if (nk) cudaFree(nk);
        if (nv) cudaFree(nv);
        return fail(ctx, e == cudaErrorMemoryAllocation ? LX2V_ERR_OOM : LX2V_ERR_CUDA, "KV cache growth: %s",
                    cudaGetErrorString(e));
    }
    if (c->k) cudaFree(c->k);
    if (c->v) cudaFree(c->v);
    c->k = nk;
    c->v = nv;
    c->cap = cap;
    return LX2V_OK;
}

// rows [src, src + n) -> [dst, dst + n) of K and V, overlapping ranges
// allowed (through a staging buffer).
static lx2v_status kv_move(lx2v_ctx *ctx, lx2v_kv_cache *c, size_t src, size_t dst, size_t n) {
    if (n == 0 || src == dst) return LX2V_OK;
    const size_t bytes = c->heads * n * c->head_dim * 2;
    if (ctx->kv_tmp_bytes < bytes) {
        if (ctx->kv_tmp) {
            CUDA_TRY(ctx, cudaStreamSynchronize(ctx->stream));
            cudaFree(ctx->kv_tmp);
            ctx->kv_tmp = nullptr;
            ctx->kv_tmp_bytes = 0;
        }
        CUDA_TRY(ctx, cudaMalloc(&ctx->kv_tmp, bytes));
        ctx->kv_tmp_bytes = bytes;
    }
    for (__nv_bfloat16 *a : {c->k, c->v}) {
        CUDA_TRY(ctx, kv_copy_rows_launch(a, 0, (int64_t)c->cap, (int64_t)src, ctx->kv_tmp, 0, (int64_t)n, 0,
                                          (int64_t)n, (int)c->head_dim, (int)c->heads, ctx->stream));
        CUDA_TRY(ctx, kv_copy_rows_launch(ctx->kv_tmp, 0, (int64_t)n, 0, a, 0, (int64_t)c->cap, (int64_t)dst,
                                          (int64_t)n, (int)c->head_dim, (int)c->heads, ctx->stream));
        ctx->launches += 2;
    }
    return LX2V_OK;
}

static lx2v_status kv_write_rows(lx2v_ctx *ctx, lx2v_kv_cache *c, const lx2v_buf *k, const lx2v_buf *v,
                                 size_t rows, size_t at) {
    CUDA_TRY(ctx, kv_copy_rows_launch(k->ptr, k->dtype == LX2V_F32, (int64_t)rows, 0, c->k, 0, (int64_t)c->cap,
                                      (int64_t)at, (int64_t)rows, (int)c->head_dim, (int)c->heads, ctx->stream));
    CUDA_TRY(ctx, kv_copy_rows_launch(v->ptr, v->dtype == LX2V_F32, (int64_t)rows, 0, c->v, 0, (int64_t)c->cap,
                                      (int64_t)at, (int64_t)rows, (int)c->head_dim, (int)c->heads, ctx->stream));
    ctx->launches += 2;
    CUDA_TRY(ctx, note_uses(ctx, {k, v}));
    return LX2V_OK;
}

static lx2v_status kv_check_rows(lx2v_ctx *ctx, lx2v_kv_cache *c, const lx2v_buf *k, const lx2v_buf *v, size_t rows,
                                 const size_t *temporal) {
    if (!c || !k || !v || (rows && !temporal)) return fail(ctx, LX2V_ERR_INVALID, "null cache, k, v or temporal");
    if (c->heads * rows * c->head_dim > k->len || c->heads * rows * c->head_dim > v->len)
        return fail(ctx, LX2V_ERR_INVALID, "k/v hold fewer than heads x rows x head_dim elements");
    return LX2V_OK;
}

static lx2v_status kv_append(lx2v_ctx *ctx, lx2v_kv_cache *c, const lx2v_buf *k, const lx2v_buf *v, size_t rows,
                             const size_t *temporal) {
    lx2v_status s = kv_reserve(ctx, c, c->rows + rows);
    if (s) return s;
    if ((s = kv_write_rows(ctx, c, k, v, rows, c->rows))) return s;
    for (size_t r = 0; r < rows; ++r) {
        c->temporal.push_back(temporal[r]);
        c->kinds.push_back(SLOT_NEW);  // graduated by memrope_update
    }
    c->rows += rows;
    return LX2V_OK;
}

extern "C" lx2v_status lx2v_kv_cache_new(lx2v_ctx *ctx, size_t heads, size_t head_dim, size_t capacity_tokens,
                                         lx2v_kv_cache **out) {
    lx2v_status s = enter(ctx);
    if (s) return s;
    if (!out || heads == 0 || head_dim == 0) return fail(ctx, LX2V_ERR_INVALID, "bad KV cache shape");
    auto *c = new lx2v_kv_cache();
    c->heads = heads;
    c->head_dim = head_dim;
    if ((s = kv_reserve(ctx, c, capacity_tokens ? capacity_tokens : 128))) {
        delete c;
        return s;
    }
    *out = c;
    return LX2V_OK;
}

extern "C" void lx2v_kv_cache_free(lx2v_ctx *ctx, lx2v_kv_cache *c) {
    if (!c) return;
    if (ctx) {
        cudaSetDevice(ctx->dev);
        cudaStreamSynchronize(ctx->stream);
    }
    if (c->k) cudaFree(c->k);
    if (c->v) cudaFree(c->v);
    delete c;
}

extern "C" lx2v_status lx2v_kv_cache_append(lx2v_ctx *ctx, lx2v_kv_cache *c, const lx2v_buf *k, const lx2v_buf *v,
                                            size_t rows, const size_t *temporal) {
    lx2v_status s = enter(ctx);
    if (s) return s;
    if ((s = kv_check_rows(ctx, c, k, v, rows, temporal))) return s;
    OpScope ps(ctx, "kv_cache_append");
    return kv_append(ctx, c, k, v, rows, temporal);
}

extern "C" lx2v_status lx2v_kv_cache_put(lx2v_ctx *ctx, lx2v_kv_cache *c, const lx2v_buf *k, const lx2v_buf *v,
                                         size_t rows, const size_t *temporal) {
    lx2v_status s = enter(ctx);
    if (s) return s;
    if ((s = kv_check_rows(ctx, c, k, v, rows, temporal))) return s;
    if (rows == 0) return LX2V_OK;
    OpScope ps(ctx, "kv_cache_put");
    // the same temporal run already cached (not in an EMA slot, which shares
    // the first non-sink frame's index): overwrite those rows in place
    for (size_t pos = 0; pos < c->rows; ++pos) {
        if (c->temporal[pos] != temporal[0] || c->kinds[pos] == SLOT_LONG_EMA || c->kinds[pos] == SLOT_SHORT_EMA)
            continue;
        bool match = pos + rows <= c->rows;
        for (size_t i = 0; match && i < rows; ++i) match = c->temporal[pos + i] == temporal[i];
        if (match) return kv_write_rows(ctx, c, k, v, rows, pos);
        break;  // the first candidate decides, as the reference's position() does
    }
    return kv_append(ctx, c, k, v, rows, temporal);
}

extern "C" lx2v_status lx2v_kv_cache_len(lx2v_ctx *ctx, const lx2v_kv_cache *c, size_t *rows) {
    if (!ctx) return fail(nullptr, LX2V_ERR_INVALID, "null context");
    if (!c || !rows) return fail(ctx, LX2V_ERR_INVALID, "null cache or output");
    *rows = c->rows;
    return LX2V_OK;
}

extern "C" lx2v_status lx2v_kv_cache_temporal(lx2v_ctx *ctx, const lx2v_kv_cache *c, size_t *out, size_t cap) {
    if (!ctx) return fail(nullptr, LX2V_ERR_INVALID, "null context");
    if (!c || (c->rows && !out)) return fail(ctx, LX2V_ERR_INVALID, "null cache or output");
    if (cap < c->rows) return fail(ctx, LX2V_ERR_INVALID, "output holds %zu of %zu rows", cap, c->rows);
    if (c->rows) memcpy(out, c->temporal.data(), c->rows * sizeof(size_t));
    return LX2V_OK;
}

extern "C" lx2v_status lx2v_kv_cache_kv(lx2v_ctx *ctx, const lx2v_kv_cache *c, lx2v_buf *k_out, lx2v_buf *v_out) {
    lx2v_status s = enter(ctx);
    if (s) return s;
    if (!c || !k_out || !v_out) return fail(ctx, LX2V_ERR_INVALID, "null cache or output");
    const size_t n = c->heads * c->rows * c->head_dim;
    if (k_out->len < n || v_out->len < n) return fail(ctx, LX2V_ERR_INVALID, "outputs hold fewer than %zu elements", n);
    OpScope ps(ctx, "kv_cache_kv");
    CUDA_TRY(ctx, kv_copy_rows_launch(c->k, 0, (int64_t)c->cap, 0, k_out->ptr, k_out->dtype == LX2V_F32,
                                      (int64_t)c->rows, 0, (int64_t)c->rows, (int)c->head_dim, (int)c->heads,
                                      ctx->stream));
    CUDA_TRY(ctx, kv_copy_rows_launch(c->v, 0, (int64_t)c->cap, 0, v_out->ptr, v_out->dtype == LX2V_F32,
                                      (int64_t)c->rows, 0, (int64_t)c->rows, (int)c->head_dim, (int)c->heads,
                                      ctx->stream));
    ctx->launches += 2;
    CUDA_TRY(ctx, note_uses(ctx, {k_out, v_out}));
    return LX2V_OK;
}

// crates/lightx2v-cpu/src/lib.rs:688-806, step for step.
extern "C" lx2v_status lx2v_kv_cache_memrope_update(lx2v_ctx *ctx, lx2v_kv_cache *c, size_t cache_frames,
                                                    size_t sink_frames, size_t new_frames, float ema_alpha_long,
                                                    float ema_alpha_short, size_t frame_tokens) {
    lx2v_status s = enter(ctx);
    if (s) return s;
    if (!c || frame_tokens == 0) return fail(ctx, LX2V_ERR_INVALID, "null cache or zero frame_tokens");
    OpScope ps(ctx, "kv_cache_memrope_update");
    const size_t ft = frame_tokens;
    auto n_frames = [&] { return c->rows / ft; };
    auto frame_kinds = [&] {
        std::vector<uint8_t> fk(n_frames());
        for (size_t f = 0; f < fk.size(); ++f) fk[f] = c->kinds[f * ft];
        return fk;
    };
    if (n_frames() == 0) return LX2V_OK;
    std::vector<uint8_t> fk = frame_kinds();
    const bool has_long = std::find(fk.begin(), fk.end(), SLOT_LONG_EMA) != fk.end();
    if (!has_long && fk.size() > sink_frames) {
        // seed the EMA slots with zero frames after the sinks: Short, then Long
        // inserted at the same row, so the order becomes [sink, long, short]
        const size_t at = sink_frames * ft;
        const size_t t = c->temporal[std::min(at, c->rows - 1)];
        for (uint8_t kind : {SLOT_SHORT_EMA, SLOT_LONG_EMA}) {
            if ((s = kv_reserve(ctx, c, c->rows + ft))) return s;
            if (at < c->rows && (s = kv_move(ctx, c, at, at + ft, c->rows - at))) return s;
            for (__nv_bfloat16 *a : {c->k, c->v})
                CUDA_TRY(ctx, cudaMemset2DAsync(a + at * c->head_dim, c->cap * c->head_dim * 2, 0,
                                                ft * c->head_dim * 2, c->heads, ctx->stream));
            c->temporal.insert(c->temporal.begin() + at, ft, t);
            c->kinds.insert(c->kinds.begin() + at, ft, kind);
            c->rows += ft;
            fk = frame_kinds();
        }
    }
    // graduate New frames beyond the newest `new_frames` to Recent
    std::vector<size_t> news;
    for (size_t f = 0; f < fk.size(); ++f)
        if (fk[f] == SLOT_NEW) news.push_back(f);
    if (news.size() > new_frames) {
        const size_t excess = news.size() - new_frames;
        for (size_t i = 0; i < excess; ++i)
            std::fill(c->kinds.begin() + news[i] * ft, c->kinds.begin() + (news[i] + 1) * ft, SLOT_RECENT);
    }
    // evict while over capacity: fold the oldest Recent (else New) frame into
    // the EMA slots, then drop it
    while (n_frames() > cache_frames) {
        const std::vector<uint8_t> kn = frame_kinds();
        auto first = [&](uint8_t kind) -> long {
            for (size_t f = 0; f < kn.size(); ++f)
                if (kn[f] == kind) return (long)f;
            return -1;
        };
        long f = first(SLOT_RECENT);
        if (f < 0) f = first(SLOT_NEW);
        if (f < 0) break;
        const std::pair<uint8_t, float> slots[2] = {{SLOT_LONG_EMA, ema_alpha_long}, {SLOT_SHORT_EMA, ema_alpha_short}};
        for (const auto &sl : slots) {
            const long sf = first(sl.first);
            if (sf < 0) continue;
            for (__nv_bfloat16 *a : {c->k, c->v})
                CUDA_TRY(ctx, kv_ema_launch(a, (int64_t)c->cap, (int64_t)sf * (int64_t)ft, (int64_t)f * (int64_t)ft,
                                            (int64_t)ft, (int)c->head_dim, (int)c->heads, sl.second, ctx->stream));
            ctx->launches += 2;
        }
        const size_t base = (size_t)f * ft;
        if ((s = kv_move(ctx, c, base + ft, base, c->rows - base - ft))) return s;
        c->temporal.erase(c->temporal.begin() + base, c->temporal.begin() + base + ft);
        c->kinds.erase(c->kinds.begin() + base, c->kinds.begin() + base + ft);
        c->rows -= ft;
    }
    // the first sink_frames frames are sinks (they were appended as New)
    for (size_t f = 0; f < std::min(sink_frames, n_frames()); ++f)
        std::fill(c->kinds.begin() + f * ft, c->kinds.begin() + (f + 1) * ft, SLOT_SINK);
    return LX2V_OK;
}

extern "C" lx2v_status lx2v_kv_cache_attention(lx2v_ctx *ctx, const lx2v_buf *q, size_t sq, const int32_t *tq,
                                               const lx2v_kv_cache *c, lx2v_buf *out) {
    lx2v_status s = enter(ctx);
    if (s) return s;
    if (!q || !c || !out || (sq && !tq)) return fail(ctx, LX2V_ERR_INVALID, "null q, cache, output or tq");
    const size_t heads = c->heads, d = c->head_dim;
    if (heads * sq * d > q->len) return fail(ctx, LX2V_ERR_INVALID, "q holds fewer than heads x sq x head_dim");
    if (sq * heads * d > out->len) return fail(ctx, LX2V_ERR_INVALID, "output holds fewer than sq x heads x head_dim");
    if (out == q) return fail(ctx, LX2V_ERR_INVALID, "output aliases q");
    std::vector<int32_t> tk(c->rows);
    for (size_t i = 0; i < c->rows; ++i) {
        if (c->temporal[i] > (size_t)INT32_MAX) return fail(ctx, LX2V_ERR_UNSUPPORTED, "temporal index beyond int32");
        tk[i] = (int32_t)c->temporal[i];
    }
    AttnMaskArgs m;
    m.mode = ATT_MASK_TEMPORAL;
    m.tq = tq;
    m.tk = tk.data();
    s = attention_queue(ctx, "kv_cache_attention", q->ptr, q->dtype == LX2V_F32, sq, c->k, c->v, 0, c->cap, heads,
                        sq, c->rows, d, m, out);
    if (s) return s;
    CUDA_TRY(ctx, note_uses(ctx, {q, out}));
    return LX2V_OK;
}

// ---- norms, head_split, patchify, dmd_step (backend.rs:214-273, 392-428) --------------------
static int is_f32(const lx2v_buf *b) { return b && b->dtype == LX2V_F32 ? 1 : 0; }

// NormKind: kind 0 = Affine { w, b } (length dim each), 1 = Mod { scale, shift }
// (rows of the mods table).
static lx2v_status norm_args(lx2v_ctx *ctx, NormArgs &a, size_t rows, size_t dim, int kind, const lx2v_buf *w,
                             const lx2v_buf *b, size_t scale, size_t shift, const lx2v_buf *mods, float eps,
                             lx2v_buf *out) {
    if (!out || (kind != 0 && kind != 1)) return fail(ctx, LX2V_ERR_INVALID, "null output or bad norm kind %d", kind);
    if (!row_op_supported((int)dim)) return fail(ctx, LX2V_ERR_UNSUPPORTED, "norm rows of %zu values (max 4096)", dim);
    if (rows * dim > out->len) return fail(ctx, LX2V_ERR_INVALID, "norm output holds fewer than rows x dim");
    if (kind == 0 && (!w || !b || w->len < dim || b->len < dim))
        return fail(ctx, LX2V_ERR_INVALID, "affine norm needs w and b of dim elements");
    if (kind == 1 && (!mods || mods->len < (std::max(scale, shift) + 1) * dim))
        return fail(ctx, LX2V_ERR_INVALID, "modulated norm: mods has too few rows");
    memset(&a, 0, sizeof a);
    a.out = out->ptr; a.out_f32 = is_f32(out);
    a.rows = (int64_t)rows; a.dim = (int)dim; a.kind = kind;
    a.w = w ? w->ptr : nullptr; a.w_f32 = is_f32(w);
    a.b = b ? b->ptr : nullptr; a.b_f32 = is_f32(b);
    a.mods = mods ? mods->ptr : nullptr; a.mods_f32 = is_f32(mods);
    a.scale = (int)scale; a.shift = (int)shift; a.eps = eps;
    return LX2V_OK;
}

extern "C" lx2v_status lx2v_layer_norm(lx2v_ctx *ctx, const lx2v_buf *x, size_t rows, size_t dim, int kind,
                                       const lx2v_buf *w, const lx2v_buf *b, size_t scale, size_t shift,
                                       const lx2v_buf *mods, float eps, lx2v_buf *out) {
    lx2v_status s = enter(ctx);
    if (s) return s;
    if (!x || rows * dim > x->len) return fail(ctx, LX2V_ERR_INVALID, "x holds fewer than rows x dim");
    if (x == out) return fail(ctx, LX2V_ERR_INVALID, "output aliases x");
    NormArgs a;
    if ((s = norm_args(ctx, a, rows, dim, kind, w, b, scale, shift, mods, eps, out))) return s;
    if (rows == 0) return LX2V_OK;
    OpScope ps(ctx, "layer_norm");
    a.x = x->ptr; a.x_f32 = is_f32(x);
    CUDA_TRY(ctx, layer_norm_launch(a, ctx->stream));
    ctx->launches++;
    CUDA_TRY(ctx, note_uses(ctx, {x, w, b, mods, out}));
    return LX2V_OK;
}

extern "C" lx2v_status lx2v_residual_norm(lx2v_ctx *ctx, lx2v_buf *h, const lx2v_buf *a_buf, size_t rows, size_t dim,
                                          const lx2v_buf *mods, long gate, int kind, const lx2v_buf *w,
                                          const lx2v_buf *b, size_t scale, size_t shift, float eps,
                                          lx2v_buf *normed) {
    lx2v_status s = enter(ctx);
    if (s) return s;
    if (!h || !a_buf || rows * dim > h->len || rows * dim > a_buf->len)
        return fail(ctx, LX2V_ERR_INVALID, "h / a hold fewer than rows x dim");
    if (normed == h || normed == a_buf) return fail(ctx, LX2V_ERR_INVALID, "normed aliases h or a");
    if (gate >= 0 && (!mods || mods->len < ((size_t)gate + 1) * dim))
        return fail(ctx, LX2V_ERR_INVALID, "gate row beyond mods");
    NormArgs a;
    if ((s = norm_args(ctx, a, rows, dim, kind, w, b, scale, shift, mods, eps, normed))) return s;
    if (rows == 0) return LX2V_OK;
    OpScope ps(ctx, "residual_norm");
    a.x = h->ptr; a.x_f32 = is_f32(h);
    CUDA_TRY(ctx, residual_norm_launch(a, h->ptr, is_f32(h), a_buf->ptr, is_f32(a_buf), gate >= 0 ? (int)gate : -1,
                                       ctx->stream));
    ctx->launches++;
    CUDA_TRY(ctx, note_uses(ctx, {h, a_buf, w, b, mods, normed}));
    return LX2V_OK;
}

static lx2v_status head_split_impl(lx2v_ctx *ctx, const lx2v_buf *src, size_t rows, size_t src_stride,
                                   size_t col_off, size_t heads, size_t head_dim, const lx2v_buf *rms_w,
                                   const lx2v_buf *sumsq, size_t rms_dim, const lx2v_buf *cos, const lx2v_buf *sin,
                                   float eps, lx2v_buf *out, size_t parts = 1);

extern "C" lx2v_status lx2v_head_split(lx2v_ctx *ctx, const lx2v_buf *src, size_t rows, size_t src_stride,
                                       size_t col_off, size_t heads, size_t head_dim, const lx2v_buf *rms_w,
                                       const lx2v_buf *cos, const lx2v_buf *sin, float eps, lx2v_buf *out) {
    return head_split_impl(ctx, src, rows, src_stride, col_off, heads, head_dim, rms_w, nullptr, 0, cos, sin, eps,
                           out);
}

extern "C" lx2v_status lx2v_head_split_rms(lx2v_ctx *ctx, const lx2v_buf *src, size_t rows, size_t src_stride,
                                           size_t col_off, size_t heads, size_t head_dim, const lx2v_buf *rms_w,
                                           const lx2v_buf *sumsq, size_t rms_dim, const lx2v_buf *cos,
                                           const lx2v_buf *sin, float eps, lx2v_buf *out) {
    if (!rms_w || !sumsq || rms_dim == 0)
        return fail(ctx, LX2V_ERR_INVALID, "head_split_rms needs the RMS weight, the row sums and their width");
    return head_split_impl(ctx, src, rows, src_stride, col_off, heads, head_dim, rms_w, sumsq, rms_dim, cos, sin, eps,
                           out);
}

extern "C" lx2v_status lx2v_head_split_rms_parts(lx2v_ctx *ctx, const lx2v_buf *src, size_t rows, size_t src_stride,
                                                 size_t col_off, size_t heads, size_t head_dim, const lx2v_buf *rms_w,
                                                 const lx2v_buf *sumsq, size_t parts, size_t rms_dim,
                                                 const lx2v_buf *cos, const lx2v_buf *sin, float eps, lx2v_buf *out) {
    if (!rms_w || !sumsq || rms_dim == 0 || parts == 0)
        return fail(ctx, LX2V_ERR_INVALID, "head_split_rms_parts needs the RMS weight, the row sums and their width");
    return head_split_impl(ctx, src, rows, src_stride, col_off, heads, head_dim, rms_w, sumsq, rms_dim, cos, sin, eps,
                           out, parts);
}

extern "C" lx2v_status lx2v_row_sumsq(lx2v_ctx *ctx, const lx2v_buf *src, size_t rows, size_t src_stride,
                                      size_t col_off, size_t width, lx2v_buf *out) {
    lx2v_status s = enter(ctx);
    if (s) return s;
    if (!src || !out || out->dtype != LX2V_F32) return fail(ctx, LX2V_ERR_INVALID, "null src or non-f32 output");
    if (col_off + width > src_stride || (rows && (rows - 1) * src_stride + col_off + width > src->len))
        return fail(ctx, LX2V_ERR_INVALID, "row_sumsq columns beyond src");
    if (rows > out->len) return fail(ctx, LX2V_ERR_INVALID, "row_sumsq output holds fewer than rows");
    if (rows == 0) return LX2V_OK;
    OpScope ps(ctx, "row_sumsq");
    CUDA_TRY(ctx, row_sumsq_launch(src->ptr, is_f32(src), (int64_t)rows, (int64_t)src_stride, (int64_t)col_off,
                                   (int)width, (float *)out->ptr, ctx->stream));
    ctx->launches++;
    CUDA_TRY(ctx, note_uses(ctx, {src, out}));
    return LX2V_OK;
}

static lx2v_status head_split_impl(lx2v_ctx *ctx, const lx2v_buf *src, size_t rows, size_t src_stride,
                                   size_t col_off, size_t heads, size_t head_dim, const lx2v_buf *rms_w,
                                   const lx2v_buf *sumsq, size_t rms_dim, const lx2v_buf *cos, const lx2v_buf *sin,
                                   float eps, lx2v_buf *out, size_t parts) {
    lx2v_status s = enter(ctx);
    if (s) return s;
    if (sumsq && (sumsq->dtype != LX2V_F32 || sumsq->len < rows * parts))
        return fail(ctx, LX2V_ERR_INVALID, "row sums of squares must be f32, one per row");
    const size_t d = heads * head_dim;
    if (!src || !out || head_dim == 0 || head_dim % 2) return fail(ctx, LX2V_ERR_INVALID, "null src/out or odd head_dim");
    if (col_off + d > src_stride || (rows && (rows - 1) * src_stride + col_off + d > src->len))
        return fail(ctx, LX2V_ERR_INVALID, "head_split columns beyond src");
    if (rows * d > out->len) return fail(ctx, LX2V_ERR_INVALID, "head_split output holds fewer than rows x heads x head_dim");
    if (rms_w && rms_w->len < d) return fail(ctx, LX2V_ERR_INVALID, "rms weight holds fewer than heads x head_dim");
    if ((cos == nullptr) != (sin == nullptr)) return fail(ctx, LX2V_ERR_INVALID, "RoPE needs both cos and sin");
    if (cos && (cos->len < rows * head_dim / 2 || sin->len < rows * head_dim / 2 || cos->dtype != sin->dtype))
        return fail(ctx, LX2V_ERR_INVALID, "cos / sin hold fewer than rows x head_dim / 2 (or differ in type)");
    if (out == src) return fail(ctx, LX2V_ERR_INVALID, "output aliases src");
    if (!row_op_supported((int)d)) return fail(ctx, LX2V_ERR_UNSUPPORTED, "head_split rows of %zu values (max 4096)", d);
    if (rows == 0) return LX2V_OK;
    OpScope ps(ctx, "head_split");
    HeadSplitArgs a;
    memset(&a, 0, sizeof a);
    a.src = src->ptr; a.src_f32 = is_f32(src);
    a.rows = (int64_t)rows; a.src_stride = (int64_t)src_stride; a.col_off = (int64_t)col_off;
    a.heads = (int)heads; a.head_dim = (int)head_dim;
    a.rms_w = rms_w ? rms_w->ptr : nullptr; a.w_f32 = is_f32(rms_w);
    a.sumsq = sumsq ? (const float *)sumsq->ptr : nullptr; a.rms_dim = (int)rms_dim;
    a.sumsq_parts = sumsq ? (int)parts : 0; a.sumsq_stride = (int64_t)rows;
    a.cos = cos ? cos->ptr : nullptr; a.sin = sin ? sin->ptr : nullptr; a.cs_f32 = is_f32(cos);
    a.eps = eps;
    a.out = out->ptr; a.out_f32 = is_f32(out);
    CUDA_TRY(ctx, head_split_launch(a, ctx->stream));
    ctx->launches++;
    CUDA_TRY(ctx, note_uses(ctx, {src, rms_w, sumsq, cos, sin, out}));
    return LX2V_OK;
}

static lx2v_status patchify_impl(lx2v_ctx *ctx, const lx2v_buf *src, size_t c, size_t t, size_t h, size_t w, size_t p,
                                 lx2v_buf *dst, int to_tokens) {
    lx2v_status s = enter(ctx);
    if (s) return s;
    if (!src || !dst || p == 0 || h % p || w % p) return fail(ctx, LX2V_ERR_INVALID, "null buffer or h, w not multiples of p");
    const size_t n = c * t * h * w;
    if (src->len < n || dst->len < n) return fail(ctx, LX2V_ERR_INVALID, "buffers hold fewer than c x t x h x w");
    if (src == dst) return fail(ctx, LX2V_ERR_INVALID, "output aliases input");
    if (n > (1ull << 31)) return fail(ctx, LX2V_ERR_UNSUPPORTED, "latent too large");
    if (n == 0) return LX2V_OK;
    OpScope ps(ctx, to_tokens ? "patchify" : "unpatchify");
    CUDA_TRY(ctx, patchify_launch(src->ptr, is_f32(src), dst->ptr, is_f32(dst), (int)c, (int)t, (int)h, (int)w, (int)p,
                                  to_tokens, ctx->stream));
    ctx->launches++;
    CUDA_TRY(ctx, note_uses(ctx, {src, dst}));
    return LX2V_OK;
}

extern "C" lx2v_status lx2v_patchify(lx2v_ctx *ctx, const lx2v_buf *latent, size_t c, size_t t, size_t h, size_t w,
                                     size_t p, lx2v_buf *out) {
    return patchify_impl(ctx, latent, c, t, h, w, p, out, 1);
}

extern "C" lx2v_status lx2v_unpatchify(lx2v_ctx *ctx, const lx2v_buf *x, size_t c, size_t t, size_t h, size_t w,
                                       size_t p, lx2v_buf *out) {
    return patchify_impl(ctx, x, c, t, h, w, p, out, 0);
}

extern "C" lx2v_status lx2v_dmd_step(lx2v_ctx *ctx, lx2v_buf *x, const lx2v_buf *v, const lx2v_buf *noise,
                                     float sigma_t, float sigma_next, size_t n) {
    lx2v_status s = enter(ctx);
    if (s) return s;
    if (!x || !v || n > x->len || n > v->len || (noise && n > noise->len))
        return fail(ctx, LX2V_ERR_INVALID, "dmd_step buffers hold fewer than n elements");
    if (n == 0) return LX2V_OK;
    OpScope ps(ctx, "dmd_step");
    CUDA_TRY(ctx, dmd_step_launch(x->ptr, is_f32(x), v->ptr, is_f32(v), noise ? noise->ptr : nullptr, is_f32(noise),
                                  sigma_t, sigma_next, (int64_t)n, ctx->stream));
    ctx->launches++;
    CUDA_TRY(ctx, note_uses(ctx, {x, v, noise}));
    return LX2V_OK;
}

// ---- profiling / knobs ---------------------------------------------------------------------
extern "C" lx2v_status lx2v_profile_json(lx2v_ctx *ctx, char *buf, size_t cap, size_t *written) {
    lx2v_status s = enter(ctx);
    if (s) return s;
    resolve_profile(ctx);
    std::string js = "{";
    bool first = true;
    for (auto &kv : ctx->prof) {
        char tmp[256];
        snprintf(tmp, sizeof tmp, "%s\"%s\": {\"calls\": %llu, \"ms\": %.6f}", first ? "" : ", ", kv.first.c_str(),
                 (unsigned long long)kv.second.calls, kv.second.ms);
        js += tmp;
        first = false;
    }
    js += "}";
    if (written) *written = js.size() + 1;
    if (buf && cap) snprintf(buf, cap, "%s", js.c_str());
    return LX2V_OK;
}

extern "C" lx2v_status lx2v_profile_reset(lx2v_ctx *ctx) {
    lx2v_status s = enter(ctx);
    if (s) return s;
    resolve_profile(ctx);
    ctx->prof.clear();
    return LX2V_OK;
}

extern "C" lx2v_status lx2v_set_linear_path(lx2v_ctx *ctx, int path) {
    if (!ctx) return fail(nullptr, LX2V_ERR_INVALID, "null context");
    if (path < 0 || path > 5) return fail(ctx, LX2V_ERR_INVALID, "bad path %d", path);
    ctx->path = path;
    return LX2V_OK;
}

extern "C" lx2v_status lx2v_set_split_mode(lx2v_ctx *ctx, int mode) {
    if (!ctx) return fail(nullptr, LX2V_ERR_INVALID, "null context");
    if (mode < 0 || mode > 2) return fail(ctx, LX2V_ERR_INVALID, "bad split mode %d", mode);
    ctx->split_mode = mode;
    return LX2V_OK;
}

extern "C" lx2v_status lx2v_set_token_tile(lx2v_ctx *ctx, int tokens) {
    if (!ctx) return fail(nullptr, LX2V_ERR_INVALID, "null context");
    if (tokens != 0 && tokens != 128 && tokens != 192 && tokens != 256)
        return fail(ctx, LX2V_ERR_INVALID, "token tile must be 0 (automatic), 128, 192 or 256, got %d", tokens);
    ctx->token_tile = tokens;
    return LX2V_OK;
}

extern "C" lx2v_status lx2v_set_wait_limit_ns(lx2v_ctx *ctx, uint64_t ns) {
    if (!ctx) return fail(nullptr, LX2V_ERR_INVALID, "null context");
    if (ns == 0) return fail(ctx, LX2V_ERR_INVALID, "wait limit must be positive");
    ctx->wait_limit_ns = ns;
    return LX2V_OK;
}

extern "C" lx2v_status lx2v_launch_count(lx2v_ctx *ctx, uint64_t *count) {
    if (!ctx) return fail(nullptr, LX2V_ERR_INVALID, "null context");
    if (!count) return fail(ctx, LX2V_ERR_INVALID, "null output");
    *count = ctx->launches;
    return LX2V_OK;
}

// ---- linear without device allocation -------------------------------------------------
// Some callers cannot let the library call cudaMalloc during a linear: a
// serving loop that planned all of its device memory up front (the
// reference's VRAM plan) and must not grow it in the middle of a request, or
// a caller for whom cudaMalloc's implicit device-wide synchronisation would
// stall work on other streams. lx2v_linear may allocate (the stream-K
// workspace, grown on first use); lx2v_linear_noalloc runs the same CTA-pair
// kernel with its stream-K scratch in a fixed array that the library holds
// on every device it is loaded on, and allocates nothing.
//
// The scratch: [flags: LX2V_NOALLOC_FLAG_BYTES][partial tiles ...]. The
// flags hold launch epochs (a per-device counter below), so they start at
// zero (static initialisation) and never need clearing while epochs grow.
static __device__ __align__(256) unsigned char g_noalloc_scratch[LX2V_NOALLOC_SCRATCH_BYTES];
static constexpr size_t LX2V_NOALLOC_FLAG_BYTES = 4096;
static constexpr int LX2V_NOALLOC_MAX_DEVICES = 64;
static constexpr int LX2V_NOALLOC_TOKENS = 128;  // token tile: smallest partial tiles

struct NoallocDevice {
    void *scratch = nullptr;  // device address of g_noalloc_scratch on this device
    int epoch = 0;
};
static NoallocDevice g_noalloc[LX2V_NOALLOC_MAX_DEVICES];
static std::mutex g_noalloc_mu;

// Device address of the scratch array on ctx->dev (current device), looked up
// once per device. In host code g_noalloc_scratch names a host-side shadow,
// not device memory, so the kernel must get this address instead.
static lx2v_status noalloc_scratch(lx2v_ctx *ctx, void **ptr, int *epoch) {
    if (ctx->dev < 0 || ctx->dev >= LX2V_NOALLOC_MAX_DEVICES)
        return fail(ctx, LX2V_ERR_UNSUPPORTED, "device %d is beyond the %d devices the static scratch tracks",
                    ctx->dev, LX2V_NOALLOC_MAX_DEVICES);
    std::lock_guard<std::mutex> lock(g_noalloc_mu);
    NoallocDevice &d = g_noalloc[ctx->dev];
    if (!d.scratch) {
        void *p = nullptr;
        cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
        if (e != cudaSuccess || !p)
            return fail(ctx, LX2V_ERR_CUDA, "cudaGetSymbolAddress(static scratch) on device %d: %s", ctx->dev,
                        cudaGetErrorString(e));
        d.scratch = p;
    }
    if (++d.epoch <= 0) {
        // epoch counter wrapped: old flags could match again, so clear them
        CUDA_TRY(ctx, cudaMemsetAsync(d.scratch, 0, LX2V_NOALLOC_FLAG_BYTES, ctx->stream));
        d.epoch = 1;
    }
    *ptr = d.scratch;
    *epoch = d.epoch;
    return LX2V_OK;
}

// Stream-K flags of this context's workspace and of the device's static
// scratch back to zero (after a kernel stopped on an expired wait).
static cudaError_t clear_split_flags(lx2v_ctx *ctx) {
    if (ctx->sk_ws) {
        const size_t flag_bytes = (size_t)ctx->num_sms * 2 * 8 * sizeof(int);
        cudaError_t e = cudaMemsetAsync((char *)ctx->sk_ws + (ctx->sk_ws_bytes - flag_bytes), 0, flag_bytes,
                                        ctx->stream);
        if (e != cudaSuccess) return e;
    }
    void *scratch = nullptr;
    if (ctx->dev >= 0 && ctx->dev < LX2V_NOALLOC_MAX_DEVICES) {
        std::lock_guard<std::mutex> lock(g_noalloc_mu);
        scratch = g_noalloc[ctx->dev].scratch;
    }
    if (scratch) return cudaMemsetAsync(scratch, 0, LX2V_NOALLOC_FLAG_BYTES, ctx->stream);
    return cudaSuccess;
}

extern "C" lx2v_status lx2v_linear_noalloc(lx2v_ctx *ctx, const lx2v_buf *x, size_t x_row, size_t rows,
                                           const lx2v_weight *w, const lx2v_buf *bias, int act, lx2v_buf *y,
                                           size_t y_row) {
    lx2v_status s = enter(ctx);
    if (s) return s;
    if (!x || !w || !y) return fail(ctx, LX2V_ERR_INVALID, "null x, weight or output");
    if (act != LX2V_ACT_NONE && act != LX2V_ACT_GELU_TANH) return fail(ctx, LX2V_ERR_INVALID, "bad act %d", act);
    if (x == y || (x->ptr && x->ptr == y->ptr)) return fail(ctx, LX2V_ERR_INVALID, "output aliases input");
    const size_t N = w->rows, K = w->cols;
    if ((x_row + rows) * K > x->len)
        return fail(ctx, LX2V_ERR_INVALID, "x has %zu elements, rows [%zu, %zu) x %zu need more", x->len, x_row,
                    x_row + rows, K);
    if ((y_row + rows) * N > y->len)
        return fail(ctx, LX2V_ERR_INVALID, "output has %zu elements, rows [%zu, %zu) x %zu need more", y->len,
                    y_row, y_row + rows, N);
    if (bias && bias->len < N) return fail(ctx, LX2V_ERR_INVALID, "bias has %zu elements, need %zu", bias->len, N);
    if (rows == 0) return LX2V_OK;
    if (rows > (1u << 30)) return fail(ctx, LX2V_ERR_UNSUPPORTED, "too many rows");
    OpScope ps(ctx, "linear_noalloc");
    const size_t grp = w->group;
    const bool groups_ok = w->fmt == LX2V_W_BF16 || grp % 64 == 0 ||
                           (w->fmt == LX2V_W_Q4 && (grp == 16 || grp == 32));
    if (!(x->dtype == LX2V_BF16 && K % 16 == 0 && N % 16 == 0 && groups_ok &&
          unit_path_ok(w->fmt, (int)K, (int)w->group) && rows >= 16))
        return fail(ctx, LX2V_ERR_UNSUPPORTED, "the tensor-core kernel does not take this shape/dtype");
    // Scratch this launch may touch: every pair of the grid holds two
    // 128 x 128 f32 partial tiles, plus the flags.
    const int bt = LX2V_NOALLOC_TOKENS;
    const int pairs = ctx->num_sms / 2;
    const size_t need = LX2V_NOALLOC_FLAG_BYTES + (size_t)pairs * 2 * 128 * bt * sizeof(float);
    if (pairs * 2 * (int)sizeof(int) > (int)LX2V_NOALLOC_FLAG_BYTES || need > LX2V_NOALLOC_SCRATCH_BYTES)
        return fail(ctx, LX2V_ERR_UNSUPPORTED,
                    "this GPU (%d SMs) needs %zu bytes of scratch, beyond the %zu-byte static maximum",
                    ctx->num_sms, need, (size_t)LX2V_NOALLOC_SCRATCH_BYTES);
    GemmParams p;
    memset(&p, 0, sizeof p);
    s = make_map(ctx, &p.tmap_x, x->ptr, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, K, x_row + rows, 64,
                 (uint32_t)(bt / 2), CU_TENSOR_MAP_SWIZZLE_128B);
    if (s) return s;
    if (w->fmt == LX2V_W_Q4)
        s = make_map(ctx, &p.tmap_w, w->codes, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, K / 2, N, 32, 128,
                     CU_TENSOR_MAP_SWIZZLE_32B);
    else if (w->fmt == LX2V_W_BF16)
        s = make_map(ctx, &p.tmap_w, w->codes, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, K, N, 64, 128,
                     CU_TENSOR_MAP_SWIZZLE_128B);
    else
        s = make_map(ctx, &p.tmap_w, w->codes, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, K, N, 64, 128,
                     CU_TENSOR_MAP_SWIZZLE_64B);
    if (s) return s;
    if (w->fmt != LX2V_W_BF16) {
        const int sgrp = grp % 64 == 0 ? 1 : (int)(64 / grp);
        p.sgrp = sgrp;
        p.gshift = grp % 64 == 0 ? 6 : (grp == 16 ? 4 : 5);
        s = make_map(ctx, &p.tmap_s, w->fmt == LX2V_W_Q4 ? (void *)w->sz_t : (void *)w->scales_t,
                     CU_TENSOR_MAP_DATA_TYPE_UINT32, 4, N, K / grp, 128, (uint32_t)sgrp, CU_TENSOR_MAP_SWIZZLE_NONE);
        if (s) return s;
    }
    if (w->fmt == LX2V_W_FP8) {
        s = make_map(ctx, &p.tmap_f, w->flags, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, N, (size_t)fp8_flag_cols((int)K),
                     128, 2, CU_TENSOR_MAP_SWIZZLE_NONE);
        if (s) return s;
    }
    void *scratch = nullptr;
    int epoch = 0;
    s = noalloc_scratch(ctx, &scratch, &epoch);
    if (s) return s;
    p.y = y->ptr;
    p.codes = (const uint8_t *)w->codes;
    p.scales_t = w->scales_t;
    p.sz_t = w->sz_t;
    p.bias = bias ? bias->ptr : nullptr;
    p.bias_f32 = bias && bias->dtype == LX2V_F32;
    p.err = ctx->err_dev;
    p.wait_limit_ns = ctx->wait_limit_ns;
    p.M = (int)rows; p.N = (int)N; p.K = (int)K; p.group = (int)w->group;
    p.x_row = (int)x_row; p.y_row = (int)y_row;
    p.act = act;
    p.out_f32 = y->dtype == LX2V_F32;
    p.kgroup = K % 128 == 0 ? 2 : 1;
    p.streamk = 1;
    p.epoch = epoch;
    p.flags = (int *)scratch;
    p.partials = (float *)((char *)scratch + LX2V_NOALLOC_FLAG_BYTES);
    CUDA_TRY(ctx, gemm_pair_launch(w->fmt, bt, p, ctx->num_sms, ctx->stream));
    ctx->launches++;
    CUDA_TRY(ctx, note_uses(ctx, {x, bias, y}));
    return LX2V_OK;
}

// ---- tensor-parallel collectives (NCCL) ------------------------------------------------------
// NCCL is opened on first use (dlopen of libnccl.so.2, the library the host
// process already uses when it has one), so that single-GPU callers of this
// library do not depend on it. The all-reduce runs on the context's stream,
// ordered like every other call.
namespace {
struct NcclApi {
    bool ok = false;
    std::string err;
    ncclResult_t (*get_unique_id)(ncclUniqueId *) = nullptr;
    ncclResult_t (*comm_init_rank)(ncclComm_t *, int, ncclUniqueId, int) = nullptr;
    ncclResult_t (*all_reduce)(const void *, void *, size_t, ncclDataType_t, ncclRedOp_t, ncclComm_t,
                               cudaStream_t) = nullptr;
    ncclResult_t (*comm_destroy)(ncclComm_t) = nullptr;
    const char *(*error_string)(ncclResult_t) = nullptr;
};

NcclApi &nccl() {
    static NcclApi api;
    static std::once_flag once;
    std::call_once(once, [] {
        void *h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
        if (!h) {
            const char *e = dlerror();
            api.err = std::string("cannot open libnccl.so.2: ") + (e ? e : "?");
            return;
        }
        api.get_unique_id = reinterpret_cast<decltype(api.get_unique_id)>(dlsym(h, "ncclGetUniqueId"));
        api.comm_init_rank = reinterpret_cast<decltype(api.comm_init_rank)>(dlsym(h, "ncclCommInitRank"));
        api.all_reduce = reinterpret_cast<decltype(api.all_reduce)>(dlsym(h, "ncclAllReduce"));
        api.comm_destroy = reinterpret_cast<decltype(api.comm_destroy)>(dlsym(h, "ncclCommDestroy"));
        api.error_string = reinterpret_cast<decltype(api.error_string)>(dlsym(h, "ncclGetErrorString"));
        api.ok = api.get_unique_id && api.comm_init_rank && api.all_reduce && api.comm_destroy && api.error_string;
        if (!api.ok) api.err = "libnccl.so.2 lacks an expected symbol";
    });
    return api;
}
}  // namespace

static void comm_destroy(lx2v_ctx *ctx) {
    if (ctx->comm && nccl().ok) nccl().comm_destroy(ctx->comm);
    ctx->comm = nullptr;
    ctx->comm_rank = 0;
    ctx->comm_world = 1;
}

static_assert(sizeof(ncclUniqueId) == LX2V_COMM_ID_BYTES, "NCCL unique id size");

extern "C" lx2v_status lx2v_comm_unique_id(unsigned char *out, size_t cap) {
    if (!out || cap < LX2V_COMM_ID_BYTES) return fail(nullptr, LX2V_ERR_INVALID, "need %d bytes for the id", LX2V_COMM_ID_BYTES);
    NcclApi &api = nccl();
    if (!api.ok) return fail(nullptr, LX2V_ERR_UNSUPPORTED, "%s", api.err.c_str());
    ncclUniqueId id;
    const ncclResult_t r = api.get_unique_id(&id);
    if (r != ncclSuccess) return fail(nullptr, LX2V_ERR_CUDA, "ncclGetUniqueId: %s", api.error_string(r));
    memcpy(out, &id, sizeof id);
    return LX2V_OK;
}

extern "C" lx2v_status lx2v_comm_init(lx2v_ctx *ctx, const unsigned char *id, int rank, int world) {
    lx2v_status s = enter(ctx);
    if (s) return s;
    if (!id || world < 1 || rank < 0 || rank >= world)
        return fail(ctx, LX2V_ERR_INVALID, "bad comm arguments (rank %d of %d)", rank, world);
    NcclApi &api = nccl();
    if (!api.ok) return fail(ctx, LX2V_ERR_UNSUPPORTED, "%s", api.err.c_str());
    CUDA_TRY(ctx, cudaStreamSynchronize(ctx->stream));
    comm_destroy(ctx);
    ncclUniqueId uid;
    memcpy(&uid, id, sizeof uid);
    ncclComm_t comm = nullptr;
    const ncclResult_t r = api.comm_init_rank(&comm, world, uid, rank);
    if (r != ncclSuccess) return fail(ctx, LX2V_ERR_CUDA, "ncclCommInitRank: %s", api.error_string(r));
    ctx->comm = comm;
    ctx->comm_rank = rank;
    ctx->comm_world = world;
    return LX2V_OK;
}

extern "C" lx2v_status lx2v_all_reduce_sum(lx2v_ctx *ctx, lx2v_buf *buf, size_t len) {
    lx2v_status s = enter(ctx);
    if (s) return s;
    if (!buf || len > buf->len) return fail(ctx, LX2V_ERR_INVALID, "all-reduce range out of bounds");
    if (!ctx->comm) return fail(ctx, LX2V_ERR_INVALID, "no communicator: call lx2v_comm_init first");
    if (len == 0) return LX2V_OK;
    OpScope ps(ctx, "all_reduce");
    const ncclResult_t r = nccl().all_reduce(buf->ptr, buf->ptr, len,
                                             buf->dtype == LX2V_F32 ? ncclFloat32 : ncclBfloat16, ncclSum,
                                             ctx->comm, ctx->stream);
    if (r != ncclSuccess) return fail(ctx, LX2V_ERR_CUDA, "ncclAllReduce: %s", nccl().error_string(r));
    CUDA_TRY(ctx, note_use(ctx, buf));
    return LX2V_OK;
}

// ---- tensor parallelism over NVLink peer memory --------------------------------------
extern "C" lx2v_status lx2v_buf_ipc_handle(lx2v_ctx *ctx, const lx2v_buf *buf, unsigned char *out, size_t cap) {
    lx2v_status s = enter(ctx);
    if (s) return s;
    if (!buf || !buf->ptr || buf->ipc) return fail(ctx, LX2V_ERR_INVALID, "no own device buffer to share");
    if (!out || cap < sizeof(cudaIpcMemHandle_t)) return fail(ctx, LX2V_ERR_INVALID, "handle buffer too small");
    cudaIpcMemHandle_t h;
    CUDA_TRY(ctx, cudaIpcGetMemHandle(&h, buf->ptr));
    memcpy(out, &h, sizeof h);
    return LX2V_OK;
}

extern "C" lx2v_status lx2v_buf_open_ipc(lx2v_ctx *ctx, const unsigned char *handle, size_t len, int dtype,
                                         lx2v_buf **out) {
    lx2v_status s = enter(ctx);
    if (s) return s;
    if (!handle || !out || !valid_dtype(dtype)) return fail(ctx, LX2V_ERR_INVALID, "bad handle, output or dtype");
    cudaIpcMemHandle_t h;
    memcpy(&h, handle, sizeof h);
    void *ptr = nullptr;
    CUDA_TRY(ctx, cudaIpcOpenMemHandle(&ptr, h, cudaIpcMemLazyEnablePeerAccess));
    auto *b = new lx2v_buf();
    b->ptr = ptr;
    b->len = len;
    b->dtype = dtype;
    b->ipc = true;
    *out = b;
    return LX2V_OK;
}

struct lx2v_peers {
    int rank = 0, world = 1;
    PeerFlags flags;
    unsigned epoch = 0;
};

extern "C" lx2v_status lx2v_peers_create(lx2v_ctx *ctx, int rank, int world, lx2v_buf *const *flag_bufs,
                                         lx2v_peers **out) {
    lx2v_status s = enter(ctx);
    if (s) return s;
    if (!out || !flag_bufs || world < 1 || world > LX2V_MAX_PEERS || rank < 0 || rank >= world)
        return fail(ctx, LX2V_ERR_INVALID, "bad peer group (rank %d, world %d, at most %d ranks)", rank, world,
                    LX2V_MAX_PEERS);
    auto *g = new lx2v_peers();
    g->rank = rank;
    g->world = world;
    memset(&g->flags, 0, sizeof g->flags);
    for (int r = 0; r < world; ++r) {
        const lx2v_buf *f = flag_bufs[r];
        if (!f || !f->ptr || f->len * esize(f->dtype) < (size_t)world * 4) {
            delete g;
            return fail(ctx, LX2V_ERR_INVALID, "flag buffer of rank %d holds fewer than %d u32", r, world);
        }
        g->flags.flags[r] = (unsigned *)f->ptr;
    }
    *out = g;
    return LX2V_OK;
}

extern "C" void lx2v_peers_free(lx2v_peers *g) { delete g; }

extern "C" lx2v_status lx2v_peers_barrier(lx2v_ctx *ctx, lx2v_peers *g) {
    lx2v_status s = enter(ctx);
    if (s) return s;
    if (!g) return fail(ctx, LX2V_ERR_INVALID, "null peer group");
    OpScope ps(ctx, "peer_barrier");
    if (++g->epoch == 0) g->epoch = 1;
    CUDA_TRY(ctx, peer_barrier_launch(g->flags, g->world, g->rank, g->epoch, ctx->err_dev, ctx->wait_limit_ns,
                                      ctx->stream));
    ctx->launches++;
    return LX2V_OK;
}

extern "C" lx2v_status lx2v_tp_reduce_norm(lx2v_ctx *ctx, lx2v_peers *g, lx2v_buf *const *parts, lx2v_buf *h,
                                           size_t row0, size_t row1, size_t dim, const lx2v_buf *gate_mods, long gate,
                                           int kind, const lx2v_buf *w, const lx2v_buf *b, const lx2v_buf *norm_mods,
                                           size_t scale, size_t shift, float eps, lx2v_buf *const *normed) {
    lx2v_status s = enter(ctx);
    if (s) return s;
    if (!g || !h || !normed) return fail(ctx, LX2V_ERR_INVALID, "null peer group, h or outputs");
    if (!is_f32(h) || row1 * dim > h->len || row0 > row1)
        return fail(ctx, LX2V_ERR_INVALID, "h must be f32 holding rows [row0, row1) of width dim");
    if (!tp_reduce_norm_supported((int)dim))
        return fail(ctx, LX2V_ERR_UNSUPPORTED, "rows of %zu values (a multiple of 8, at most 8192)", dim);
    if (parts && gate >= 0 && (!gate_mods || gate_mods->len < ((size_t)gate + 1) * dim))
        return fail(ctx, LX2V_ERR_INVALID, "gate row beyond mods");
    NormArgs na;  // the norm's parameter checks, on this rank's output
    if ((s = norm_args(ctx, na, row1, dim, kind, w, b, scale, shift, norm_mods, eps, normed[g->rank]))) return s;
    TpNormArgs a;
    memset(&a, 0, sizeof a);
    for (int r = 0; r < g->world; ++r) {
        const lx2v_buf *o = normed[r];
        if (!o || o->len < row1 * dim || o->dtype != normed[g->rank]->dtype)
            return fail(ctx, LX2V_ERR_INVALID, "output of rank %d holds fewer than row1 x dim or differs in dtype", r);
        a.outs[r] = o->ptr;
        if (parts) {
            const lx2v_buf *p = parts[r];
            if (!p || p->len < row1 * dim || p->dtype != parts[0]->dtype)
                return fail(ctx, LX2V_ERR_INVALID, "partial of rank %d holds fewer than row1 x dim or differs in dtype",
                            r);
            a.parts[r] = p->ptr;
        }
    }
    a.n_outs = g->world;
    a.out_f32 = is_f32(normed[g->rank]);
    a.n_parts = parts ? g->world : 0;
    a.parts_f32 = parts ? is_f32(parts[0]) : 0;
    a.h = h->ptr;
    a.row0 = (int64_t)row0; a.row1 = (int64_t)row1; a.dim = (int)dim;
    a.gmods = gate_mods ? gate_mods->ptr : nullptr; a.gmods_f32 = is_f32(gate_mods);
    a.gate = parts && gate >= 0 ? (int)gate : -1;
    a.kind = kind;
    a.w = na.w; a.w_f32 = na.w_f32; a.b = na.b; a.b_f32 = na.b_f32;
    a.nmods = na.mods; a.nmods_f32 = na.mods_f32; a.scale = na.scale; a.shift = na.shift;
    a.eps = eps;
    if (row1 == row0) return LX2V_OK;
    OpScope ps(ctx, "tp_reduce_norm");
    CUDA_TRY(ctx, tp_reduce_norm_launch(a, ctx->stream));
    ctx->launches++;
    CUDA_TRY(ctx, note_uses(ctx, {h, gate_mods, w, b, norm_mods, normed[g->rank]}));
    return LX2V_OK;
}

extern "C" lx2v_status lx2v_row_sumsq_peers(lx2v_ctx *ctx, lx2v_peers *g, const lx2v_buf *src, size_t rows,
                                            size_t src_stride, size_t col_off, size_t width, lx2v_buf *const *outs) {
    lx2v_status s = enter(ctx);
    if (s) return s;
    if (!g || !src || !outs) return fail(ctx, LX2V_ERR_INVALID, "null peer group, source or outputs");
    if (col_off + width > src_stride || (rows && (rows - 1) * src_stride + col_off + width > src->len))
        return fail(ctx, LX2V_ERR_INVALID, "row_sumsq columns beyond src");
    PeerRowSums a;
    memset(&a, 0, sizeof a);
    for (int r = 0; r < g->world; ++r) {
        const lx2v_buf *o = outs[r];
        if (!o || o->dtype != LX2V_F32 || o->len < rows * (size_t)g->world)
            return fail(ctx, LX2V_ERR_INVALID, "sums of rank %d: f32 of world x rows elements needed", r);
        a.outs[r] = (float *)o->ptr;
    }
    a.n_outs = g->world;
    a.slot = (int64_t)g->rank * (int64_t)rows;
    a.src = src->ptr; a.src_f32 = is_f32(src);
    a.rows = (int64_t)rows; a.stride = (int64_t)src_stride; a.col_off = (int64_t)col_off; a.width = (int)width;
    if (rows == 0) return LX2V_OK;
    OpScope ps(ctx, "row_sumsq_peers");
    CUDA_TRY(ctx, row_sumsq_peers_launch(a, ctx->stream));
    ctx->launches++;
    CUDA_TRY(ctx, note_uses(ctx, {src, outs[g->rank]}));
    return LX2V_OK;
}

// ---- sparse attention (backend.rs:309-331, crates/lightx2v-core/src/sparse.rs) ---------------
struct lx2v_sparse {
    int heads = 0, seq = 0, d = 0, nt = 0, topk = 0, sel_words = 0, words = 0;
    float scale = 0.0f;
    uint32_t *slot_src = nullptr;
    int *block_sizes = nullptr, *token_tile = nullptr;
    float *pooled = nullptr;  // cq, ck, cv, coarse_out: 4 x [heads][nt][d]
    uint32_t *sel = nullptr, *bits = nullptr;
};

static void sparse_release(lx2v_sparse *sp) {
    if (!sp) return;
    cudaFree(sp->slot_src); cudaFree(sp->block_sizes); cudaFree(sp->token_tile);
    cudaFree(sp->pooled); cudaFree(sp->sel); cudaFree(sp->bits);
    delete sp;
}

// The fine stage's per-head token mask is heads x seq x seq bits.
static constexpr size_t SPARSE_MASK_MAX_BYTES = 512ull << 20;

extern "C" lx2v_status lx2v_sparse_prepare(lx2v_ctx *ctx, const uint32_t *slot_src, const uint32_t *block_sizes,
                                           size_t num_tiles, size_t seq, size_t heads, size_t head_dim, size_t topk,
                                           float scale, lx2v_sparse **out) {
    lx2v_status s = enter(ctx);
    if (s) return s;
    if (!out || !slot_src || !block_sizes || num_tiles == 0 || seq == 0 || heads == 0 || head_dim == 0 ||
        topk == 0 || topk > num_tiles)
        return fail(ctx, LX2V_ERR_INVALID, "bad sparse plan (tiles %zu, seq %zu, heads %zu, topk %zu)", num_tiles, seq,
                    heads, topk);
    const size_t words = (seq + 31) / 32;
    if (heads * seq * words * 4 > SPARSE_MASK_MAX_BYTES || num_tiles > 16384 || seq > (1u << 30))
        return fail(ctx, LX2V_ERR_UNSUPPORTED, "sparse attention over %zu tokens x %zu heads: the fine-stage mask "
                    "would exceed %zu MiB", seq, heads, SPARSE_MASK_MAX_BYTES >> 20);
    // host checks of the plan: every token in exactly one slot, tile sizes as the slots say
    std::vector<int> token_tile(seq, -1), sizes(num_tiles);
    for (size_t t = 0; t < num_tiles; ++t) {
        if (block_sizes[t] > (uint32_t)VSA_TILE) return fail(ctx, LX2V_ERR_INVALID, "tile %zu holds > 64 tokens", t);
        sizes[t] = (int)block_sizes[t];
        for (size_t i = 0; i < VSA_TILE; ++i) {
            const uint32_t tok = slot_src[t * VSA_TILE + i];
            const bool real = i < block_sizes[t];
            if (real != (tok != 0xFFFFFFFFu) || (real && (tok >= seq || token_tile[tok] >= 0)))
                return fail(ctx, LX2V_ERR_INVALID, "slot %zu of tile %zu disagrees with the plan", i, t);
            if (real) token_tile[tok] = (int)t;
        }
    }
    for (size_t i = 0; i < seq; ++i)
        if (token_tile[i] < 0) return fail(ctx, LX2V_ERR_INVALID, "token %zu is in no tile", i);
    auto *sp = new lx2v_sparse();
    sp->heads = (int)heads; sp->seq = (int)seq; sp->d = (int)head_dim; sp->nt = (int)num_tiles;
    sp->topk = (int)topk; sp->scale = scale; sp->words = (int)words; sp->sel_words = (int)((num_tiles + 31) / 32);
    const size_t hnd = heads * num_tiles * head_dim;
    cudaError_t e = cudaMalloc(&sp->slot_src, num_tiles * VSA_TILE * 4);
    if (e == cudaSuccess) e = cudaMalloc(&sp->block_sizes, num_tiles * 4);
    if (e == cudaSuccess) e = cudaMalloc(&sp->token_tile, seq * 4);
    if (e == cudaSuccess) e = cudaMalloc(&sp->pooled, 4 * hnd * 4);
    if (e == cudaSuccess) e = cudaMalloc(&sp->sel, heads * num_tiles * sp->sel_words * 4);
    if (e == cudaSuccess) e = cudaMalloc(&sp->bits, heads * seq * words * 4);
    if (e == cudaSuccess) e = cudaMemcpy(sp->slot_src, slot_src, num_tiles * VSA_TILE * 4, cudaMemcpyHostToDevice);
    if (e == cudaSuccess) e = cudaMemcpy(sp->block_sizes, sizes.data(), num_tiles * 4, cudaMemcpyHostToDevice);
    if (e == cudaSuccess) e = cudaMemcpy(sp->token_tile, token_tile.data(), seq * 4, cudaMemcpyHostToDevice);
    if (e != cudaSuccess) {
        sparse_release(sp);
        return fail(ctx, e == cudaErrorMemoryAllocation ? LX2V_ERR_OOM : LX2V_ERR_CUDA, "sparse state: %s",
                    cudaGetErrorString(e));
    }
    *out = sp;
    return LX2V_OK;
}

extern "C" void lx2v_sparse_free(lx2v_ctx *ctx, lx2v_sparse *sp) {
    if (!sp) return;
    if (ctx) {
        cudaSetDevice(ctx->dev);
        cudaStreamSynchronize(ctx->stream);
    }
    sparse_release(sp);
}

extern "C" lx2v_status lx2v_sparse_attention(lx2v_ctx *ctx, const lx2v_buf *q, const lx2v_buf *k, const lx2v_buf *v,
                                             const lx2v_buf *gate, const lx2v_sparse *sp, lx2v_buf *out) {
    lx2v_status s = enter(ctx);
    if (s) return s;
    if (!sp || !gate) return fail(ctx, LX2V_ERR_INVALID, "null sparse state or gate");
    const size_t n = (size_t)sp->heads * sp->seq * sp->d;
    if (!q || !k || !v || q->len < n || k->len < n || v->len < n || gate->len < n)
        return fail(ctx, LX2V_ERR_INVALID, "q / k / v / gate hold fewer than heads x seq x head_dim");
    if (q->dtype != k->dtype || k->dtype != v->dtype)
        return fail(ctx, LX2V_ERR_INVALID, "q, k and v must have the same element type");
    if (out == gate) return fail(ctx, LX2V_ERR_INVALID, "output aliases the gate");
    VsaArgs a;
    memset(&a, 0, sizeof a);
    a.heads = sp->heads; a.seq = sp->seq; a.d = sp->d; a.nt = sp->nt; a.topk = sp->topk; a.scale = sp->scale;
    a.q = q->ptr; a.k = k->ptr; a.v = v->ptr; a.qkv_f32 = is_f32(q);
    a.gate = gate->ptr; a.gate_f32 = is_f32(gate);
    a.out = out ? out->ptr : nullptr; a.out_f32 = is_f32(out);
    a.slot_src = sp->slot_src; a.block_sizes = sp->block_sizes; a.token_tile = sp->token_tile;
    const size_t hnd = (size_t)sp->heads * sp->nt * sp->d;
    a.cq = sp->pooled; a.ck = sp->pooled + hnd; a.cv = sp->pooled + 2 * hnd; a.coarse_out = sp->pooled + 3 * hnd;
    a.sel = sp->sel; a.sel_words = sp->sel_words; a.bits = sp->bits; a.words = sp->words;
    {
        OpScope ps(ctx, "sparse_select");
        CUDA_TRY(ctx, vsa_select_launch(a, ctx->stream));
        ctx->launches += 3;
    }
    AttnMaskArgs m;
    m.mode = ATT_MASK_BITS;
    m.dev_bits = sp->bits;
    if ((s = attention_buffers(ctx, "sparse_attention", q, k, v, sp->heads, sp->seq, sp->seq, sp->d, m, out)))
        return s;
    OpScope ps(ctx, "sparse_combine");
    CUDA_TRY(ctx, vsa_combine_launch(a, ctx->stream));
    ctx->launches++;
    CUDA_TRY(ctx, note_uses(ctx, {q, k, v, gate, out}));
    return LX2V_OK;
}

