// api.cu -- the extern "C" surface of libstyx_moe.so (include/styx_moe.h).
//
// Host-side validation, workspace layout and launch planning for the MoE
// block; the kernels live in moe_kernels.cu and synth.cu.
#include <algorithm>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <string>

#include <cuda.h>
#include <cuda_runtime.h>

#include "../../include/styx_attn.h"
#include "../../include/styx_moe.h"
#include "kernels.h"

// the context's scratch: styx_argmax_f32's partial maxima and ticket, then
// the dense GEMV's id block (expert 0 from the full tensor) and its weight 1
constexpr size_t kScratchDenseIds = 2560, kScratchOne = kScratchDenseIds + 256, kScratchBytes = 4096;
static_assert(styx::kArgmaxCtas * 8 + 4 <= kScratchDenseIds, "argmax scratch overlaps the id block");

struct styx_ctx {
    int device = 0;
    int sm_count = 0;
    char name[256] = {0};
    int *d_err = nullptr;   // device error word of bounded waits; d_err[4..7]: zeros (a one-expert id row)
    void *d_scratch = nullptr;   // styx_argmax_f32's partial maxima and ticket (zeroed at init)
    int moe_kernels = 0;    // STYX_OPT_MOE_KERNELS
    int last_path = 0;      // STYX_OPT_MOE_LAST_PATH
    int trace = 0;          // STYX_OPT_TRACE
    int moe_layers = 0;     // STYX_OPT_MOE_LAYERS
    int exclusive = 0;      // STYX_OPT_EXCLUSIVE
    int attn_kernels = 0;   // STYX_OPT_ATTN_KERNELS
    int attn_last_path = 0; // STYX_OPT_ATTN_LAST_PATH
    int last_cluster = 0;   // STYX_OPT_MOE_LAST_CLUSTER
};

namespace {

thread_local std::string g_err;

int fail(int code, const char *fmt, ...) {
    char buf[1024];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof(buf), fmt, ap);
    va_end(ap);
    g_err = buf;
    return code;
}

#define CK(call)                                                                                   \
    do {                                                                                           \
        cudaError_t e_ = (call);                                                                   \
        if (e_ != cudaSuccess) return fail(STYX_ECUDA, "%s: %s", #call, cudaGetErrorString(e_));   \
    } while (0)

#define NEED(cond, ...)                                                                            \
    do {                                                                                           \
        if (!(cond)) return fail(STYX_EINVAL, __VA_ARGS__);                                        \
    } while (0)

inline cudaStream_t S(styx_stream s) { return static_cast<cudaStream_t>(s); }

int enter(styx_ctx *ctx) {
    if (!ctx) return fail(STYX_EINVAL, "null ctx");
    CK(cudaSetDevice(ctx->device));
    return STYX_OK;
}
#define ENTER(ctx)                                                                                 \
    do {                                                                                           \
        int rc_ = enter(ctx);                                                                      \
        if (rc_) return rc_;                                                                       \
    } while (0)

bool qtype_ok(int qt) { return qt == STYX_Q8_0 || qt == STYX_Q4_K || qt == STYX_Q5_K || qt == STYX_Q6_K; }
int blk_elems(int qt) { return qt == STYX_Q8_0 ? 32 : 256; }
int blk_bytes(int qt) {
    return qt == STYX_Q8_0 ? 34 : qt == STYX_Q4_K ? 144 : qt == STYX_Q5_K ? 176 : qt == STYX_Q6_K ? 210 : 0;
}
// bytes of one row of ncols elements, 0 if not representable
long long row_bytes(int qt, int ncols) {
    if (!qtype_ok(qt) || ncols <= 0 || ncols % blk_elems(qt)) return 0;
    return static_cast<long long>(ncols / blk_elems(qt)) * blk_bytes(qt);
}
// 64-element units (qdot.cuh) need ncols % 64 == 0 (q8_0) / % 256 (k-quants)
bool units_ok(int qt, int ncols) { return ncols > 0 && ncols % (qt == STYX_Q8_0 ? 64 : 256) == 0; }
int pow2ceil(int v) {
    int p = 1;
    while (p < v) p <<= 1;
    return p;
}
bool al16(const void *p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

// [p, p+bytes) inside the device allocation that holds p.  Pointers the
// driver does not know as device allocations (mapped host memory) pass:
// their extent cannot be queried here.
// (The driver function is looked up through the runtime, so the library has
// no link-time dependency on libcuda.)
using MemRangeFn = CUresult (*)(CUdeviceptr *, size_t *, CUdeviceptr);
MemRangeFn mem_range_fn() {
    static MemRangeFn fn = [] {
        void *f = nullptr;
        cudaDriverEntryPointQueryResult q{};
        if (cudaGetDriverEntryPoint("cuMemGetAddressRange", &f, cudaEnableDefault, &q) != cudaSuccess ||
            q != cudaDriverEntryPointSuccess) {
            cudaGetLastError();
            f = nullptr;
        }
        return reinterpret_cast<MemRangeFn>(f);
    }();
    return fn;
}

bool extent_ok(const void *p, uint64_t bytes) {
    if (!p || bytes == 0) return true;
    MemRangeFn fn = mem_range_fn();
    if (!fn) return true;
    CUdeviceptr base = 0;
    size_t size = 0;
    if (fn(&base, &size, reinterpret_cast<CUdeviceptr>(p)) != CUDA_SUCCESS) return true;
    return reinterpret_cast<uintptr_t>(p) + bytes <= static_cast<uintptr_t>(base) + size;
}
size_t a16(size_t v) { return (v + 15) & ~size_t(15); }
size_t a128(size_t v) { return (v + 127) & ~size_t(127); }

constexpr size_t kTraceCtas = 256;   // phase stamps: styx::kTraceStamps per CTA

// The counter block (512 B): word 0 is the three-kernel route's hand-off
// counter (zero between launches); the single kernels' 64-bit launch counter
// sits at kGenOffset, and their per-slot h-arrival counters in a region of
// their own (one 128-byte line each); both are never reset except by
// styx_moe_workspace_init (which also clears the tagged words they guard).
constexpr size_t kGenOffset = 128;
struct WsLayout {
    size_t counter, hcnt, xnorm, xd1, xd2, xd3, xscale, logits, weights, h, g, u, d, lgslot, xslot, ccnt, trace, total;
};

WsLayout ws_layout(const styx_moe_dims &d) {
    WsLayout L{};
    size_t o = 0;
    auto take = [&](size_t n) {
        size_t r = o;
        o = (o + n + 255) & ~size_t(255);
        return r;
    };
    const size_t H = d.n_embd, E = d.n_expert, kF = static_cast<size_t>(d.n_expert_used) * d.n_ff;
    L.counter = take(512);
    L.hcnt = take(16 * styx::kHcStride * 8);   // per-slot h counters, one 128-byte line each
    L.xnorm = take(H * 4);
    L.xd1 = take(H);
    L.xd2 = take(H);
    L.xd3 = take(H);
    L.xscale = take(H / 32 * 4);
    L.logits = take(E * 4);
    L.weights = take(16 * 4);
    L.h = take(kF * 4);
    L.g = take(kF * 4);   // gate / up outputs of the mul_mat_vec_id forms
    L.u = take(kF * 4);
    L.d = take(static_cast<size_t>(d.n_expert_used) * H * 4);   // down outputs of the host-read form
    L.lgslot = take(2 * E * 8);   // two banks of logit words, by launch-tag parity
    L.xslot = take(H * 8);        // x rows passed from one layer to the next
    L.ccnt = take(styx::kClusterMaxC * styx::kCntStride * 4);   // cluster form: row-block counters
    L.trace = take(kTraceCtas * styx::kTraceStamps * 8);
    L.total = o;
    return L;
}

int check_dims(const styx_moe_dims *d) {
    NEED(d, "null dims");
    NEED(d->n_embd > 0 && d->n_embd % 256 == 0 && d->n_embd <= 16384, "n_embd %d: need a multiple of 256, <= 16384",
         d->n_embd);
    NEED(d->n_ff > 0 && d->n_ff % 256 == 0 && d->n_ff <= 2048, "n_ff %d: need a multiple of 256, <= 2048",
         d->n_ff);
    NEED(d->n_expert > 0 && d->n_expert <= STYX_MAX_EXPERTS, "n_expert %d out of range", d->n_expert);
    NEED(d->n_expert_used > 0 && d->n_expert_used <= STYX_MAX_TOPK && d->n_expert_used <= d->n_expert,
         "n_expert_used %d out of range", d->n_expert_used);
    return STYX_OK;
}

int check_tensor(const styx_expert_tensor &t, const char *what, int nrows, int ncols, int n_expert) {
    NEED(qtype_ok(t.qtype), "%s: unsupported qtype %d", what, t.qtype);
    NEED(!t.hot || t.n_hot > 0, "%s: hot buffer with n_hot = 0", what);
    NEED(!t.arena || t.n_arena > 0, "%s: arena with n_arena = 0", what);
    NEED(extent_ok(t.full, t.slab_bytes * static_cast<uint64_t>(n_expert)), "%s: full tensor smaller than %d slabs",
         what, n_expert);
    NEED(extent_ok(t.hot, t.slab_bytes * t.n_hot), "%s: hot buffer smaller than n_hot slabs", what);
    NEED(extent_ok(t.arena, t.arena_slab_bytes * t.n_arena), "%s: arena smaller than n_arena slots", what);
    NEED(units_ok(t.qtype, ncols), "%s: %d columns not supported for qtype %d", what, ncols, t.qtype);
    const long long need = row_bytes(t.qtype, ncols) * nrows;
    NEED(static_cast<long long>(t.slab_bytes) >= need, "%s: slab_bytes %llu < %lld", what,
         (unsigned long long)t.slab_bytes, need);
    NEED(t.full || t.hot || t.arena, "%s: no source buffer", what);
    NEED(t.slab_bytes % 16 == 0, "%s: slab_bytes must be a multiple of 16", what);
    NEED(t.arena_slab_bytes % 16 == 0, "%s: arena_slab_bytes must be a multiple of 16", what);
    NEED(al16(t.full) && al16(t.hot) && al16(t.arena), "%s: buffers must be 16-byte aligned", what);
    if (t.full) {
        cudaPointerAttributes pa{};
        if (cudaPointerGetAttributes(&pa, t.full) == cudaSuccess) {
            // device memory, or pinned host memory mapped at the same address
            // (the cold tier: read in place over the host link)
            NEED(pa.type == cudaMemoryTypeDevice || pa.type == cudaMemoryTypeManaged ||
                     (pa.type == cudaMemoryTypeHost && pa.devicePointer == t.full),
                 "%s: full tensor must be device memory or STYX_MEM_HOST memory", what);
        } else {
            cudaGetLastError();
        }
    }
    for (const void *b : {t.hot, t.arena}) {
        cudaPointerAttributes pa{};
        if (b && cudaPointerGetAttributes(&pa, b) == cudaSuccess)
            NEED(pa.type == cudaMemoryTypeDevice || pa.type == cudaMemoryTypeManaged,
                 "%s: hot buffer and arena must be device memory", what);
        else if (b)
            cudaGetLastError();
    }
    return STYX_OK;
}

// full tensor held in pinned host memory (the cold tier)
bool full_in_host(const styx_expert_tensor &t) {
    if (!t.full) return false;
    cudaPointerAttributes pa{};
    if (cudaPointerGetAttributes(&pa, t.full) != cudaSuccess) {
        cudaGetLastError();
        return false;
    }
    return pa.type == cudaMemoryTypeHost;
}

styx::ExpSrc to_src(const styx_expert_tensor &t, int n_expert) {
    return styx::ExpSrc{static_cast<const uint8_t *>(t.full),
                        static_cast<const uint8_t *>(t.hot),
                        static_cast<const uint8_t *>(t.arena),
                        t.slab_bytes,
                        t.arena_slab_bytes,
                        static_cast<uint32_t>(n_expert),
                        t.n_hot,
                        t.n_arena};
}

// rows per CTA of k_matvec_id: about two CTAs per SM over all slots, a whole
// number of the kernel's passes
int mv_rows_per_cta(int nrows, int n_ids, int gs, int sms) {
    const int step = styx::kMvRowStep(gs);
    const long long want = (static_cast<long long>(nrows) * n_ids + 2LL * sms - 1) / (2LL * sms);
    return static_cast<int>(std::max<long long>(step, (want + step - 1) / step * step));
}

// reference-shaped 3-way expert GEMV (rec_matvec_id, moe.rs:1649-1700): hot,
// arena and full-tensor rows in one launch, each slot reading from the last
// of its three sources whose id is set and in range -- the output the
// reference's three SKIP-gated dispatches, in that order, leave
int matvec_id_3way(const styx_expert_tensor &t, int n_expert, const int32_t *ids64, int nrows, int ncols, int k,
                   const float *x, int ne11, float *y, int *err, int sms, cudaStream_t st) {
    const int units = ncols / 64;
    styx::MatVecIdArgs a{};
    a.err = err;
    a.nrows = nrows;
    a.ncols = ncols;
    a.rb = static_cast<int>(row_bytes(t.qtype, ncols));
    a.n_ids = k;
    a.x = x;
    a.stride_b = ncols;
    a.ne11 = ne11;
    a.y = y;
    a.stride_d = nrows;
    a.units = units;
    a.gs = std::min(32, pow2ceil(units));
    a.rows_per_cta = mv_rows_per_cta(nrows, k, a.gs, sms);
    a.src3[0] = static_cast<const uint8_t *>(t.hot);
    a.src3[1] = static_cast<const uint8_t *>(t.arena);
    a.src3[2] = static_cast<const uint8_t *>(t.full);
    a.stride3[0] = t.slab_bytes;
    a.stride3[1] = t.arena_slab_bytes;
    a.stride3[2] = t.slab_bytes;
    a.count3[0] = static_cast<int>(t.n_hot);
    a.count3[1] = static_cast<int>(t.n_arena);
    a.count3[2] = n_expert;
    a.ids = ids64;
    if (!t.hot && !t.arena && !t.full) return STYX_OK;
    CK(styx::launch_matvec_id(a, t.qtype, st));
    return STYX_OK;
}

}  // namespace

// error reporting for the library's other translation units
int styx::set_error(int code, const char *msg) {
    g_err = msg;
    return code;
}

// Scratch of styx_moe_block_noalloc: one statically sized array per device
// (module global memory, zero at module load), shared by every call on that
// device.  Its address is looked up once per device with the device current,
// and forgotten when the last context on that device is destroyed (so a
// context made after a device reset looks it up again).
static __device__ __align__(256) uint8_t g_noalloc_scratch[STYX_NOALLOC_SCRATCH_BYTES];

namespace {
constexpr int kMaxDevices = 64;
std::mutex g_noalloc_mu;
void *g_noalloc_ptr[kMaxDevices] = {};
int g_noalloc_ctxs[kMaxDevices] = {};

void noalloc_ctx_made(int device) {
    std::lock_guard<std::mutex> lock(g_noalloc_mu);
    if (device >= 0 && device < kMaxDevices) g_noalloc_ctxs[device]++;
}
void noalloc_ctx_gone(int device) {
    std::lock_guard<std::mutex> lock(g_noalloc_mu);
    if (device >= 0 && device < kMaxDevices && --g_noalloc_ctxs[device] <= 0) {
        g_noalloc_ctxs[device] = 0;
        g_noalloc_ptr[device] = nullptr;
    }
}

// first call on a device: resolve the symbol's device address (the array's
// name in host code is only a host-side stand-in)
int noalloc_scratch(styx_ctx *ctx, cudaStream_t st, void **out) {
    std::lock_guard<std::mutex> lock(g_noalloc_mu);
    NEED(ctx->device >= 0 && ctx->device < kMaxDevices, "device %d out of range", ctx->device);
    void *&p = g_noalloc_ptr[ctx->device];
    if (!p) {
        cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
        CK(cudaStreamIsCapturing(st, &cs));
        NEED(cs == cudaStreamCaptureStatusNone,
             "styx_moe_block_noalloc: the first call on a device sets up its scratch and must not be "
             "made while the stream is being captured");
        void *q = nullptr;
        CK(cudaGetSymbolAddress(&q, g_noalloc_scratch));
        p = q;
    }
    *out = p;
    return STYX_OK;
}
}  // namespace

extern "C" {

const char *styx_last_error(void) { return g_err.c_str(); }


int styx_init(int device, styx_ctx **out) {
    NEED(out, "null out");
    int n = 0;
    CK(cudaGetDeviceCount(&n));
    NEED(device >= 0 && device < n, "device %d not present (%d devices)", device, n);
    CK(cudaSetDevice(device));
    cudaDeviceProp prop{};
    CK(cudaGetDeviceProperties(&prop, device));
    if (prop.major < 10)
        return fail(STYX_EUNSUPPORTED, "device %d (%s) is sm_%d%d; this library is built for sm_100a", device,
                    prop.name, prop.major, prop.minor);
    auto *c = new styx_ctx();
    c->device = device;
    c->sm_count = prop.multiProcessorCount;
    snprintf(c->name, sizeof(c->name), "%s", prop.name);
    cudaError_t e = cudaMalloc(&c->d_err, 8 * sizeof(int));
    if (e == cudaSuccess) e = cudaMemset(c->d_err, 0, 8 * sizeof(int));
    if (e == cudaSuccess) e = cudaMalloc(&c->d_scratch, kScratchBytes);
    if (e == cudaSuccess) e = cudaMemset(c->d_scratch, 0, kScratchBytes);
    if (e == cudaSuccess) {
        int32_t ids[64];
        for (int i = 0; i < 64; i++) ids[i] = (i >= 16 && i < 48) ? -1 : 0;   // hot / arena SKIP, full row 0
        const float one = 1.0f;
        e = cudaMemcpy(static_cast<uint8_t *>(c->d_scratch) + kScratchDenseIds, ids, sizeof(ids),
                       cudaMemcpyHostToDevice);
        if (e == cudaSuccess)
            e = cudaMemcpy(static_cast<uint8_t *>(c->d_scratch) + kScratchOne, &one, 4, cudaMemcpyHostToDevice);
    }
    if (e != cudaSuccess) {
        cudaFree(c->d_err);
        cudaFree(c->d_scratch);
        delete c;
        return fail(STYX_ECUDA, "error word / scratch: %s", cudaGetErrorString(e));
    }
    noalloc_ctx_made(device);
    *out = c;
    return STYX_OK;
}

void styx_destroy(styx_ctx *ctx) {
    if (!ctx) return;
    cudaSetDevice(ctx->device);
    cudaFree(ctx->d_err);
    cudaFree(ctx->d_scratch);
    noalloc_ctx_gone(ctx->device);
    delete ctx;
}

int styx_vram_bytes(styx_ctx *ctx, uint64_t *out) {
    ENTER(ctx);
    NEED(out, "null out");
    size_t fr = 0, tot = 0;
    CK(cudaMemGetInfo(&fr, &tot));
    *out = tot;
    return STYX_OK;
}

int styx_device_info(styx_ctx *ctx, int *sm_count, char *name, int name_len) {
    NEED(ctx, "null ctx");
    if (sm_count) *sm_count = ctx->sm_count;
    if (name && name_len > 0) snprintf(name, static_cast<size_t>(name_len), "%s", ctx->name);
    return STYX_OK;
}

int styx_check_device_error(styx_ctx *ctx, styx_stream stream) {
    ENTER(ctx);
    int h = 0;
    CK(cudaMemcpyAsync(&h, ctx->d_err, sizeof(int), cudaMemcpyDeviceToHost, S(stream)));
    CK(cudaStreamSynchronize(S(stream)));
    if (h) {
        CK(cudaMemsetAsync(ctx->d_err, 0, sizeof(int), S(stream)));
        CK(cudaStreamSynchronize(S(stream)));
        if (h == 4) return fail(STYX_EINVAL, "a kernel skipped an out-of-range expert id / hot index / arena slot");
        if (h == 5) return fail(STYX_EINVAL, "a kernel skipped a KV cache row outside [0, n_ctx)");
        if (h == 6) return fail(STYX_ETIMEOUT, "expert parallelism: a peer rank's rows did not arrive (bounded wait gave up)");
        return fail(STYX_ETIMEOUT, "device-side bounded wait gave up (code %d)", h);
    }
    return STYX_OK;
}

int styx_set_option(styx_ctx *ctx, int option, int64_t value) {
    NEED(ctx, "null ctx");
    switch (option) {
    case STYX_OPT_MOE_KERNELS:
        NEED(value >= 0 && value <= 3, "STYX_OPT_MOE_KERNELS: 0, 1, 2 or 3");
        ctx->moe_kernels = static_cast<int>(value);
        return STYX_OK;
    case STYX_OPT_TRACE:
        ctx->trace = value ? 1 : 0;
        return STYX_OK;
    case STYX_OPT_MOE_LAYERS:
        NEED(value >= 0 && value <= 2, "STYX_OPT_MOE_LAYERS: 0, 1 or 2");
        ctx->moe_layers = static_cast<int>(value);
        return STYX_OK;
    case STYX_OPT_EXCLUSIVE:
        ctx->exclusive = value ? 1 : 0;
        return STYX_OK;
    case STYX_OPT_ATTN_KERNELS:
        NEED(value >= 0 && value <= 3, "STYX_OPT_ATTN_KERNELS: 0, 1, 2 or 3");
        ctx->attn_kernels = static_cast<int>(value);
        return STYX_OK;
    default: return fail(STYX_EINVAL, "unknown or read-only option %d", option);
    }
}

int styx_get_option(styx_ctx *ctx, int option, int64_t *value) {
    NEED(ctx && value, "null pointer");
    switch (option) {
    case STYX_OPT_MOE_KERNELS: *value = ctx->moe_kernels; return STYX_OK;
    case STYX_OPT_MOE_LAST_PATH: *value = ctx->last_path; return STYX_OK;
    case STYX_OPT_TRACE: *value = ctx->trace; return STYX_OK;
    case STYX_OPT_MOE_LAYERS: *value = ctx->moe_layers; return STYX_OK;
    case STYX_OPT_EXCLUSIVE: *value = ctx->exclusive; return STYX_OK;
    case STYX_OPT_ATTN_KERNELS: *value = ctx->attn_kernels; return STYX_OK;
    case STYX_OPT_ATTN_LAST_PATH: *value = ctx->attn_last_path; return STYX_OK;
    case STYX_OPT_MOE_LAST_CLUSTER: *value = ctx->last_cluster; return STYX_OK;
    default: return fail(STYX_EINVAL, "unknown option %d", option);
    }
}

int styx_alloc(styx_ctx *ctx, uint64_t bytes, int kind, void **out) {
    ENTER(ctx);
    NEED(out, "null out");
    NEED(bytes > 0, "zero-byte allocation");
    void *p = nullptr;
    cudaError_t e;
    if (kind == STYX_MEM_DEVICE) e = cudaMalloc(&p, bytes);
    else if (kind == STYX_MEM_HOST) e = cudaHostAlloc(&p, bytes, cudaHostAllocMapped | cudaHostAllocPortable);
    else return fail(STYX_EINVAL, "unknown memory kind %d", kind);
    if (e != cudaSuccess) {
        cudaGetLastError();
        return fail(STYX_ENOMEM, "allocating %llu bytes (kind %d): %s", (unsigned long long)bytes, kind,
                    cudaGetErrorString(e));
    }
    if (kind == STYX_MEM_HOST) {
        // kernels read the GTT tier through the host address (UVA)
        void *dp = nullptr;
        if (cudaHostGetDevicePointer(&dp, p, 0) != cudaSuccess || dp != p) {
            cudaGetLastError();
            cudaFreeHost(p);
            return fail(STYX_EUNSUPPORTED, "pinned host memory is not mapped at its host address");
        }
    }
    *out = p;
    return STYX_OK;
}

int styx_free(styx_ctx *ctx, void *ptr) {
    ENTER(ctx);
    if (!ptr) return STYX_OK;
    cudaPointerAttributes pa{};
    CK(cudaPointerGetAttributes(&pa, ptr));
    if (pa.type == cudaMemoryTypeHost) CK(cudaFreeHost(ptr));
    else CK(cudaFree(ptr));
    return STYX_OK;
}

int styx_upload(styx_ctx *ctx, void *dst, uint64_t dst_off, const void *src, uint64_t n, styx_stream stream) {
    ENTER(ctx);
    NEED(dst && src, "null pointer");
    CK(cudaMemcpyAsync(static_cast<uint8_t *>(dst) + dst_off, src, n, cudaMemcpyDefault, S(stream)));
    return STYX_OK;
}

int styx_download(styx_ctx *ctx, void *dst, const void *src, uint64_t src_off, uint64_t n, styx_stream stream) {
    ENTER(ctx);
    NEED(dst && src, "null pointer");
    CK(cudaMemcpyAsync(dst, static_cast<const uint8_t *>(src) + src_off, n, cudaMemcpyDefault, S(stream)));
    CK(cudaStreamSynchronize(S(stream)));
    return STYX_OK;
}

int styx_copy(styx_ctx *ctx, const void *src, uint64_t src_off, void *dst, uint64_t dst_off, uint64_t n,
              styx_stream stream) {
    ENTER(ctx);
    NEED(dst && src, "null pointer");
    CK(cudaMemcpyAsync(static_cast<uint8_t *>(dst) + dst_off, static_cast<const uint8_t *>(src) + src_off, n,
                       cudaMemcpyDefault, S(stream)));
    return STYX_OK;
}

int styx_memset(styx_ctx *ctx, void *dst, int value, uint64_t n, styx_stream stream) {
    ENTER(ctx);
    NEED(dst, "null pointer");
    CK(cudaMemsetAsync(dst, value, n, S(stream)));
    return STYX_OK;
}

int styx_stream_create(styx_ctx *ctx, styx_stream *out) {
    ENTER(ctx);
    NEED(out, "null out");
    cudaStream_t s;
    CK(cudaStreamCreateWithFlags(&s, cudaStreamNonBlocking));
    *out = s;
    return STYX_OK;
}
int styx_stream_destroy(styx_ctx *ctx, styx_stream stream) {
    ENTER(ctx);
    if (stream) CK(cudaStreamDestroy(S(stream)));
    return STYX_OK;
}
int styx_stream_sync(styx_ctx *ctx, styx_stream stream) {
    ENTER(ctx);
    CK(cudaStreamSynchronize(S(stream)));
    return STYX_OK;
}
int styx_event_create(styx_ctx *ctx, styx_event *out) {
    ENTER(ctx);
    NEED(out, "null out");
    cudaEvent_t e;
    CK(cudaEventCreateWithFlags(&e, cudaEventDisableTiming));
    *out = e;
    return STYX_OK;
}
int styx_event_destroy(styx_ctx *ctx, styx_event ev) {
    ENTER(ctx);
    if (ev) CK(cudaEventDestroy(static_cast<cudaEvent_t>(ev)));
    return STYX_OK;
}
int styx_event_record(styx_ctx *ctx, styx_event ev, styx_stream stream) {
    ENTER(ctx);
    CK(cudaEventRecord(static_cast<cudaEvent_t>(ev), S(stream)));
    return STYX_OK;
}
int styx_stream_wait_event(styx_ctx *ctx, styx_stream stream, styx_event ev) {
    ENTER(ctx);
    CK(cudaStreamWaitEvent(S(stream), static_cast<cudaEvent_t>(ev), 0));
    return STYX_OK;
}

int styx_graph_begin(styx_ctx *ctx, styx_stream stream) {
    ENTER(ctx);
    NEED(stream, "graph recording needs a non-default stream");
    CK(cudaStreamBeginCapture(S(stream), cudaStreamCaptureModeThreadLocal));
    return STYX_OK;
}

int styx_graph_end(styx_ctx *ctx, styx_stream stream, styx_graph *out) {
    ENTER(ctx);
    NEED(stream && out, "null stream / out");
    cudaGraph_t g = nullptr;
    CK(cudaStreamEndCapture(S(stream), &g));
    cudaGraphExec_t ex = nullptr;
    cudaError_t e = cudaGraphInstantiate(&ex, g, 0);
    cudaGraphDestroy(g);
    if (e != cudaSuccess) return fail(STYX_ECUDA, "cudaGraphInstantiate: %s", cudaGetErrorString(e));
    *out = ex;
    return STYX_OK;
}

int styx_graph_launch(styx_ctx *ctx, styx_graph graph, styx_stream stream) {
    ENTER(ctx);
    NEED(graph, "null graph");
    CK(cudaGraphLaunch(static_cast<cudaGraphExec_t>(graph), S(stream)));
    return STYX_OK;
}

int styx_graph_destroy(styx_ctx *ctx, styx_graph graph) {
    ENTER(ctx);
    if (graph) CK(cudaGraphExecDestroy(static_cast<cudaGraphExec_t>(graph)));
    return STYX_OK;
}

// ------------------------------------------------------------ single ops
int styx_rms_norm(styx_ctx *ctx, styx_stream stream, const float *x, const float *w, float eps, int ncols,
                  int nrows, float *out) {
    ENTER(ctx);
    NEED(x && out && ncols > 0 && nrows > 0, "bad rms_norm arguments");
    CK(styx::launch_rms_norm(x, w, eps, ncols, nrows, out, S(stream)));
    return STYX_OK;
}

int styx_matvec_f32(styx_ctx *ctx, styx_stream stream, const float *a, int nrows, int ncols, int stride_a,
                    const float *x, float *d) {
    ENTER(ctx);
    NEED(a && x && d && nrows > 0 && ncols > 0 && stride_a >= ncols, "bad matvec_f32 arguments");
    CK(styx::launch_matvec_f32(a, nrows, ncols, stride_a, x, d, S(stream)));
    return STYX_OK;
}

int styx_topk_softmax(styx_ctx *ctx, styx_stream stream, const float *logits, int n, int k, int renorm,
                      const uint32_t *remap, const uint32_t *pmap, float *weights, int32_t *ids64) {
    ENTER(ctx);
    NEED(logits && weights && ids64, "null pointer");
    NEED(n > 0 && n <= STYX_MAX_EXPERTS, "n %d out of range", n);
    NEED(k > 0 && k <= STYX_MAX_TOPK && k <= n, "k %d out of range", k);
    CK(styx::launch_topk(logits, n, k, renorm, remap, pmap, weights, ids64, S(stream)));
    return STYX_OK;
}

int styx_mul_mat_vec_id(styx_ctx *ctx, styx_stream stream, int qtype, const void *a, uint64_t expert_bytes,
                        int n_expert, int nrows, int ncols, const int32_t *ids, int n_ids, const float *x,
                        int stride_b, int ne11, float *y, int stride_d) {
    ENTER(ctx);
    NEED(a && ids && x && y, "null pointer");
    NEED(qtype_ok(qtype), "unsupported qtype %d", qtype);
    NEED(units_ok(qtype, ncols), "ncols %d not supported for qtype %d", ncols, qtype);
    NEED(nrows > 0 && n_ids > 0 && ne11 > 0 && stride_b >= ncols && stride_d >= nrows && n_expert > 0, "bad shape");
    NEED(ncols <= 65536, "ncols too large");
    const long long rb = row_bytes(qtype, ncols);
    NEED(expert_bytes >= static_cast<uint64_t>(rb) * nrows, "expert_bytes smaller than nrows rows");
    if (qtype == STYX_Q4_K || qtype == STYX_Q5_K)
        NEED(al16(a) && expert_bytes % 16 == 0 && rb % 16 == 0, "q4_K/q5_K matrices must be 16-byte aligned");
    else
        NEED((reinterpret_cast<uintptr_t>(a) & 1) == 0 && expert_bytes % 2 == 0, "matrix must be 2-byte aligned");
    NEED(extent_ok(a, expert_bytes * static_cast<uint64_t>(n_expert)), "matrix buffer smaller than n_expert experts");
    NEED(extent_ok(y, (static_cast<uint64_t>(n_ids - 1) * stride_d + nrows) * 4), "y buffer too small");
    NEED(extent_ok(x, (static_cast<uint64_t>(std::min(ne11, n_ids) - 1) * stride_b + ncols) * 4), "x buffer too small");
    styx::MatVecIdArgs m{};
    m.a = static_cast<const uint8_t *>(a);
    m.expert_bytes = expert_bytes;
    m.n_expert = n_expert;
    m.err = ctx->d_err;
    m.nrows = nrows;
    m.ncols = ncols;
    m.rb = static_cast<int>(rb);
    m.ids = ids;
    m.n_ids = n_ids;
    m.x = x;
    m.stride_b = stride_b;
    m.ne11 = ne11;
    m.y = y;
    m.stride_d = stride_d;
    m.units = ncols / 64;
    m.gs = std::min(32, pow2ceil(m.units));
    m.rows_per_cta = mv_rows_per_cta(nrows, n_ids, m.gs, ctx->sm_count);
    CK(styx::launch_matvec_id(m, qtype, S(stream)));
    return STYX_OK;
}

int styx_swiglu(styx_ctx *ctx, styx_stream stream, const float *g, const float *u, float *out, int n) {
    ENTER(ctx);
    NEED(g && u && out && n > 0, "bad swiglu arguments");
    CK(styx::launch_swiglu(g, u, out, n, S(stream)));
    return STYX_OK;
}

int styx_moe_reduce(styx_ctx *ctx, styx_stream stream, const float *d, const float *w, float *x, int ne, int k) {
    ENTER(ctx);
    NEED(d && w && x && ne > 0 && k > 0, "bad moe_reduce arguments");
    CK(styx::launch_moe_reduce(d, w, x, ne, k, S(stream)));
    return STYX_OK;
}

// true if a kernel may dereference p: device/managed memory, or pinned host
// memory mapped at the same address (UVA)
static bool device_readable(const void *p) {
    cudaPointerAttributes pa{};
    if (cudaPointerGetAttributes(&pa, p) != cudaSuccess) {
        cudaGetLastError();
        return false;
    }
    if (pa.type == cudaMemoryTypeDevice || pa.type == cudaMemoryTypeManaged) return true;
    return pa.type == cudaMemoryTypeHost && pa.devicePointer == p;
}

static bool is_device_mem(const void *p) {
    cudaPointerAttributes pa{};
    if (cudaPointerGetAttributes(&pa, p) != cudaSuccess) {
        cudaGetLastError();
        return false;
    }
    return pa.type == cudaMemoryTypeDevice || pa.type == cudaMemoryTypeManaged;
}

static int gather_check(const void *sg, const void *su, const void *sd, uint64_t bg, uint64_t bu, uint64_t bd,
                        void *ag, void *au, void *ad, uint64_t dg, uint64_t du, uint64_t dd, int n_expert, int layer,
                        int k) {
    NEED(sg && su && sd && ag && au && ad, "null pointer");
    NEED(n_expert > 0 && layer >= 0, "bad n_expert / layer");
    const uint64_t ne = static_cast<uint64_t>(n_expert), slots = (static_cast<uint64_t>(layer) + 1) * k;
    NEED(extent_ok(sg, bg * ne) && extent_ok(su, bu * ne) && extent_ok(sd, bd * ne),
         "a source tensor is smaller than n_expert slabs");
    NEED(extent_ok(ag, dg * slots) && extent_ok(au, du * slots) && extent_ok(ad, dd * slots),
         "an arena is smaller than (layer+1)*k slots");
    NEED(device_readable(sg) && device_readable(su) && device_readable(sd),
         "gather sources must be device memory or mapped pinned host memory (STYX_MEM_HOST)");
    NEED(is_device_mem(ag) && is_device_mem(au) && is_device_mem(ad), "arenas must be device memory");
    NEED(bg % 16 == 0 && bu % 16 == 0 && bd % 16 == 0 && dg % 16 == 0 && du % 16 == 0 && dd % 16 == 0,
         "slab sizes must be multiples of 16 bytes");
    NEED(bg <= dg && bu <= du && bd <= dd, "arena slot smaller than the source slab");
    NEED(al16(sg) && al16(su) && al16(sd) && al16(ag) && al16(au) && al16(ad), "buffers must be 16-byte aligned");
    NEED(k > 0 && k <= STYX_MAX_TOPK, "k %d out of range", k);
    return STYX_OK;
}

int styx_gather_slabs(styx_ctx *ctx, styx_stream stream, const void *src_g, const void *src_u, const void *src_d,
                      uint64_t src_bytes_g, uint64_t src_bytes_u, uint64_t src_bytes_d, void *arena_g,
                      void *arena_u, void *arena_d, uint64_t dst_bytes_g, uint64_t dst_bytes_u,
                      uint64_t dst_bytes_d, const int32_t *ids, int n_expert, int layer, int k) {
    ENTER(ctx);
    int rc = gather_check(src_g, src_u, src_d, src_bytes_g, src_bytes_u, src_bytes_d, arena_g, arena_u, arena_d,
                          dst_bytes_g, dst_bytes_u, dst_bytes_d, n_expert, layer, k);
    if (rc) return rc;
    NEED(ids, "null ids");
    styx::GatherArgs a{};
    a.n_expert = n_expert;
    a.err = ctx->d_err;
    a.src[0] = static_cast<const uint8_t *>(src_g);
    a.src[1] = static_cast<const uint8_t *>(src_u);
    a.src[2] = static_cast<const uint8_t *>(src_d);
    a.src_bytes[0] = src_bytes_g;
    a.src_bytes[1] = src_bytes_u;
    a.src_bytes[2] = src_bytes_d;
    a.dst[0] = static_cast<uint8_t *>(arena_g);
    a.dst[1] = static_cast<uint8_t *>(arena_u);
    a.dst[2] = static_cast<uint8_t *>(arena_d);
    a.dst_bytes[0] = dst_bytes_g;
    a.dst_bytes[1] = dst_bytes_u;
    a.dst_bytes[2] = dst_bytes_d;
    a.ids = ids;
    a.layer = layer;
    a.k = k;
    CK(styx::launch_gather(a, S(stream)));
    return STYX_OK;
}

int styx_gather_slabs_async(styx_ctx *ctx, styx_stream stream, const void *src_g, const void *src_u,
                            const void *src_d, uint64_t src_bytes_g, uint64_t src_bytes_u, uint64_t src_bytes_d,
                            void *arena_g, void *arena_u, void *arena_d, uint64_t dst_bytes_g,
                            uint64_t dst_bytes_u, uint64_t dst_bytes_d, const int32_t *host_ids, int n_expert,
                            int layer, int k) {
    ENTER(ctx);
    int rc = gather_check(src_g, src_u, src_d, src_bytes_g, src_bytes_u, src_bytes_d, arena_g, arena_u, arena_d,
                          dst_bytes_g, dst_bytes_u, dst_bytes_d, n_expert, layer, k);
    if (rc) return rc;
    NEED(host_ids, "null ids");
    for (int s = 0; s < k; s++)
        NEED(static_cast<uint32_t>(host_ids[s]) == STYX_SKIP || (host_ids[s] >= 0 && host_ids[s] < n_expert),
             "id %d of slot %d out of range", host_ids[s], s);
    const void *src[3] = {src_g, src_u, src_d};
    void *dst[3] = {arena_g, arena_u, arena_d};
    const uint64_t sb[3] = {src_bytes_g, src_bytes_u, src_bytes_d}, db[3] = {dst_bytes_g, dst_bytes_u, dst_bytes_d};
    for (int s = 0; s < k; s++) {
        const uint32_t e = static_cast<uint32_t>(host_ids[s]);
        if (e == STYX_SKIP) continue;
        const uint64_t slot = static_cast<uint64_t>(layer) * k + s;
        for (int t = 0; t < 3; t++)
            CK(cudaMemcpyAsync(static_cast<uint8_t *>(dst[t]) + slot * db[t],
                               static_cast<const uint8_t *>(src[t]) + e * sb[t], sb[t], cudaMemcpyDefault,
                               S(stream)));
    }
    return STYX_OK;
}

// ---------------------------------------------------------- MoE block
int styx_moe_workspace_bytes(const styx_moe_dims *dims, uint64_t *out) {
    int rc = check_dims(dims);
    if (rc) return rc;
    NEED(out, "null out");
    *out = ws_layout(*dims).total;
    return STYX_OK;
}

int styx_moe_workspace_init(styx_ctx *ctx, styx_stream stream, void *ws, uint64_t bytes) {
    ENTER(ctx);
    NEED(ws, "null workspace");
    CK(cudaMemsetAsync(ws, 0, bytes, S(stream)));
    return STYX_OK;
}

int styx_moe_workspace_view(const styx_moe_dims *dims, void *workspace, int which, void **out) {
    int rc = check_dims(dims);
    if (rc) return rc;
    NEED(workspace && out, "null pointer");
    const WsLayout L = ws_layout(*dims);
    size_t off;
    switch (which) {
    case 0: off = L.xnorm; break;
    case 1: off = L.logits; break;
    case 2: off = L.h; break;
    case 3: off = L.weights; break;
    case 4: off = L.trace; break;
    default: return fail(STYX_EINVAL, "unknown view %d", which);
    }
    *out = static_cast<uint8_t *>(workspace) + off;
    return STYX_OK;
}

// The MoE block when some expert tensor's full slabs are in pinned host
// memory (the cold tier of MoeModel::load, moe.rs:856-870): every expert
// matvec is a mul_mat_vec_id dispatch per source row (hot, arena, full), as
// rec_matvec_id records them (moe.rs:1649-1700), reading the host slabs in
// place over the host link with plain loads; then SiLU, the down matvec of
// every slot and moe_reduce.  Slots without an expert keep zeros (weight 0).
static int moe_block_host_read(styx_ctx *ctx, cudaStream_t st, const styx_moe_dims &d, const styx_moe_layer &lw,
                               float *x, int32_t *ids64, float *wts, uint8_t *ws, const WsLayout &L) {
    const int H = d.n_embd, F = d.n_ff, E = d.n_expert, k = d.n_expert_used;
    styx::RouteArgs ra{};
    ra.x = x;
    ra.norm_w = lw.ffn_norm;
    ra.eps = d.rms_eps;
    ra.router = lw.router;
    ra.E = E;
    ra.H = H;
    ra.k = k;
    ra.renorm = d.norm_topk;
    ra.remap = lw.remap;
    ra.pmap = lw.pmap;
    ra.xnorm = reinterpret_cast<float *>(ws + L.xnorm);
    ra.xd1 = reinterpret_cast<int8_t *>(ws + L.xd1);
    ra.xd2 = ws + L.xd2;
    ra.xd3 = ws + L.xd3;
    ra.xscale = reinterpret_cast<float *>(ws + L.xscale);
    ra.logits = reinterpret_cast<float *>(ws + L.logits);
    ra.weights = wts;
    ra.ids64 = ids64;
    ra.counter = reinterpret_cast<unsigned *>(ws + L.counter);
    ra.err = ctx->d_err;
    CK(styx::launch_route(ra, st));
    float *g = reinterpret_cast<float *>(ws + L.g), *u = reinterpret_cast<float *>(ws + L.u);
    float *h = reinterpret_cast<float *>(ws + L.h), *dd = reinterpret_cast<float *>(ws + L.d);
    const size_t kF = static_cast<size_t>(k) * F;
    CK(cudaMemsetAsync(g, 0, kF * 4, st));
    CK(cudaMemsetAsync(u, 0, kF * 4, st));
    CK(cudaMemsetAsync(dd, 0, static_cast<size_t>(k) * H * 4, st));
    int rc;
    if ((rc = matvec_id_3way(lw.gate, E, ids64, F, H, k, ra.xnorm, 1, g, ctx->d_err, ctx->sm_count, st))) return rc;
    if ((rc = matvec_id_3way(lw.up, E, ids64, F, H, k, ra.xnorm, 1, u, ctx->d_err, ctx->sm_count, st))) return rc;
    CK(styx::launch_swiglu(g, u, h, static_cast<int>(kF), st));
    if ((rc = matvec_id_3way(lw.down, E, ids64, H, F, k, h, k, dd, ctx->d_err, ctx->sm_count, st))) return rc;
    CK(styx::launch_moe_reduce(dd, wts, x, H, k, st));
    return STYX_OK;
}

// The three-kernel MoE block (route, gate/up + SiLU, down + combine).  With
// `partial` the down kernel writes w[s]*d[s][r] per slot there instead of
// updating x; `quiet` makes a missing full tensor mean "another device's
// expert" (expert parallelism) rather than an error.
static int moe_block_split(styx_ctx *ctx, cudaStream_t st, const styx_moe_dims &dm, const styx_moe_layer &lwr,
                           float *x, int32_t *ids64, float *wts, uint8_t *ws, const WsLayout &L, float *partial,
                           bool quiet) {
    const styx_moe_dims *dims = &dm;
    const styx_moe_layer *lw = &lwr;
    const int H = dims->n_embd, F = dims->n_ff, E = dims->n_expert, k = dims->n_expert_used;
    int rc = STYX_OK;
    // 1. route
    styx::RouteArgs ra{};
    ra.x = x;
    ra.norm_w = lw->ffn_norm;
    ra.eps = dims->rms_eps;
    ra.router = lw->router;
    ra.E = E;
    ra.H = H;
    ra.k = k;
    ra.renorm = dims->norm_topk;
    ra.remap = lw->remap;
    ra.pmap = lw->pmap;
    ra.xnorm = reinterpret_cast<float *>(ws + L.xnorm);
    ra.xd1 = reinterpret_cast<int8_t *>(ws + L.xd1);
    ra.xd2 = ws + L.xd2;
    ra.xd3 = ws + L.xd3;
    ra.xscale = reinterpret_cast<float *>(ws + L.xscale);
    ra.logits = reinterpret_cast<float *>(ws + L.logits);
    ra.weights = wts;
    ra.ids64 = ids64;
    ra.counter = reinterpret_cast<unsigned *>(ws + L.counter);
    ra.err = ctx->d_err;
    CK(styx::launch_route(ra, st));

    float *h = reinterpret_cast<float *>(ws + L.h);
    const int units_g = H / 64;
    // 2. gate/up + SiLU
    if (lw->gate.qtype == lw->up.qtype && units_g <= 32) {
        styx::GateUpArgs ga{};
        ga.gate = to_src(lw->gate, E);
        ga.up = to_src(lw->up, E);
        ga.ids64 = ids64;
        ga.xd1 = ra.xd1;
        ga.xd2 = ra.xd2;
        ga.xd3 = ra.xd3;
        ga.xscale = ra.xscale;
        ga.h = h;
        ga.H = H;
        ga.F = F;
        ga.k = k;
        ga.rb_g = static_cast<int>(row_bytes(lw->gate.qtype, H));
        ga.rb_u = static_cast<int>(row_bytes(lw->up.qtype, H));
        ga.units = units_g;
        ga.gs = pow2ceil(units_g);
        ga.ch = 8;
        ga.up_off = static_cast<uint32_t>(a16(static_cast<size_t>(ga.ch) * ga.rb_g + 32));
        ga.stage_bytes = ga.up_off + static_cast<uint32_t>(a16(static_cast<size_t>(ga.ch) * ga.rb_u + 32));
        const int T = k * F;
        const int grid = std::max(1, std::min(ctx->sm_count, (T + ga.ch - 1) / ga.ch));
        const int rows_per_cta = (T + grid - 1) / grid;
        const int max_st = static_cast<int>((227 * 1024 - 256) / ga.stage_bytes);
        NEED(max_st >= 2, "gate/up rows too large for shared memory");
        ga.nst = std::max(2, std::min({16, max_st, (rows_per_cta + ga.ch - 1) / ga.ch + 1}));
        ga.quiet = quiet ? 1 : 0;
        ga.err = ctx->d_err;
        CK(styx::launch_gate_up(ga, lw->gate.qtype, grid, st));
    } else {
        float *g = reinterpret_cast<float *>(ws + L.g), *u = reinterpret_cast<float *>(ws + L.u);
        // slots no dispatch writes (another device's experts) must not hold stale values
        if (quiet) {
            CK(cudaMemsetAsync(g, 0, static_cast<size_t>(k) * F * 4, st));
            CK(cudaMemsetAsync(u, 0, static_cast<size_t>(k) * F * 4, st));
        }
        if ((rc = matvec_id_3way(lw->gate, E, ids64, F, H, k, ra.xnorm, 1, g, ctx->d_err, ctx->sm_count, st))) return rc;
        if ((rc = matvec_id_3way(lw->up, E, ids64, F, H, k, ra.xnorm, 1, u, ctx->d_err, ctx->sm_count, st))) return rc;
        CK(styx::launch_swiglu(g, u, h, k * F, st));
    }

    // 3. down + weighted combine into x
    styx::DownArgs da{};
    da.down = to_src(lw->down, E);
    da.ids64 = ids64;
    da.h = h;
    da.w = wts;
    da.x = x;
    da.partial = partial;
    da.quiet = quiet ? 1 : 0;
    da.H = H;
    da.F = F;
    da.k = k;
    da.rb = static_cast<int>(row_bytes(lw->down.qtype, F));
    da.units = F / 64;
    da.gs = pow2ceil(da.units);
    da.rc = 4;
    da.slot_stride = static_cast<uint32_t>(a16(static_cast<size_t>(da.rc) * da.rb + 32));
    da.stage_bytes = da.slot_stride * static_cast<uint32_t>(k);
    const int grid_d = std::max(1, std::min(ctx->sm_count, H / da.rc));
    const int rows_d = (H + grid_d - 1) / grid_d;
    da.dig_off = 512;
    const size_t kF = static_cast<size_t>(k) * F;
    const size_t dig_bytes = kF * 3 + kF / 32 * 4;
    const int chunks = (rows_d + da.rc - 1) / da.rc;
    const size_t fixed = a128(a128(da.dig_off + dig_bytes) + static_cast<size_t>(std::max(2, chunks)) * k * da.rc * 4);
    NEED(fixed < 227 * 1024, "down kernel: k*n_ff too large for shared memory");
    int nst = std::min({16, chunks, static_cast<int>((227 * 1024 - fixed) / da.stage_bytes)});
    NEED(nst >= 1, "down rows too large for shared memory");
    da.nst = nst;
    da.part_off = static_cast<uint32_t>(a128(da.dig_off + dig_bytes));
    da.stage_off = static_cast<uint32_t>(a128(da.part_off + static_cast<size_t>(std::max(2, nst)) * k * da.rc * 4));
    const uint32_t smem_d = da.stage_off + static_cast<uint32_t>(nst) * da.stage_bytes;
    NEED(smem_d <= 227 * 1024, "down kernel needs %u bytes of shared memory", smem_d);
    da.err = ctx->d_err;
    CK(styx::launch_down(da, lw->down.qtype, grid_d, smem_d, st));
    return STYX_OK;
}

constexpr int kGuChunks = 1;   // gate/up chunks per CTA of the single-kernel MoE block

// Shared-memory plan of the single-kernel MoE block for these dims; false if
// it does not fit one CTA per SM (the caller then uses three kernels).
static bool plan_fused(const styx_moe_dims &d, const styx_moe_layer &lw, int sms, styx::FusedArgs &a,
                       uint32_t &smem) {
    const int H = d.n_embd, F = d.n_ff, k = d.n_expert_used;
    const int qg = lw.gate.qtype, qd = lw.down.qtype;
    if (lw.up.qtype != qg || !styx::fused_supported(qg, qd)) return false;
    const int units_g = H / 64, units_d = F / 64;
    if (units_g > 32 || units_d > 32 || k > 16) return false;
    const size_t kLimit = 227 * 1024;
    const int G = sms;
    a.units_g = units_g;
    a.gs_g = pow2ceil(units_g);
    a.units_d = units_d;
    a.gs_d = pow2ceil(units_d);
    a.rb_g = static_cast<int>(row_bytes(qg, H));
    a.rb_u = static_cast<int>(row_bytes(lw.up.qtype, H));
    a.rb_d = static_cast<int>(row_bytes(qd, F));
    // region A: x_norm and its digits, reused for h digits in the down phase;
    // then the E logits (kept until the softmax after the gate/up phase)
    const size_t a_route = static_cast<size_t>(H) * 4 + 3 * static_cast<size_t>(H) + H / 32 * 4;
    const size_t kF = static_cast<size_t>(k) * F;
    const size_t a_down = 3 * kF + kF / 32 * 4;
    // (then the remap / pmap tables, then the logits, at the end of region A)
    const size_t size_a = a128(std::max(a_route, a_down)) + 3 * a128(static_cast<size_t>(d.n_expert) * 4);
    // gate/up: kGuChunks chunks per CTA (each at most two slot segments of
    // gate rows and of up rows); every chunk of the CTA resident.  Fewer,
    // larger chunks issue fewer bulk copies from the one issuing warp
    // (~60 cycles each), and splitting a CTA's rows buys no overlap: every
    // SM's bytes arrive at the HBM rate together.  At the 30B shape, per
    // block: 6 chunks 22.68 us, 4 22.38, 3 22.15, 2 21.97, 1 21.90.
    const int rpw_g = 32 / a.gs_g;
    const long long T = static_cast<long long>(k) * F;
    const int rows_g = static_cast<int>((T + G - 1) / G);
    a.ch = std::max(rpw_g, ((rows_g + kGuChunks - 1) / kGuChunks + rpw_g - 1) / rpw_g * rpw_g);
    const int chunks_g = (rows_g + a.ch - 1) / a.ch;
    if (chunks_g > 16 || a.ch > F) return false;
    a.gu_up_off = static_cast<uint32_t>(a16(static_cast<size_t>(a.ch) * a.rb_g + 96));
    a.gu_stride = a.gu_up_off + static_cast<uint32_t>(a16(static_cast<size_t>(a.ch) * a.rb_u + 96));
    const size_t gu_bytes = static_cast<size_t>(chunks_g) * a.gu_stride;
    // down: all of the CTA's output rows, every slot, one chunk
    const int rows_d = (H + G - 1) / G;
    a.rc = rows_d;
    a.dslot_stride = static_cast<uint32_t>(a16(static_cast<size_t>(a.rc) * a.rb_d + 32));
    a.dstage_bytes = a.dslot_stride * static_cast<uint32_t>(k);
    const size_t part = a128(2 * static_cast<size_t>(k) * a.rc * 4);
    a.off_a = styx::kFusedHeader;
    a.off_part = static_cast<uint32_t>(a.off_a + size_a);
    a.off_ring = static_cast<uint32_t>(a.off_part + part);
    a.off_down = static_cast<uint32_t>(a128(a.off_ring + gu_bytes));
    const size_t total = a.off_down + a.dstage_bytes;
    if (total > kLimit) return false;
    smem = static_cast<uint32_t>(total);
    return true;
}

// The per-layer part of the single kernel's arguments (the plan part comes
// from plan_fused).
static void fill_fused(styx::FusedArgs &fa, const styx_ctx *ctx, const styx_moe_dims &d, const styx_moe_layer &lw,
                       float *x, int32_t *ids64, float *wts, uint8_t *ws, const WsLayout &L) {
    const int E = d.n_expert;
    fa.x = x;
    fa.norm_w = lw.ffn_norm;
    fa.eps = d.rms_eps;
    fa.router = lw.router;
    fa.E = E;
    fa.H = d.n_embd;
    fa.F = d.n_ff;
    fa.k = d.n_expert_used;
    fa.renorm = d.norm_topk;
    fa.remap = lw.remap;
    fa.pmap = lw.pmap;
    fa.gate = to_src(lw.gate, E);
    fa.up = to_src(lw.up, E);
    fa.down = to_src(lw.down, E);
    fa.ids64 = ids64;
    fa.weights = wts;
    fa.logits = reinterpret_cast<float *>(ws + L.logits);
    fa.xnorm = reinterpret_cast<float *>(ws + L.xnorm);
    fa.h = reinterpret_cast<float *>(ws + L.h);
    fa.lgslot = reinterpret_cast<uint64_t *>(ws + L.lgslot);
    fa.gen = reinterpret_cast<unsigned long long *>(ws + L.counter + kGenOffset);
    fa.hcount = reinterpret_cast<unsigned long long *>(ws + L.hcnt);
    fa.err = ctx->d_err;
    fa.trace = ctx->trace ? reinterpret_cast<long long *>(ws + L.trace) : nullptr;
}

// Shared-memory plan of the cluster form for these dims; false if no cluster
// size fits (the caller then takes the single kernel or three kernels).  The
// largest cluster (16 CTAs, else 8, 4, 2, 1) whose per-CTA share of slot s's
// rows fits in shared memory and of which the device holds k at once; with
// `waves`, failing that, the largest that fits at all (its clusters then run
// in waves: correct, but slower than the single kernel).  On B200 at most 7
// clusters of 16 CTAs of ~210 KB are resident at once, so the 30B-A3B layer
// (k 8, whose rows need 16 CTAs per slot) takes the single kernel in auto.
static bool plan_cluster(const styx_moe_dims &d, const styx_moe_layer &lw, int sms, bool waves, styx::ClusterArgs &a,
                         uint32_t &smem) {
    const int H = d.n_embd, F = d.n_ff, E = d.n_expert, k = d.n_expert_used;
    const int qg = lw.gate.qtype, qd = lw.down.qtype;
    if (lw.up.qtype != qg || !styx::cluster_supported(qg, qd)) return false;
    if (H % 64 || F % 64 || H / 4 > styx::fused_block_threads() || F / 64 > 32 || k > 16 || E > 512) return false;
    a.units_g = H / 64;
    a.gs_g = pow2ceil(a.units_g);
    a.units_d = F / 64;
    a.gs_d = pow2ceil(a.units_d);
    a.rb_g = static_cast<int>(row_bytes(qg, H));
    a.rb_u = static_cast<int>(row_bytes(lw.up.qtype, H));
    a.rb_d = static_cast<int>(row_bytes(qd, F));
    const int rpw_g = 32 / a.gs_g;
    const size_t kLimit = 227 * 1024;
    styx::ClusterArgs fallback{};
    uint32_t fallback_smem = 0;
    for (int C = styx::kClusterMaxC; C >= 1; C >>= 1) {
        if (k * C > sms) continue;
        const int ngr = (F + C - 1) / C, ndr = (H + C - 1) / C, nrr = (E + C - 1) / C;
        // gate/up chunks of about 16 row pairs (at most 8; a multiple of the rows a warp takes at once)
        int ng = std::min(8, std::max(1, (ngr + 15) / 16));
        const int chg = ((ngr + ng - 1) / ng + rpw_g - 1) / rpw_g * rpw_g;
        ng = (ngr + chg - 1) / chg;
        a.C = C;
        a.ng = ng;
        a.chg = chg;
        a.gu_up_off = static_cast<uint32_t>(a16(static_cast<size_t>(chg) * a.rb_g + 32));
        a.gu_stride = a.gu_up_off + static_cast<uint32_t>(a16(static_cast<size_t>(chg) * a.rb_u + 32));
        size_t o = styx::kClusterHeader;
        a.off_lg = static_cast<uint32_t>(o);   // logits, keys, ranks, remap, pmap
        o = a128(o + 5 * static_cast<size_t>(E) * 4);
        a.off_x = static_cast<uint32_t>(o);
        o = a128(o + static_cast<size_t>(H) * 4);
        a.off_xd = static_cast<uint32_t>(o);
        o = a128(o + 3 * static_cast<size_t>(H) + H / 32 * 4);
        a.off_hf = static_cast<uint32_t>(o);
        o = a128(o + static_cast<size_t>(F) * 4);
        a.off_hd = static_cast<uint32_t>(o);
        o = a128(o + 3 * static_cast<size_t>(F) + F / 32 * 4);
        a.off_y = static_cast<uint32_t>(o);
        o = a128(o + static_cast<size_t>(ndr) * 4);
        a.off_gu = static_cast<uint32_t>(o);
        o = a128(o + static_cast<size_t>(ng) * a.gu_stride);
        a.off_dn = static_cast<uint32_t>(o);   // the router rows, then the down rows
        o += std::max(a16(static_cast<size_t>(ndr) * a.rb_d + 32), static_cast<size_t>(nrr) * H * 4);
        if (o > kLimit) continue;
        const int n = styx::cluster_max_active(qg, qd, C, static_cast<uint32_t>(o));
        if (n >= k) {
            smem = static_cast<uint32_t>(o);
            return true;
        }
        if (n >= 1 && !fallback_smem) {
            fallback = a;
            fallback_smem = static_cast<uint32_t>(o);
        }
    }
    if (!fallback_smem || !waves) return false;
    a = fallback;
    smem = fallback_smem;
    return true;
}

static void fill_cluster(styx::ClusterArgs &ca, const styx_ctx *ctx, const styx_moe_dims &d,
                         const styx_moe_layer &lw, float *x, int32_t *ids64, float *wts, uint8_t *ws,
                         const WsLayout &L) {
    const int E = d.n_expert;
    ca.x = x;
    ca.norm_w = lw.ffn_norm;
    ca.eps = d.rms_eps;
    ca.router = lw.router;
    ca.E = E;
    ca.H = d.n_embd;
    ca.F = d.n_ff;
    ca.k = d.n_expert_used;
    ca.renorm = d.norm_topk;
    ca.remap = lw.remap;
    ca.pmap = lw.pmap;
    ca.gate = to_src(lw.gate, E);
    ca.up = to_src(lw.up, E);
    ca.down = to_src(lw.down, E);
    ca.ids64 = ids64;
    ca.weights = wts;
    ca.logits = reinterpret_cast<float *>(ws + L.logits);
    ca.xnorm = reinterpret_cast<float *>(ws + L.xnorm);
    ca.h = reinterpret_cast<float *>(ws + L.h);
    ca.y = reinterpret_cast<float *>(ws + L.d);
    ca.cnt = reinterpret_cast<unsigned *>(ws + L.ccnt);
    ca.err = ctx->d_err;
    ca.trace = ctx->trace ? reinterpret_cast<long long *>(ws + L.trace) : nullptr;
    ca.partial = nullptr;
    ca.quiet = 0;
}

// The cluster form when it fits and the option allows it: STYX_OK after the
// launch, 1 when the caller should take another form, or an error.
static int try_cluster(styx_ctx *ctx, cudaStream_t st, const styx_moe_dims &d, const styx_moe_layer &lw, float *x,
                       int32_t *ids64, float *wts, uint8_t *ws, const WsLayout &L, float *partial) {
    if (ctx->moe_kernels != 0 && ctx->moe_kernels != 3) return 1;
    styx::ClusterArgs ca{};
    uint32_t smem = 0;
    const bool fits = al16(lw.ffn_norm) && plan_cluster(d, lw, ctx->sm_count, ctx->moe_kernels == 3, ca, smem);
    if (!fits) {
        if (ctx->moe_kernels == 3) return fail(STYX_EUNSUPPORTED, "cluster MoE block does not fit these dims / formats");
        return 1;
    }
    fill_cluster(ca, ctx, d, lw, x, ids64, wts, ws, L);
    if (partial) {
        ca.partial = partial;
        ca.quiet = 1;
    }
    CK(styx::launch_cluster(ca, lw.gate.qtype, lw.down.qtype, smem, st));
    ctx->last_path = 6;
    ctx->last_cluster = ca.C;
    return STYX_OK;
}

// Argument checks shared by the MoE block entry points.
static int check_block(styx_ctx *ctx, const styx_moe_dims *dims, const styx_moe_layer *lw, int layer, const float *x,
                       const int32_t *ids, void *workspace, uint64_t workspace_bytes, WsLayout &Lout) {
    ENTER(ctx);
    int rc = check_dims(dims);
    if (rc) return rc;
    NEED(lw && x && ids && workspace, "null pointer");
    NEED(layer >= 0, "negative layer");
    NEED(lw->router && lw->ffn_norm, "router and ffn_norm are required");
    const int H = dims->n_embd, F = dims->n_ff, E = dims->n_expert, k = dims->n_expert_used;
    if ((rc = check_tensor(lw->gate, "gate", F, H, E))) return rc;
    if ((rc = check_tensor(lw->up, "up", F, H, E))) return rc;
    if ((rc = check_tensor(lw->down, "down", H, F, E))) return rc;
    const WsLayout L = ws_layout(*dims);
    Lout = L;
    NEED(workspace_bytes >= L.total, "workspace %llu bytes < %llu", (unsigned long long)workspace_bytes,
         (unsigned long long)L.total);
    NEED(al16(workspace) && al16(x) && al16(lw->router), "workspace, x and router must be 16-byte aligned");
    NEED(extent_ok(workspace, L.total), "workspace allocation smaller than workspace_bytes");
    NEED(extent_ok(lw->router, static_cast<uint64_t>(E) * H * 4), "router smaller than n_expert x n_embd");
    NEED(extent_ok(lw->ffn_norm, static_cast<uint64_t>(H) * 4) && extent_ok(x, static_cast<uint64_t>(H) * 4),
         "ffn_norm / x smaller than n_embd");
    NEED(extent_ok(ids, (static_cast<uint64_t>(layer) + 1) * STYX_IDS_PER_LAYER * 4), "ids buffer too small");
    NEED(!lw->remap || extent_ok(lw->remap, static_cast<uint64_t>(E) * 4), "remap smaller than n_expert");
    NEED(!lw->pmap || extent_ok(lw->pmap, static_cast<uint64_t>(E) * 4), "pmap smaller than n_expert");
    (void)F;
    (void)k;
    return STYX_OK;
}

int styx_moe_block(styx_ctx *ctx, styx_stream stream, const styx_moe_dims *dims, const styx_moe_layer *lw, int layer,
                   float *x, int32_t *ids, float *weights_out, void *workspace, uint64_t workspace_bytes) {
    WsLayout L;
    int rc = check_block(ctx, dims, lw, layer, x, ids, workspace, workspace_bytes, L);
    if (rc) return rc;
    uint8_t *ws = static_cast<uint8_t *>(workspace);
    int32_t *ids64 = ids + static_cast<size_t>(layer) * STYX_IDS_PER_LAYER;
    float *wts = weights_out ? weights_out : reinterpret_cast<float *>(ws + L.weights);
    const cudaStream_t st = S(stream);

    // experts read in place from pinned host memory: mul_mat_vec_id dispatches
    if (full_in_host(lw->gate) || full_in_host(lw->up) || full_in_host(lw->down)) {
        ctx->last_path = 3;
        return moe_block_host_read(ctx, st, *dims, *lw, x, ids64, wts, ws, L);
    }

    // the cluster form when the shape fits, else the single cooperative
    // kernel, else three kernels
    if ((rc = try_cluster(ctx, st, *dims, *lw, x, ids64, wts, ws, L, nullptr)) <= 0) return rc;
    if (ctx->moe_kernels != 2) {
        styx::FusedArgs fa{};
        uint32_t smem = 0;
        const bool fits = al16(lw->ffn_norm) && plan_fused(*dims, *lw, ctx->sm_count, fa, smem);
        if (!fits && ctx->moe_kernels == 1)
            return fail(STYX_EUNSUPPORTED, "single-kernel MoE block does not fit these dims / formats");
        if (fits) {
            NEED(!ctx->trace || ctx->sm_count <= static_cast<int>(kTraceCtas), "too many CTAs to trace");
            fill_fused(fa, ctx, *dims, *lw, x, ids64, wts, ws, L);
            const styx::LayerLink alone{0, false, false, true, nullptr, nullptr, nullptr};
            CK(styx::launch_fused(fa, alone, lw->gate.qtype, lw->down.qtype, ctx->sm_count, smem, !ctx->exclusive,
                                  st));
            ctx->last_path = 1;
            return STYX_OK;
        }
    }
    ctx->last_path = 2;
    return moe_block_split(ctx, st, *dims, *lw, x, ids64, wts, ws, L, nullptr, false);
}

// ------------------------------------------------ MoE blocks of consecutive layers
int styx_moe_blocks(styx_ctx *ctx, styx_stream stream, const styx_moe_dims *dims, const styx_moe_layer *layers,
                    int n_layers, int first_layer, float *x, int32_t *ids, float *weights_out, void *workspace,
                    uint64_t workspace_bytes) {
    ENTER(ctx);
    NEED(layers && n_layers >= 1, "need at least one layer");
    NEED(first_layer >= 0, "negative first layer");
    WsLayout L{};
    for (int i = 0; i < n_layers; i++) {
        const int rc = check_block(ctx, dims, &layers[i], first_layer + i, x, ids, workspace, workspace_bytes, L);
        if (rc) return rc;
    }
    const int k = dims->n_expert_used;
    // x passes between the layers as tagged words when every layer takes the
    // single kernel (and a CTA's residual rows fit its 16 spare words)
    styx::FusedArgs plan{};
    uint32_t smem = 0;
    const styx_moe_layer &l0 = layers[0];
    bool linked = ctx->moe_layers != 0 && n_layers > 1 && ctx->moe_kernels != 2 && ctx->moe_kernels != 3 &&
                  !(ctx->trace && ctx->sm_count > static_cast<int>(kTraceCtas));
    for (int i = 0; linked && i < n_layers; i++) {
        const styx_moe_layer &li = layers[i];
        linked = al16(li.ffn_norm) && !full_in_host(li.gate) && !full_in_host(li.up) && !full_in_host(li.down) &&
                 plan_fused(*dims, li, ctx->sm_count, plan, smem) && plan.rc <= 16;
    }
    uint8_t *ws = static_cast<uint8_t *>(workspace);
    const cudaStream_t st = S(stream);
    auto wts_of = [&](int i) {
        return weights_out ? weights_out + static_cast<size_t>(i) * k : reinterpret_cast<float *>(ws + L.weights);
    };
    if (linked && ctx->moe_layers == 2) {   // one chained launch per layer
        uint64_t *xslot = reinterpret_cast<uint64_t *>(ws + L.xslot);
        for (int i = 0; i < n_layers; i++) {
            const styx_moe_layer &li = layers[i];
            plan_fused(*dims, li, ctx->sm_count, plan, smem);
            fill_fused(plan, ctx, *dims, li, x, ids + static_cast<size_t>(first_layer + i) * STYX_IDS_PER_LAYER,
                       wts_of(i), ws, L);
            const bool more = i + 1 < n_layers;
            const styx::LayerLink lk{0, i > 0, more, i == 0, xslot, more ? layers[i + 1].router : nullptr,
                                     more ? layers[i + 1].ffn_norm : nullptr};
            CK(styx::launch_fused(plan, lk, li.gate.qtype, li.down.qtype, ctx->sm_count, smem, !ctx->exclusive,
                                  st));
        }
        ctx->last_path = 5;
        return STYX_OK;
    }
    // one persistent launch (per 80 layers) when, also, every layer has the same formats
    bool multi = linked && ctx->moe_layers == 1 && plan_fused(*dims, l0, ctx->sm_count, plan, smem);
    for (int i = 0; multi && i < n_layers; i++)
        multi = layers[i].gate.qtype == l0.gate.qtype && layers[i].up.qtype == l0.up.qtype &&
                layers[i].down.qtype == l0.down.qtype;
    if (!multi) {
        for (int i = 0; i < n_layers; i++) {
            const int rc = styx_moe_block(ctx, stream, dims, &layers[i], first_layer + i, x, ids,
                                          weights_out ? weights_out + static_cast<size_t>(i) * k : nullptr,
                                          workspace, workspace_bytes);
            if (rc) return rc;
        }
        return STYX_OK;
    }
    static thread_local styx::FusedLaunch la;   // 31 KB of kernel parameter, built here
    for (int base = 0; base < n_layers; base += styx::kMaxFusedLayers) {
        const int n = std::min(styx::kMaxFusedLayers, n_layers - base);
        la.n = n;
        la.xslot = reinterpret_cast<uint64_t *>(ws + L.xslot);
        for (int j = 0; j < n; j++) {
            const int i = base + j;
            la.layer[j] = plan;
            fill_fused(la.layer[j], ctx, *dims, layers[i], x,
                       ids + static_cast<size_t>(first_layer + i) * STYX_IDS_PER_LAYER, wts_of(i), ws, L);
        }
        CK(styx::launch_fused_layers(la, l0.gate.qtype, l0.down.qtype, ctx->sm_count, smem, !ctx->exclusive, st));
    }
    ctx->last_path = 4;
    return STYX_OK;
}

// ------------------------------------------------ MoE block, expert parallel
int styx_moe_block_ep(styx_ctx *ctx, styx_stream stream, const styx_moe_dims *dims, const styx_moe_layer *lw,
                      int layer, const float *x, int32_t *ids, float *weights_out, float *partial, void *workspace,
                      uint64_t workspace_bytes) {
    WsLayout L;
    int rc = check_block(ctx, dims, lw, layer, x, ids, workspace, workspace_bytes, L);
    if (rc) return rc;
    const uint64_t pbytes = static_cast<uint64_t>(dims->n_expert_used) * dims->n_embd * 4;
    NEED(partial && al16(partial) && extent_ok(partial, pbytes), "partial: 16-byte aligned f32[k * n_embd] required");
    uint8_t *ws = static_cast<uint8_t *>(workspace);
    int32_t *ids64 = ids + static_cast<size_t>(layer) * STYX_IDS_PER_LAYER;
    float *wts = weights_out ? weights_out : reinterpret_cast<float *>(ws + L.weights);
    const cudaStream_t st = S(stream);
    // the cluster form or the single kernel, with their partial-output
    // epilogues, when the shape fits
    const bool in_hbm = !full_in_host(lw->gate) && !full_in_host(lw->up) && !full_in_host(lw->down);
    if (in_hbm && (rc = try_cluster(ctx, st, *dims, *lw, const_cast<float *>(x), ids64, wts, ws, L, partial)) <= 0)
        return rc;
    if (ctx->moe_kernels != 2 && ctx->moe_kernels != 3 && in_hbm) {
        styx::FusedArgs fa{};
        uint32_t smem = 0;
        if (al16(lw->ffn_norm) && plan_fused(*dims, *lw, ctx->sm_count, fa, smem)) {
            NEED(!ctx->trace || ctx->sm_count <= static_cast<int>(kTraceCtas), "too many CTAs to trace");
            fill_fused(fa, ctx, *dims, *lw, const_cast<float *>(x), ids64, wts, ws, L);
            fa.partial = partial;
            fa.quiet = 1;
            const styx::LayerLink alone{0, false, false, true, nullptr, nullptr, nullptr};
            CK(styx::launch_fused(fa, alone, lw->gate.qtype, lw->down.qtype, ctx->sm_count, smem, !ctx->exclusive,
                                  st));
            ctx->last_path = 1;
            return STYX_OK;
        }
    }
    ctx->last_path = 2;
    return moe_block_split(ctx, st, *dims, *lw, const_cast<float *>(x), ids64, wts, ws, L, partial, true);
}

// ------------------------------------------------ MoE block, a batch of tokens (tensor cores)
namespace {
struct BatchLayout {
    size_t xh, n_used, used_e, cnt, off, pair, pv, srcs, panel_x, panel_h, d, logits, gpart, upart, item_cnt, split,
        src_sel, total;
};
BatchLayout batch_layout(const styx_moe_dims &d, int B) {
    BatchLayout L{};
    size_t o = 0;
    auto take = [&](size_t n) {
        const size_t r = o;
        o = (o + n + 255) & ~size_t(255);
        return r;
    };
    const size_t H = d.n_embd, E = d.n_expert, F = d.n_ff, P = static_cast<size_t>(B) * d.n_expert_used;
    L.xh = take(static_cast<size_t>(B) * H * 2);
    L.n_used = take(16);
    L.used_e = take(E * 4);
    L.cnt = take(E * 4);
    L.off = take((E + 1) * 4);
    L.pair = take(P * 4);
    L.pv = take(P * 4);
    L.srcs = take(E * 3 * 8);
    const size_t npm = static_cast<size_t>((B + 15) & ~15);
    L.panel_x = take(E * npm * H * 2);
    L.panel_h = take(E * npm * F * 2);
    L.d = take(static_cast<size_t>(styx::batch_split_max(d.n_ff)) * P * H * 4);
    L.logits = take(static_cast<size_t>(B) * E * 4);
    L.gpart = take(static_cast<size_t>(styx::batch_split_max(d.n_embd)) * P * F * 4);
    L.upart = take(static_cast<size_t>(styx::batch_split_max(d.n_embd)) * P * F * 4);
    L.item_cnt = take(E * (F / 128) * 4);
    L.split = take(16);
    L.src_sel = take(E * 4);
    L.total = o;
    return L;
}
// cuTensorMapEncodeTiled through the runtime's driver entry point (no link
// against libcuda)
typedef CUresult (*EncodeTiledFn)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *, const cuuint64_t *,
                                  const cuuint64_t *, const cuuint32_t *, const cuuint32_t *, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);
EncodeTiledFn encode_tiled() {
    static EncodeTiledFn fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void *p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<EncodeTiledFn>(p);
    });
    return fn;
}
// The TMA descriptors of one expert matrix: for each source present (hot,
// arena, full) a 3-D byte tensor {row bytes, rows, slabs} with strides {row
// bytes, slab stride}, box {one 256-element chunk of a row, 128 rows, 1}.
int encode_expert_maps(const styx_expert_tensor &t, int nrows, int ncols, int n_expert, CUtensorMap out[3]) {
    EncodeTiledFn fn = encode_tiled();
    NEED(fn, "cuTensorMapEncodeTiled is not available");
    const uint64_t rb = static_cast<uint64_t>(row_bytes(t.qtype, ncols));
    const uint32_t bb = static_cast<uint32_t>(row_bytes(t.qtype, 256));
    const void *base[3] = {t.hot, t.arena, t.full};
    const uint64_t n[3] = {t.n_hot, t.n_arena, static_cast<uint64_t>(n_expert)};
    const uint64_t stride[3] = {t.slab_bytes, t.arena_slab_bytes, t.slab_bytes};
    for (int i = 0; i < 3; i++) {
        memset(&out[i], 0, sizeof(CUtensorMap));
        if (!base[i] || !n[i]) continue;
        const cuuint64_t dims[3] = {rb, static_cast<cuuint64_t>(nrows), n[i]};
        const cuuint64_t strides[2] = {rb, stride[i]};
        const cuuint32_t box[3] = {bb, 128, 1}, es[3] = {1, 1, 1};
        const CUresult r = fn(&out[i], CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, const_cast<void *>(base[i]), dims, strides, box,
                              es, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                              CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
        NEED(r == CUDA_SUCCESS, "cuTensorMapEncodeTiled failed (%d)", static_cast<int>(r));
    }
    return STYX_OK;
}
}  // namespace

int styx_moe_batch_workspace_bytes(const styx_moe_dims *dims, int n_tokens, uint64_t *out) {
    int rc = check_dims(dims);
    if (rc) return rc;
    NEED(out, "null out");
    NEED(n_tokens >= 1 && n_tokens <= STYX_MAX_BATCH, "n_tokens %d: 1..%d", n_tokens, STYX_MAX_BATCH);
    *out = batch_layout(*dims, n_tokens).total;
    return STYX_OK;
}

int styx_moe_block_batch(styx_ctx *ctx, styx_stream stream, const styx_moe_dims *dims, const styx_moe_layer *lw,
                         int n_tokens, float *x, int32_t *ids, float *weights_out, void *workspace,
                         uint64_t workspace_bytes) {
    ENTER(ctx);
    int rc = check_dims(dims);
    if (rc) return rc;
    NEED(lw && x && ids && weights_out && workspace, "null pointer");
    NEED(n_tokens >= 1 && n_tokens <= STYX_MAX_BATCH, "n_tokens %d: 1..%d", n_tokens, STYX_MAX_BATCH);
    NEED(lw->router && lw->ffn_norm, "router and ffn_norm are required");
    const int H = dims->n_embd, F = dims->n_ff, E = dims->n_expert, k = dims->n_expert_used, B = n_tokens;
    if ((rc = check_tensor(lw->gate, "gate", F, H, E))) return rc;
    if ((rc = check_tensor(lw->up, "up", F, H, E))) return rc;
    if ((rc = check_tensor(lw->down, "down", H, F, E))) return rc;
    NEED(lw->up.qtype == lw->gate.qtype, "gate and up must share one format");
    NEED(styx::batch_supported(lw->gate.qtype, lw->down.qtype), "formats %d / %d not supported by the batch path",
         lw->gate.qtype, lw->down.qtype);
    NEED(!full_in_host(lw->gate) && !full_in_host(lw->up) && !full_in_host(lw->down),
         "the batch path reads experts from device memory only");
    const BatchLayout L = batch_layout(*dims, B);
    NEED(workspace_bytes >= L.total, "workspace %llu bytes < %llu", (unsigned long long)workspace_bytes,
         (unsigned long long)L.total);
    NEED(al16(workspace) && extent_ok(workspace, L.total), "workspace: 16-byte aligned, workspace_bytes long");
    NEED(al16(x) && al16(lw->router) && al16(lw->ffn_norm), "x, router and ffn_norm must be 16-byte aligned");
    NEED(extent_ok(x, static_cast<uint64_t>(B) * H * 4), "x smaller than n_tokens x n_embd");
    NEED(extent_ok(ids, static_cast<uint64_t>(B) * STYX_IDS_PER_LAYER * 4), "ids smaller than n_tokens id blocks");
    NEED(extent_ok(weights_out, static_cast<uint64_t>(B) * k * 4), "weights_out smaller than n_tokens x k");
    NEED(extent_ok(lw->router, static_cast<uint64_t>(E) * H * 4), "router smaller than n_expert x n_embd");
    NEED(extent_ok(lw->ffn_norm, static_cast<uint64_t>(H) * 4), "ffn_norm smaller than n_embd");
    NEED(!lw->remap || extent_ok(lw->remap, static_cast<uint64_t>(E) * 4), "remap smaller than n_expert");
    NEED(!lw->pmap || extent_ok(lw->pmap, static_cast<uint64_t>(E) * 4), "pmap smaller than n_expert");
    uint8_t *ws = static_cast<uint8_t *>(workspace);
    styx::BatchArgs a{};
    a.x = x;
    a.norm_w = lw->ffn_norm;
    a.eps = dims->rms_eps;
    a.router = lw->router;
    a.E = E;
    a.H = H;
    a.F = F;
    a.k = k;
    a.renorm = dims->norm_topk;
    a.B = B;
    a.rb_g = static_cast<int>(row_bytes(lw->gate.qtype, H));
    a.rb_d = static_cast<int>(row_bytes(lw->down.qtype, F));
    a.remap = lw->remap;
    a.pmap = lw->pmap;
    a.gate = to_src(lw->gate, E);
    a.up = to_src(lw->up, E);
    a.down = to_src(lw->down, E);
    a.ids = ids;
    a.weights = weights_out;
    a.xh = reinterpret_cast<__half *>(ws + L.xh);
    a.n_used = reinterpret_cast<int *>(ws + L.n_used);
    a.used_e = reinterpret_cast<int *>(ws + L.used_e);
    a.cnt = reinterpret_cast<int *>(ws + L.cnt);
    a.off = reinterpret_cast<int *>(ws + L.off);
    a.pair = reinterpret_cast<int *>(ws + L.pair);
    a.pv = reinterpret_cast<int *>(ws + L.pv);
    a.srcs = reinterpret_cast<const uint8_t **>(ws + L.srcs);
    a.panel_x = reinterpret_cast<__half *>(ws + L.panel_x);
    a.panel_h = reinterpret_cast<__half *>(ws + L.panel_h);
    a.npm = (B + 15) & ~15;
    a.d = reinterpret_cast<float *>(ws + L.d);
    a.logits = reinterpret_cast<float *>(ws + L.logits);
    a.gpart = reinterpret_cast<float *>(ws + L.gpart);
    a.upart = reinterpret_cast<float *>(ws + L.upart);
    a.item_cnt = reinterpret_cast<int *>(ws + L.item_cnt);
    a.n_item_cnt = E * (F / 128);
    a.split_d = reinterpret_cast<int *>(ws + L.split);
    a.sms = ctx->sm_count;
    a.src_sel = reinterpret_cast<uint32_t *>(ws + L.src_sel);
    a.quiet = 0;
    a.err = ctx->d_err;
    styx::TmaSet tgu, tdn;
    memset(&tgu, 0, sizeof(tgu));
    memset(&tdn, 0, sizeof(tdn));
    if (styx::batch_uses_tma(lw->gate.qtype)) {
        if ((rc = encode_expert_maps(lw->gate, F, H, E, tgu.m[0]))) return rc;
        if ((rc = encode_expert_maps(lw->up, F, H, E, tgu.m[1]))) return rc;
    }
    if (styx::batch_uses_tma(lw->down.qtype) && (rc = encode_expert_maps(lw->down, H, F, E, tdn.m[0]))) return rc;
    CK(styx::launch_batch(a, lw->gate.qtype, lw->down.qtype, tgu, tdn, S(stream)));
    return STYX_OK;
}

int styx_moe_combine(styx_ctx *ctx, styx_stream stream, const float *partial, float *x, int ne, int k) {
    ENTER(ctx);
    NEED(partial && x, "null pointer");
    NEED(ne > 0 && k > 0 && k <= STYX_MAX_TOPK, "bad ne %d / k %d", ne, k);
    NEED(extent_ok(partial, static_cast<uint64_t>(ne) * k * 4) && extent_ok(x, static_cast<uint64_t>(ne) * 4),
         "partial / x smaller than k * ne / ne");
    CK(styx::launch_combine_partial(partial, x, ne, k, S(stream)));
    return STYX_OK;
}

// ------------------------------------------------ cross-rank combine over peer memory
// One device allocation per rank, mapped by every peer: the inbox (two
// halves of world x k x H tagged 8-byte words), then (ctl_off) the call
// counter (u64) and the CTAs done of the current call (u32); then, read only
// by this rank, the EpPeers table the kernels take and the partial buffer
// styx_ep_moe_block uses when the block does not run as the single kernel.
struct styx_ep {
    int dev = 0, rank = 0, world = 1, k = 0, H = 0;
    uint8_t *base = nullptr;
    size_t ctl_off = 0, peers_off = 0, partial_off = 0;
    styx::EpPeers peers{};                        // host copy of the table
    styx::EpPeers *d_peers = nullptr;             // device copy (in base)
    void *peer_base[styx::kEpMaxRanks] = {};      // the peers' mappings (closed by styx_ep_close)
    bool connected = false;
};
static_assert(sizeof(cudaIpcMemHandle_t) == STYX_EP_HANDLE_BYTES, "IPC handle size");
static_assert(styx::kEpMaxRanks == STYX_EP_MAX_RANKS, "rank limit");

namespace {
void ep_bind(styx_ep *ep, int p, uint8_t *b) { ep->peers.inbox[p] = reinterpret_cast<unsigned long long *>(b); }
}  // namespace

int styx_ep_open(styx_ctx *ctx, int rank, int world, int k, int n_embd, styx_ep **out, void *handle) {
    ENTER(ctx);
    NEED(out && handle, "null pointer");
    NEED(world >= 1 && world <= STYX_EP_MAX_RANKS && rank >= 0 && rank < world, "rank %d of world %d (at most %d)",
         rank, world, STYX_EP_MAX_RANKS);
    NEED(k >= 1 && k <= STYX_MAX_TOPK && n_embd > 0 && n_embd % 4 == 0, "bad k %d / n_embd %d", k, n_embd);
    styx_ep *ep = new styx_ep();
    ep->dev = ctx->device;
    ep->rank = rank;
    ep->world = world;
    ep->k = k;
    ep->H = n_embd;
    ep->ctl_off = a128(2 * static_cast<size_t>(world) * k * n_embd * 8);
    ep->peers_off = ep->ctl_off + 128;
    ep->partial_off = a128(ep->peers_off + sizeof(styx::EpPeers));
    const size_t total = ep->partial_off + static_cast<size_t>(k) * n_embd * 4;
    void *p = nullptr;
    cudaError_t e = cudaMalloc(&p, total);
    if (e == cudaSuccess) e = cudaMemset(p, 0, total);
    if (e == cudaSuccess) e = cudaDeviceSynchronize();   // zeroed before any peer can map it
    cudaIpcMemHandle_t h{};
    if (e == cudaSuccess) e = cudaIpcGetMemHandle(&h, p);
    if (e != cudaSuccess) {
        if (p) cudaFree(p);
        delete ep;
        return fail(STYX_ECUDA, "styx_ep_open: %s", cudaGetErrorString(e));
    }
    ep->base = static_cast<uint8_t *>(p);
    ep->d_peers = reinterpret_cast<styx::EpPeers *>(ep->base + ep->peers_off);
    ep_bind(ep, rank, ep->base);
    ep->peers.calls = reinterpret_cast<unsigned long long *>(ep->base + ep->ctl_off);
    ep->peers.done = reinterpret_cast<unsigned *>(ep->peers.calls + 1);
    ep->peers.rank = rank;
    ep->peers.world = world;
    ep->peers.k = k;
    ep->peers.H = n_embd;
    memcpy(handle, &h, sizeof(h));
    *out = ep;
    return STYX_OK;
}

int styx_ep_connect(styx_ep *ep, const void *handles) {
    NEED(ep && handles, "null pointer");
    NEED(!ep->connected, "styx_ep_connect: already connected");
    CK(cudaSetDevice(ep->dev));
    const uint8_t *hb = static_cast<const uint8_t *>(handles);
    for (int p = 0; p < ep->world; p++) {
        if (p == ep->rank) continue;
        cudaIpcMemHandle_t h;
        memcpy(&h, hb + static_cast<size_t>(p) * STYX_EP_HANDLE_BYTES, sizeof(h));
        void *ptr = nullptr;
        const cudaError_t e = cudaIpcOpenMemHandle(&ptr, h, cudaIpcMemLazyEnablePeerAccess);
        if (e != cudaSuccess) {
            for (int q = 0; q < p; q++)
                if (ep->peer_base[q]) {
                    cudaIpcCloseMemHandle(ep->peer_base[q]);
                    ep->peer_base[q] = nullptr;
                }
            return fail(STYX_ECUDA, "styx_ep_connect: rank %d's inbox: %s", p, cudaGetErrorString(e));
        }
        ep->peer_base[p] = ptr;
        ep_bind(ep, p, static_cast<uint8_t *>(ptr));
    }
    CK(cudaMemcpy(ep->d_peers, &ep->peers, sizeof(styx::EpPeers), cudaMemcpyHostToDevice));
    ep->connected = true;
    return STYX_OK;
}

namespace {
int ep_check(styx_ctx *ctx, styx_ep *ep) {
    NEED(ep, "null styx_ep");
    NEED(ep->connected, "styx_ep used before styx_ep_connect");
    NEED(ep->dev == ctx->device, "styx_ep of device %d used with a context of device %d", ep->dev, ctx->device);
    return STYX_OK;
}
}  // namespace

int styx_ep_combine(styx_ctx *ctx, styx_ep *ep, styx_stream stream, const float *partial, float *x) {
    ENTER(ctx);
    int rc = ep_check(ctx, ep);
    if (rc) return rc;
    NEED(partial && x, "null pointer");
    NEED(al16(partial), "partial must be 16-byte aligned");
    NEED(extent_ok(partial, static_cast<uint64_t>(ep->k) * ep->H * 4) && extent_ok(x, static_cast<uint64_t>(ep->H) * 4),
         "partial / x smaller than k * n_embd / n_embd");
    styx::EpCombineArgs a{};
    a.partial = partial;
    a.x = x;
    a.ep = ep->d_peers;
    a.H = ep->H;
    a.err = ctx->d_err;
    CK(styx::launch_ep_combine(a, S(stream)));
    return STYX_OK;
}

int styx_ep_moe_block(styx_ctx *ctx, styx_ep *ep, styx_stream stream, const styx_moe_dims *dims,
                      const styx_moe_layer *lw, int layer, float *x, int32_t *ids, float *weights_out, void *workspace,
                      uint64_t workspace_bytes) {
    ENTER(ctx);
    int rc = ep_check(ctx, ep);
    if (rc) return rc;
    WsLayout L;
    if ((rc = check_block(ctx, dims, lw, layer, x, ids, workspace, workspace_bytes, L))) return rc;
    NEED(dims->n_expert_used == ep->k && dims->n_embd == ep->H, "styx_ep opened for k %d / n_embd %d, dims say %d / %d",
         ep->k, ep->H, dims->n_expert_used, dims->n_embd);
    const bool in_hbm = !full_in_host(lw->gate) && !full_in_host(lw->up) && !full_in_host(lw->down);
    if (in_hbm && (ctx->moe_kernels == 0 || ctx->moe_kernels == 1)) {
        styx::FusedArgs fa{};
        uint32_t smem = 0;
        if (al16(lw->ffn_norm) && plan_fused(*dims, *lw, ctx->sm_count, fa, smem) && ctx->sm_count <= dims->n_embd) {
            NEED(!ctx->trace || ctx->sm_count <= static_cast<int>(kTraceCtas), "too many CTAs to trace");
            uint8_t *ws = static_cast<uint8_t *>(workspace);
            int32_t *ids64 = ids + static_cast<size_t>(layer) * STYX_IDS_PER_LAYER;
            float *wts = weights_out ? weights_out : reinterpret_cast<float *>(ws + L.weights);
            fill_fused(fa, ctx, *dims, *lw, x, ids64, wts, ws, L);
            fa.ep = ep->d_peers;
            fa.quiet = 1;
            const styx::LayerLink alone{0, false, false, true, nullptr, nullptr, nullptr};
            CK(styx::launch_fused(fa, alone, lw->gate.qtype, lw->down.qtype, ctx->sm_count, smem, !ctx->exclusive,
                                  S(stream)));
            ctx->last_path = 1;
            return STYX_OK;
        }
    }
    float *partial = reinterpret_cast<float *>(ep->base + ep->partial_off);
    if ((rc = styx_moe_block_ep(ctx, stream, dims, lw, layer, x, ids, weights_out, partial, workspace,
                                workspace_bytes)))
        return rc;
    const int path = ctx->last_path;
    rc = styx_ep_combine(ctx, ep, stream, partial, x);
    ctx->last_path = path;
    return rc;
}

int styx_ep_close(styx_ep *ep) {
    if (!ep) return STYX_OK;
    cudaSetDevice(ep->dev);
    cudaDeviceSynchronize();   // no call of this rank still reads or writes the inboxes
    for (int p = 0; p < ep->world; p++)
        if (ep->peer_base[p]) cudaIpcCloseMemHandle(ep->peer_base[p]);
    if (ep->base) cudaFree(ep->base);
    delete ep;
    return STYX_OK;
}

// ------------------------------------------------ MoE block, no allocation
int styx_moe_block_noalloc(styx_ctx *ctx, styx_stream stream, const styx_moe_dims *dims, const styx_moe_layer *lw,
                           int layer, float *x, int32_t *ids, float *weights_out) {
    ENTER(ctx);
    int rc = check_dims(dims);
    if (rc) return rc;
    const WsLayout L = ws_layout(*dims);
    NEED(L.total <= STYX_NOALLOC_SCRATCH_BYTES,
         "styx_moe_block_noalloc: these dims need %llu bytes of scratch, above its static %llu bytes; "
         "use styx_moe_block with a caller workspace",
         (unsigned long long)L.total, (unsigned long long)STYX_NOALLOC_SCRATCH_BYTES);
    void *scratch = nullptr;
    if ((rc = noalloc_scratch(ctx, S(stream), &scratch))) return rc;
    // Every call starts from a clean scratch: the counter block (the hand-off
    // counter, the launch counter, the h-arrival counts) and the tagged logit
    // and x words are cleared on `stream` first.  Their places depend on the
    // dims, and a call whose bounded wait ran out leaves them part-advanced;
    // cleared, neither an earlier call with other dims nor a timed-out one
    // leaves a word this call could take for its own.
    CK(cudaMemsetAsync(scratch, 0, L.trace, S(stream)));
    return styx_moe_block(ctx, stream, dims, lw, layer, x, ids, weights_out, scratch, STYX_NOALLOC_SCRATCH_BYTES);
}

// ------------------------------------------------------------- synth
int styx_synth_quant(styx_ctx *ctx, styx_stream stream, int qtype, void *dst, uint64_t nrows, int ncols,
                     uint64_t seed, float sigma) {
    ENTER(ctx);
    NEED(dst, "null dst");
    NEED(qtype_ok(qtype) && row_bytes(qtype, ncols) > 0, "bad qtype/ncols");
    CK(styx::launch_synth_quant(qtype, static_cast<uint8_t *>(dst), nrows, ncols, seed, sigma, S(stream)));
    return STYX_OK;
}

int styx_synth_f32(styx_ctx *ctx, styx_stream stream, float *dst, uint64_t n, uint64_t seed, uint64_t offset,
                   float sigma) {
    ENTER(ctx);
    NEED(dst, "null dst");
    CK(styx::launch_synth_f32(dst, n, seed, offset, sigma, S(stream)));
    return STYX_OK;
}

}  // extern "C"

// ------------------------------------------------ attention half of a decode layer (styx_attn.h)
// A dense GEMV streamed by the down kernel as a one-slot block: rows in
// chunks of 16 lane groups' rows through a ring of bulk copies, x as digits
// in shared memory; y = W x (the kernel's per-slot output) or, with
// `accumulate`, y += W x (its weighted combine with weight 1, which rounds
// exactly as a separate add).
static int dense_gemv(styx_ctx *ctx, cudaStream_t st, int qtype, const void *a, int nrows, int ncols,
                      const float *x, float *y, bool accumulate) {
    NEED(a && x && y && nrows > 0, "bad mul_mat_vec arguments");
    NEED(qtype_ok(qtype), "unsupported qtype %d", qtype);
    NEED(units_ok(qtype, ncols) && ncols <= 16384, "ncols %d not supported for qtype %d", ncols, qtype);
    const long long rb = row_bytes(qtype, ncols);
    if (qtype == STYX_Q4_K || qtype == STYX_Q5_K)
        NEED(al16(a) && rb % 16 == 0, "q4_K/q5_K matrices must be 16-byte aligned");
    else
        NEED((reinterpret_cast<uintptr_t>(a) & 1) == 0, "matrix must be 2-byte aligned");
    NEED(extent_ok(a, static_cast<uint64_t>(rb) * nrows), "matrix smaller than nrows rows");
    NEED(extent_ok(x, static_cast<uint64_t>(ncols) * 4) && extent_ok(y, static_cast<uint64_t>(nrows) * 4),
         "x / y smaller than their lengths");
    styx_expert_tensor t{};
    t.full = a;
    t.slab_bytes = static_cast<uint64_t>(rb) * nrows;
    t.qtype = qtype;
    styx::DownArgs da{};
    da.down = to_src(t, 1);
    da.ids64 = reinterpret_cast<const int32_t *>(static_cast<uint8_t *>(ctx->d_scratch) + kScratchDenseIds);
    da.h = x;
    da.w = reinterpret_cast<const float *>(static_cast<uint8_t *>(ctx->d_scratch) + kScratchOne);
    da.x = accumulate ? y : nullptr;
    da.partial = accumulate ? nullptr : y;
    da.H = nrows;
    da.F = ncols;
    da.k = 1;
    da.rb = static_cast<int>(rb);
    da.units = ncols / 64;
    da.gs = std::min(32, pow2ceil(da.units));
    da.rc = 2 * styx::kWideConsumerWarps * (32 / da.gs);   // two rows per lane group per chunk
    da.slot_stride = static_cast<uint32_t>(a16(static_cast<size_t>(da.rc) * da.rb + 32));
    da.stage_bytes = da.slot_stride;
    const int grid = std::max(1, std::min(ctx->sm_count, (nrows + da.rc - 1) / da.rc));
    const int rows = (nrows + grid - 1) / grid;
    da.dig_off = 512;
    const size_t dig_bytes = static_cast<size_t>(ncols) * 3 + ncols / 32 * 4;
    const int chunks = (rows + da.rc - 1) / da.rc;
    const size_t fixed = a128(a128(da.dig_off + dig_bytes) + static_cast<size_t>(std::max(2, chunks)) * da.rc * 4);
    const int nst = std::min({16, chunks, static_cast<int>((227 * 1024 - std::min<size_t>(fixed, 227 * 1024)) /
                                                            da.stage_bytes)});
    NEED(nst >= 1, "rows of %d columns too large for shared memory", ncols);
    da.nst = nst;
    da.part_off = static_cast<uint32_t>(a128(da.dig_off + dig_bytes));
    da.stage_off = static_cast<uint32_t>(a128(da.part_off + static_cast<size_t>(std::max(2, nst)) * da.rc * 4));
    const uint32_t smem = da.stage_off + static_cast<uint32_t>(nst) * da.stage_bytes;
    NEED(smem <= 227 * 1024, "dense GEMV needs %u bytes of shared memory", smem);
    da.err = ctx->d_err;
    CK(styx::launch_down(da, qtype, grid, smem, st, true));
    return STYX_OK;
}

int styx_mul_mat_vec(styx_ctx *ctx, styx_stream stream, int qtype, const void *a, int nrows, int ncols,
                     const float *x, float *y) {
    ENTER(ctx);
    return dense_gemv(ctx, S(stream), qtype, a, nrows, ncols, x, y, false);
}

int styx_mul_mat_vec_add(styx_ctx *ctx, styx_stream stream, int qtype, const void *a, int nrows, int ncols,
                         const float *x, float *y) {
    ENTER(ctx);
    return dense_gemv(ctx, S(stream), qtype, a, nrows, ncols, x, y, true);
}

int styx_add_f32(styx_ctx *ctx, styx_stream stream, const float *a, const float *b, float *d, int n) {
    ENTER(ctx);
    NEED(a && b && d && n > 0, "bad add arguments");
    NEED(extent_ok(a, static_cast<uint64_t>(n) * 4) && extent_ok(b, static_cast<uint64_t>(n) * 4) &&
             extent_ok(d, static_cast<uint64_t>(n) * 4),
         "buffer smaller than n");
    CK(styx::launch_add_f32(a, b, d, n, S(stream)));
    return STYX_OK;
}

int styx_qk_norm_rope_kv(styx_ctx *ctx, styx_stream stream, float *q, float *k, const float *v,
                         const float *q_norm, const float *k_norm, float eps, int n_heads, int n_kv,
                         int head_dim, int n_tokens, float freq_base, const int32_t *pos, float *kcache,
                         float *vcache, int n_ctx) {
    ENTER(ctx);
    NEED(head_dim > 0 && head_dim % 2 == 0 && head_dim <= 256, "head_dim %d: need even, <= 256", head_dim);
    NEED(n_heads >= 0 && n_kv >= 0 && n_heads + n_kv > 0 && n_tokens > 0, "bad head / token counts");
    NEED(pos && (n_heads == 0 || q) && (n_kv == 0 || k), "null pointer");
    NEED(!(kcache || vcache) || n_ctx > 0, "n_ctx %d with a cache", n_ctx);
    NEED(!vcache || v, "vcache without v");
    NEED(freq_base > 0.f, "freq_base must be positive");
    const uint64_t hd = static_cast<uint64_t>(head_dim), kv_dim = hd * n_kv;
    NEED(extent_ok(q, hd * n_heads * n_tokens * 4) && extent_ok(k, kv_dim * n_tokens * 4) &&
             extent_ok(v, kv_dim * n_tokens * 4) && extent_ok(pos, static_cast<uint64_t>(n_tokens) * 4),
         "q / k / v / pos smaller than their shapes");
    NEED(extent_ok(q_norm, hd * 4) && extent_ok(k_norm, hd * 4), "q_norm / k_norm smaller than head_dim");
    NEED(extent_ok(kcache, kv_dim * n_ctx * 4) && extent_ok(vcache, kv_dim * n_ctx * 4), "cache smaller than n_ctx rows");
    styx::QkRopeArgs a{};
    a.q = q;
    a.k = k;
    a.v = v;
    a.q_norm = n_heads ? q_norm : nullptr;
    a.k_norm = n_kv ? k_norm : nullptr;
    a.eps = eps;
    a.pos = pos;
    // RopePush::neox's theta_scale (ops.rs:428), kept in double as the
    // reference test's CPU form evaluates it (tests/ops2.rs:427)
    a.theta_scale = std::pow(static_cast<double>(freq_base), -2.0 / static_cast<double>(head_dim));
    a.n_heads = n_heads;
    a.n_kv = n_kv;
    a.hd = head_dim;
    a.kv_dim = static_cast<int>(kv_dim);
    a.n_tokens = n_tokens;
    a.n_ctx = n_ctx;
    a.kcache = kcache;
    a.vcache = vcache;
    a.err = ctx->d_err;
    CK(styx::launch_qk_norm_rope_kv(a, S(stream)));
    return STYX_OK;
}

int styx_rope_neox(styx_ctx *ctx, styx_stream stream, float *x, int head_dim, int n_heads, int n_tokens,
                   float freq_base, const int32_t *pos) {
    return styx_qk_norm_rope_kv(ctx, stream, x, nullptr, nullptr, nullptr, nullptr, 0.f, n_heads, 0, head_dim,
                                n_tokens, freq_base, pos, nullptr, nullptr, 0);
}

namespace {
constexpr int kAttnMaxSplits = 256;
constexpr int kAttnMinTokensPerSplit = 16;

// splits of the sequence: about two CTAs per SM over the kv heads, at least
// 16 tokens each, shared memory within the per-CTA limit
void attn_plan(int sms, int n_kv, int gqa, int hd, int n_t, int &tps, int &n_splits) {
    int want = std::max(1, (2 * sms + n_kv - 1) / n_kv);
    want = std::min(want, std::max(1, (n_t + kAttnMinTokensPerSplit - 1) / kAttnMinTokensPerSplit));
    want = std::min(want, kAttnMaxSplits);
    tps = (n_t + want - 1) / want;
    while (styx::attn_smem_bytes(gqa, hd, tps) > 200 * 1024 && want < kAttnMaxSplits) {
        want = std::min(kAttnMaxSplits, want * 2);
        tps = (n_t + want - 1) / want;
    }
    n_splits = (n_t + tps - 1) / tps;
}
}  // namespace

int styx_attn_workspace_bytes(int n_heads, int head_dim, uint64_t *out) {
    NEED(out && n_heads > 0 && head_dim > 0, "bad arguments");
    *out = static_cast<uint64_t>(n_heads) * kAttnMaxSplits * (static_cast<uint64_t>(head_dim) + 2) * 4;
    return STYX_OK;
}

int styx_attn_decode(styx_ctx *ctx, styx_stream stream, const float *q, const float *kcache,
                     const float *vcache, float *out, int n_t, int head_dim, int kv_dim, int gqa, float scale,
                     void *workspace, uint64_t workspace_bytes) {
    ENTER(ctx);
    NEED(q && kcache && vcache && out && workspace, "null pointer");
    NEED(head_dim > 0 && head_dim % 4 == 0 && head_dim <= 256, "head_dim %d: need a multiple of 4, <= 256", head_dim);
    NEED(kv_dim > 0 && kv_dim % head_dim == 0 && gqa > 0 && n_t > 0, "bad kv_dim / gqa / n_t");
    NEED(al16(q) && al16(kcache) && al16(vcache) && al16(out), "q, caches and out must be 16-byte aligned");
    const int n_kv = kv_dim / head_dim, n_heads = n_kv * gqa;
    uint64_t need = 0;
    styx_attn_workspace_bytes(n_heads, head_dim, &need);
    NEED(workspace_bytes >= need && al16(workspace), "workspace: %llu bytes, 16-byte aligned, needed",
         static_cast<unsigned long long>(need));
    NEED(extent_ok(q, static_cast<uint64_t>(n_heads) * head_dim * 4) &&
             extent_ok(out, static_cast<uint64_t>(n_heads) * head_dim * 4),
         "q / out smaller than n_heads * head_dim");
    NEED(extent_ok(kcache, static_cast<uint64_t>(n_t) * kv_dim * 4) &&
             extent_ok(vcache, static_cast<uint64_t>(n_t) * kv_dim * 4),
         "caches smaller than n_t rows");
    NEED(extent_ok(workspace, need), "workspace allocation smaller than needed");
    styx::AttnArgs a{};
    a.q = q;
    a.kcache = kcache;
    a.vcache = vcache;
    a.out = out;
    a.n_t = n_t;
    a.hd = head_dim;
    a.kv_dim = kv_dim;
    a.gqa = gqa;
    a.n_kv = n_kv;
    a.scale = scale;
    attn_plan(ctx->sm_count, n_kv, gqa, head_dim, n_t, a.tps, a.n_splits);
    NEED(styx::attn_smem_bytes(gqa, head_dim, a.tps) <= 227 * 1024, "gqa %d x head_dim %d too large", gqa, head_dim);
    a.part_acc = static_cast<float *>(workspace);
    a.part_ml = a.part_acc + static_cast<size_t>(n_heads) * a.n_splits * head_dim;
    CK(styx::launch_attn_decode(a, S(stream)));
    return STYX_OK;
}

namespace {
struct AttnWs {
    size_t cnt, xnorm, qkv, att, part, opart, ccnt, trace, total;
};
AttnWs attn_ws(const styx_attn_dims &d) {
    AttnWs w{};
    size_t o = 0;
    auto take = [&](size_t n) {
        const size_t r = o;
        o = (o + n + 255) & ~size_t(255);
        return r;
    };
    const size_t H = d.n_embd, qd = static_cast<size_t>(d.n_heads) * d.head_dim,
                 kvd = static_cast<size_t>(d.n_kv_heads) * d.head_dim;
    // the single kernel's counters: launch counter, per-head arrivals (q, k,
    // v heads), per-kv-head split arrivals, attention-output arrivals
    w.cnt = take(8 * (1 + static_cast<size_t>(d.n_heads) + 3 * static_cast<size_t>(d.n_kv_heads) + 1));
    w.xnorm = take(H * 4);
    w.qkv = take((qd + 2 * kvd) * 4);   // q | k | v, contiguous
    w.att = take(qd * 4);
    uint64_t pb = 0;
    styx_attn_workspace_bytes(d.n_heads, d.head_dim, &pb);
    w.part = take(pb);
    w.opart = take(static_cast<size_t>(d.n_kv_heads) * H * 4);   // cluster form: each cluster's o rows
    w.ccnt = take(styx::kClusterMaxC * styx::kCntStride * 4);     // cluster form: row-block counters
    w.trace = take(kTraceCtas * styx::kAttnTraceStamps * 8);   // last: STYX_OPT_TRACE stamps
    w.total = o;
    return w;
}
}  // namespace

int styx_attn_block_workspace_bytes(const styx_attn_dims *dims, uint64_t *out) {
    NEED(dims && out && dims->n_embd > 0 && dims->n_heads > 0 && dims->n_kv_heads > 0 && dims->head_dim > 0,
         "bad dims");
    *out = attn_ws(*dims).total;
    return STYX_OK;
}

int styx_attn_block_workspace_init(styx_ctx *ctx, styx_stream stream, void *workspace, uint64_t workspace_bytes) {
    ENTER(ctx);
    NEED(workspace && workspace_bytes > 0, "null workspace");
    CK(cudaMemsetAsync(workspace, 0, workspace_bytes, S(stream)));
    return STYX_OK;
}

namespace {
// The single-kernel plan (attn_fused.cu) for these dims / formats at n_t
// cache rows; false when it does not apply (the caller runs seven kernels).
bool plan_attn_fused(const styx_attn_dims &d, const styx_attn_layer &lw, int sms, int n_t, styx::AttnFusedArgs &a,
                     uint32_t &smem) {
    const int H = d.n_embd, hd = d.head_dim, nh = d.n_heads, nkv = d.n_kv_heads;
    if (hd != 128 || nh > sms || nh % nkv || nh / nkv > 16 || H > 2048 || H % 256) return false;
    const int qw = lw.wq.qtype, qv = lw.wv.qtype;
    if (lw.wk.qtype != qw || lw.wo.qtype != qw || !styx::attn_fused_supported(qw, qv)) return false;
    const int qd = nh * hd, kvd = nkv * hd, gqa = nh / nkv;
    if (!units_ok(qw, H) || !units_ok(qv, H) || !units_ok(qw, qd)) return false;
    a.rb_q = static_cast<int>(row_bytes(qw, H));
    a.rb_v = static_cast<int>(row_bytes(qv, H));
    a.rb_o = static_cast<int>(row_bytes(qw, qd));
    // splits of the sequence over the CTAs of each kv head, >= 16 rows each
    int S = std::max(1, std::min(sms / nkv, (n_t + 15) / 16));
    a.tps = (n_t + S - 1) / S;
    S = (n_t + a.tps - 1) / a.tps;
    a.n_splits = S;
    const int R = qd + 2 * kvd, dmax = std::max(H, qd);
    const size_t dig = static_cast<size_t>(dmax) * 3 + dmax / 32 * 4;
    const size_t w1_rows = static_cast<size_t>((R + sms - 1) / sms) * std::max(a.rb_q, a.rb_v) + 3 * 32;
    const size_t w1_attn = (static_cast<size_t>(gqa) * hd + 2 * hd) * 4 + 64 * 16 +
                           (static_cast<size_t>(a.tps) * gqa + ((2 * gqa + 3) & ~3)) * 4 + 8 * 8 * 128 * 4;
    const size_t w2 = static_cast<size_t>((H + sms - 1) / sms) * a.rb_o + 32;
    a.off_dig = 256;
    a.off_f32 = static_cast<uint32_t>(a16(a.off_dig + dig));
    a.off_w1 = static_cast<uint32_t>(a128(a.off_f32 + static_cast<size_t>(dmax) * 4));
    a.off_w2 = static_cast<uint32_t>(a128(a.off_w1 + std::max(w1_rows, w1_attn)));
    a.off_kv = static_cast<uint32_t>(a128(a.off_w2 + w2));
    a.off_rope = static_cast<uint32_t>(a128(a.off_kv + 2 * static_cast<size_t>(styx::kPreRows) * hd * 4));
    const size_t total = a.off_rope + static_cast<size_t>(hd / 2) * 16;   // the RoPE table (double cos, sin)
    if (total > 227 * 1024) return false;
    smem = static_cast<uint32_t>(total);
    return true;
}
}  // namespace

namespace {
// The cluster-form plan (attn_cluster.cu) for these dims / formats at n_t
// cache rows; false when it does not apply.  One cluster of 16 CTAs per kv
// head (8, 4, 2 when the device holds fewer of 16 at once); the Wo columns of
// a cluster's heads are a whole number of blocks on 16-byte boundaries.
bool plan_attn_cluster(const styx_attn_dims &d, const styx_attn_layer &lw, int sms, int n_t,
                       styx::AttnClusterArgs &a, uint32_t &smem) {
    const int H = d.n_embd, hd = d.head_dim, nh = d.n_heads, nkv = d.n_kv_heads;
    if (hd != 128 || nh % nkv || H % 64 || H > 2048) return false;
    const int gqa = nh / nkv, nq = gqa * hd;
    const int qw = lw.wq.qtype, qv = lw.wv.qtype;
    if (lw.wk.qtype != qw || lw.wo.qtype != qw || !styx::attn_cluster_supported(qw, qv)) return false;
    if (!units_ok(qw, H) || !units_ok(qv, H) || !units_ok(qw, nq) || nq / 64 > 32) return false;
    a.rb_q = static_cast<int>(row_bytes(qw, H));
    a.rb_v = static_cast<int>(row_bytes(qv, H));
    a.rb_o = static_cast<int>(row_bytes(qw, nh * hd));
    const long long blk_o = row_bytes(qw, nq);
    if (blk_o * nkv != a.rb_o || blk_o % 16 || a.rb_o % 16 || !al16(lw.wo.data)) return false;
    for (int C = styx::kClusterMaxC; C >= 2; C >>= 1) {
        if (gqa > C || nkv * C > sms) continue;
        a.C = C;
        a.tps = (n_t + C - 1) / C;
        if (a.tps > 512) return false;
        a.npre = std::min(a.tps, 48);
        const int nqr = (nq + C - 1) / C, nkr = (hd + C - 1) / C, nor = (H + C - 1) / C;
        const int hpw = std::max(1, 16 / gqa);
        size_t o = styx::kAttnClusterHeader;
        auto take = [&](size_t n) {
            const size_t r = o;
            o = a128(o + n);
            return static_cast<uint32_t>(r);
        };
        a.off_x = take(static_cast<size_t>(H) * 4);
        a.off_dig = take(3 * static_cast<size_t>(H) + H / 32 * 4);
        a.off_q = take((static_cast<size_t>(nq) + 2 * hd) * 4);
        a.off_rope = take(hd / 2 * 16);
        a.off_sc = take((((static_cast<size_t>(a.tps) * gqa + 3) & ~size_t(3)) + 2 * gqa) * 4);
        a.off_acc = take(static_cast<size_t>(hpw) * gqa * hd * 4);
        a.off_mrecv = take(static_cast<size_t>(C) * 132 * 4);
        a.off_att = take(static_cast<size_t>(nq) * 4);
        a.off_adig = take(3 * static_cast<size_t>(nq) + nq / 32 * 4);
        a.off_o = take(static_cast<size_t>(nor) * 4);
        const size_t wqkv = static_cast<size_t>(nqr) * a.rb_q + static_cast<size_t>(nkr) * (a.rb_q + a.rb_v) + 96;
        a.off_w = take(std::max(wqkv, static_cast<size_t>(nor) * static_cast<size_t>(blk_o)));
        a.off_kv = take(2 * static_cast<size_t>(a.npre) * hd * 4);
        if (o > 227 * 1024) continue;
        if (styx::attn_cluster_max_active(qw, qv, C, static_cast<uint32_t>(o)) < nkv) continue;
        smem = static_cast<uint32_t>(o);
        return true;
    }
    return false;
}
}  // namespace

int styx_attn_block(styx_ctx *ctx, styx_stream stream, const styx_attn_dims *dims, const styx_attn_layer *lw,
                    float *x, int pos, const int32_t *pos_dev, float *kcache, float *vcache, int n_ctx,
                    void *workspace, uint64_t workspace_bytes) {
    ENTER(ctx);
    NEED(dims && lw && x && pos_dev && kcache && vcache && workspace, "null pointer");
    const styx_attn_dims &d = *dims;
    NEED(d.n_embd > 0 && d.n_heads > 0 && d.n_kv_heads > 0 && d.n_heads % d.n_kv_heads == 0,
         "n_heads %d must be a multiple of n_kv_heads %d", d.n_heads, d.n_kv_heads);
    NEED(d.head_dim > 0 && d.head_dim % 4 == 0 && d.head_dim <= 256, "head_dim %d", d.head_dim);
    NEED(pos >= 0 && pos < n_ctx, "pos %d outside the caches (n_ctx %d)", pos, n_ctx);
    NEED(lw->attn_norm && lw->wq.data && lw->wk.data && lw->wv.data && lw->wo.data, "null weight");
    NEED(!d.qk_norm || (lw->q_norm && lw->k_norm), "qk_norm without q_norm / k_norm");
    const AttnWs w = attn_ws(d);
    NEED(workspace_bytes >= w.total && al16(workspace), "workspace: %llu bytes, 16-byte aligned, needed",
         static_cast<unsigned long long>(w.total));
    uint8_t *ws = static_cast<uint8_t *>(workspace);
    const int H = d.n_embd, hd = d.head_dim, qd = d.n_heads * hd, kvd = d.n_kv_heads * hd;
    float *xn = reinterpret_cast<float *>(ws + w.xnorm), *q = reinterpret_cast<float *>(ws + w.qkv);
    float *k = q + qd, *v = k + kvd;
    float *att = reinterpret_cast<float *>(ws + w.att);
    NEED(al16(kcache) && al16(vcache), "caches must be 16-byte aligned");
    NEED(extent_ok(kcache, static_cast<uint64_t>(n_ctx) * kvd * 4) &&
             extent_ok(vcache, static_cast<uint64_t>(n_ctx) * kvd * 4),
         "caches smaller than n_ctx rows");
    NEED(extent_ok(x, static_cast<uint64_t>(H) * 4) && extent_ok(lw->attn_norm, static_cast<uint64_t>(H) * 4),
         "x / attn_norm smaller than n_embd");
    int rc;
    // auto: one cooperative kernel when the shape fits, else the cluster form
    // when it fits, else seven launches (on B200 the cooperative kernel is
    // the faster of the two one-launch forms at the 30B-A3B shape)
    styx::AttnFusedArgs fa{};
    uint32_t fsmem = 0;
    const bool fused_fits = ctx->attn_kernels == 0 && plan_attn_fused(d, *lw, ctx->sm_count, pos + 1, fa, fsmem);
    if ((ctx->attn_kernels == 0 && !fused_fits) || ctx->attn_kernels == 3) {
        styx::AttnClusterArgs a{};
        uint32_t smem = 0;
        const bool fits = al16(x) && al16(lw->attn_norm) && plan_attn_cluster(d, *lw, ctx->sm_count, pos + 1, a, smem);
        if (!fits && ctx->attn_kernels == 3)
            return fail(STYX_EUNSUPPORTED, "cluster attention does not fit these dims / formats");
        if (fits) {
            NEED(extent_ok(lw->wq.data, static_cast<uint64_t>(a.rb_q) * qd) &&
                     extent_ok(lw->wk.data, static_cast<uint64_t>(a.rb_q) * kvd) &&
                     extent_ok(lw->wv.data, static_cast<uint64_t>(a.rb_v) * kvd) &&
                     extent_ok(lw->wo.data, static_cast<uint64_t>(a.rb_o) * H),
                 "a weight matrix is smaller than its shape");
            a.x = x;
            a.attn_norm = lw->attn_norm;
            a.eps = d.rms_eps;
            a.wq = static_cast<const uint8_t *>(lw->wq.data);
            a.wk = static_cast<const uint8_t *>(lw->wk.data);
            a.wv = static_cast<const uint8_t *>(lw->wv.data);
            a.wo = static_cast<const uint8_t *>(lw->wo.data);
            a.H = H;
            a.n_heads = d.n_heads;
            a.n_kv = d.n_kv_heads;
            a.q_norm = d.qk_norm ? lw->q_norm : nullptr;
            a.k_norm = d.qk_norm ? lw->k_norm : nullptr;
            a.theta_scale = std::pow(static_cast<double>(d.rope_base), -2.0 / static_cast<double>(hd));
            a.scale = 1.0f / std::sqrt(static_cast<float>(hd));
            a.n_t = pos + 1;
            a.kcache = kcache;
            a.vcache = vcache;
            a.opart = reinterpret_cast<float *>(ws + w.opart);
            a.cnt = reinterpret_cast<unsigned *>(ws + w.ccnt);
            a.err = ctx->d_err;
            a.trace = ctx->trace ? reinterpret_cast<long long *>(ws + w.trace) : nullptr;
            CK(styx::launch_attn_cluster(a, lw->wq.qtype, lw->wv.qtype, smem, S(stream)));
            ctx->attn_last_path = 3;
            return STYX_OK;
        }
    }
    if (ctx->attn_kernels != 2 && ctx->attn_kernels != 3) {
        styx::AttnFusedArgs a{};
        uint32_t smem = 0;
        const bool fits = plan_attn_fused(d, *lw, ctx->sm_count, pos + 1, a, smem);
        if (!fits && ctx->attn_kernels == 1)
            return fail(STYX_EUNSUPPORTED, "single-kernel attention does not fit these dims / formats");
        if (fits) {
            const int qw = lw->wq.qtype, qv = lw->wv.qtype;
            NEED(extent_ok(lw->wq.data, static_cast<uint64_t>(a.rb_q) * qd) &&
                     extent_ok(lw->wk.data, static_cast<uint64_t>(a.rb_q) * kvd) &&
                     extent_ok(lw->wv.data, static_cast<uint64_t>(a.rb_v) * kvd) &&
                     extent_ok(lw->wo.data, static_cast<uint64_t>(a.rb_o) * H),
                 "a weight matrix is smaller than its shape");
            a.x = x;
            a.attn_norm = lw->attn_norm;
            a.eps = d.rms_eps;
            a.wq = static_cast<const uint8_t *>(lw->wq.data);
            a.wk = static_cast<const uint8_t *>(lw->wk.data);
            a.wv = static_cast<const uint8_t *>(lw->wv.data);
            a.wo = static_cast<const uint8_t *>(lw->wo.data);
            a.H = H;
            a.n_heads = d.n_heads;
            a.n_kv = d.n_kv_heads;
            a.q_norm = d.qk_norm ? lw->q_norm : nullptr;
            a.k_norm = d.qk_norm ? lw->k_norm : nullptr;
            a.theta_scale = std::pow(static_cast<double>(d.rope_base), -2.0 / static_cast<double>(hd));
            a.scale = 1.0f / std::sqrt(static_cast<float>(hd));
            a.n_t = pos + 1;
            a.kcache = kcache;
            a.vcache = vcache;
            a.qkv = q;
            a.part_acc = reinterpret_cast<float *>(ws + w.part);
            a.part_ml = a.part_acc + static_cast<size_t>(d.n_heads) * a.n_splits * hd;
            // att as digits, in the att region (3 bytes + 1/8 float per element)
            a.att_d1 = reinterpret_cast<int8_t *>(att);
            a.att_d2 = reinterpret_cast<uint8_t *>(att) + qd;
            a.att_d3 = a.att_d2 + qd;
            a.att_sc = reinterpret_cast<float *>(a.att_d3 + qd);
            a.gen = reinterpret_cast<unsigned long long *>(ws + w.cnt);
            a.head_cnt = a.gen + 1;
            a.split_cnt = a.head_cnt + d.n_heads + 2 * d.n_kv_heads;
            a.att_cnt = a.split_cnt + d.n_kv_heads;
            a.err = ctx->d_err;
            a.trace = ctx->trace && ctx->sm_count <= static_cast<int>(kTraceCtas)
                          ? reinterpret_cast<long long *>(ws + w.trace)
                          : nullptr;
            CK(styx::launch_attn_fused(a, qw, qv, ctx->sm_count, smem, !ctx->exclusive, S(stream)));
            ctx->attn_last_path = 1;
            return STYX_OK;
        }
    }
    ctx->attn_last_path = 2;
    if ((rc = styx_rms_norm(ctx, stream, x, lw->attn_norm, d.rms_eps, H, 1, xn))) return rc;
    if ((rc = styx_mul_mat_vec(ctx, stream, lw->wq.qtype, lw->wq.data, qd, H, xn, q))) return rc;
    if ((rc = styx_mul_mat_vec(ctx, stream, lw->wk.qtype, lw->wk.data, kvd, H, xn, k))) return rc;
    if ((rc = styx_mul_mat_vec(ctx, stream, lw->wv.qtype, lw->wv.data, kvd, H, xn, v))) return rc;
    if ((rc = styx_qk_norm_rope_kv(ctx, stream, q, k, v, d.qk_norm ? lw->q_norm : nullptr,
                                   d.qk_norm ? lw->k_norm : nullptr, d.rms_eps, d.n_heads, d.n_kv_heads, hd, 1,
                                   d.rope_base, pos_dev, kcache, vcache, n_ctx)))
        return rc;
    if ((rc = styx_attn_decode(ctx, stream, q, kcache, vcache, att, pos + 1, hd, kvd, d.n_heads / d.n_kv_heads,
                               1.0f / std::sqrt(static_cast<float>(hd)), ws + w.part, workspace_bytes - w.part)))
        return rc;
    return styx_mul_mat_vec_add(ctx, stream, lw->wo.qtype, lw->wo.data, H, qd, att, x);   // x += o, rec_add fused
}

int styx_get_rows(styx_ctx *ctx, styx_stream stream, int qtype, const void *w, int nrows, int ncols,
                  const int32_t *rows, int n, float *out) {
    ENTER(ctx);
    NEED(w && rows && out && nrows > 0 && n > 0, "bad get_rows arguments");
    const long long rb = row_bytes(qtype, ncols);
    NEED(rb > 0, "ncols %d not representable in qtype %d", ncols, qtype);
    NEED(extent_ok(w, static_cast<uint64_t>(rb) * nrows), "matrix smaller than nrows rows");
    NEED(extent_ok(out, static_cast<uint64_t>(n) * ncols * 4) && extent_ok(rows, static_cast<uint64_t>(n) * 4),
         "rows / out smaller than n");
    styx::GetRowsArgs a{};
    a.w = static_cast<const uint8_t *>(w);
    a.row_bytes = rb;
    a.qtype = qtype;
    a.nrows = nrows;
    a.ncols = ncols;
    a.rows = rows;
    a.n = n;
    a.out = out;
    a.err = ctx->d_err;
    CK(styx::launch_get_rows(a, S(stream)));
    return STYX_OK;
}

int styx_argmax_f32(styx_ctx *ctx, styx_stream stream, const float *x, int n, int32_t *out) {
    ENTER(ctx);
    NEED(x && out && n > 0, "bad argmax arguments");
    NEED(extent_ok(x, static_cast<uint64_t>(n) * 4), "x smaller than n");
    CK(styx::launch_argmax(x, n, out, ctx->d_scratch, S(stream)));
    return STYX_OK;
}
