// The C ABI (include/mako_attn.h): argument checks, the context's scratch, kernel choice, launch.  Replaces the
// attention slice of mako-common's gpu::Runtime (scratch by name src/gpu/runtime.cpp:117-125, dispatch :243-259,
// error check in finish :453-475) and of TransformerRuntime (src/models/runtime.cpp:262-317).
#include "kernels.h"
#include "mako_attn.h"

#include <cuda_runtime.h>

#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <new>
#include <string>
#include <unordered_map>
#include <utility>
#include <vector>

struct mako_attn_ctx {
    int device = 0;
    int num_sms = 148;
    int cc_major = 0;
    int* err = nullptr;      // device flag the pipelined kernels set when a wait times out
    int prefill_kernel = 0;  // MAKO_OPT_PREFILL_KERNEL
    int decode_route = 1;    // MAKO_OPT_DECODE_ROUTE
    uint32_t decode_chunk = 0;  // MAKO_OPT_DECODE_CHUNK
    uint64_t launches = 0;   // kernels enqueued
    bool timing = false;     // MAKO_OPT_KERNEL_TIMING
    bool out16 = false;      // MAKO_OPT_OUTPUT_16BIT
    int grid_ctas = 0;       // MAKO_OPT_GRID_CTAS
    // CTAs of a persistent kernel's grid: one per SM, or fewer when MAKO_OPT_GRID_CTAS asks
    uint32_t persistent_ctas() const { return uint32_t(grid_ctas > 0 && grid_ctas < num_sms ? grid_ctas : num_sms); }
    std::vector<std::pair<cudaEvent_t, cudaEvent_t>> events;  // main-kernel event pairs, [0, used) recorded
    size_t used = 0;
    struct Buf {
        void* ptr = nullptr;
        size_t bytes = 0;
    };
    std::unordered_map<std::string, Buf> scratch;
};

namespace {
thread_local std::string g_error;
} // namespace

namespace mako {
int set_error(int code, const char* fmt, ...)
{
    char buf[512];
    va_list ap;
    va_start(ap, fmt);
    std::vsnprintf(buf, sizeof(buf), fmt, ap);
    va_end(ap);
    g_error = buf;
    return code;
}
void clear_error() { g_error.clear(); }
} // namespace mako

namespace {

template <typename... A>
int fail(int code, const char* fmt, A... args)
{
    return mako::set_error(code, fmt, args...);
}

int cuda_fail(const char* what, cudaError_t e)
{
    return fail(MAKO_ECUDA, "%s: %s (%s)", what, cudaGetErrorString(e), cudaGetErrorName(e));
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }
// Element type of o for a call of `dtype`: 0 fp32, else the call's 16-bit type (MAKO_OPT_OUTPUT_16BIT).
uint32_t out_type(const mako_attn_ctx* ctx, int dtype) { return ctx->out16 ? (dtype == MAKO_BF16 ? 2u : 1u) : 0u; }

// Runs the calls of one entry point with the context's device current, the caller's device restored after.
struct DeviceGuard {
    int prev = -1;
    cudaError_t err = cudaSuccess;
    explicit DeviceGuard(int dev)
    {
        if ((err = cudaGetDevice(&prev)) == cudaSuccess && prev != dev)
            err = cudaSetDevice(dev);
    }
    ~DeviceGuard()
    {
        int cur;
        if (prev >= 0 && cudaGetDevice(&cur) == cudaSuccess && cur != prev)
            cudaSetDevice(prev);
    }
};

// A named scratch buffer of at least `bytes`, grown (never shrunk) on demand like gpu::Runtime::scratch.
int scratch(mako_attn_ctx* ctx, const char* name, size_t bytes, void** out)
{
    auto& b = ctx->scratch[name];
    if (b.bytes < bytes) {
        if (b.ptr) {
            cudaError_t e = cudaFree(b.ptr);  // synchronises with work still reading it
            b.ptr = nullptr;
            b.bytes = 0;
            if (e != cudaSuccess)
                return cuda_fail("scratch free", e);
        }
        cudaError_t e = cudaMalloc(&b.ptr, bytes);
        if (e != cudaSuccess) {
            b.ptr = nullptr;
            cudaGetLastError();
            return fail(MAKO_ENOMEM, "scratch %s: %zu bytes: %s", name, bytes, cudaGetErrorString(e));
        }
        b.bytes = bytes;
    }
    *out = b.ptr;
    return MAKO_OK;
}

int check_ctx(mako_attn_ctx* ctx, int dtype)
{
    if (!ctx)
        return fail(MAKO_EINVAL, "null context");
    if (dtype != MAKO_F16 && dtype != MAKO_BF16)
        return fail(MAKO_EINVAL, "element type %d (MAKO_F16 or MAKO_BF16)", dtype);
    return MAKO_OK;
}

// Brackets a call's main kernel with a recorded event pair when the context times kernels (no-op otherwise).
struct KernelTimer {
    mako_attn_ctx* ctx;
    cudaStream_t st;
    bool on = false;
    KernelTimer(mako_attn_ctx* c, cudaStream_t s) : ctx(c), st(s)
    {
        if (!ctx->timing)
            return;
        if (ctx->used == ctx->events.size()) {
            cudaEvent_t a, b;
            if (cudaEventCreate(&a) != cudaSuccess)
                return;
            if (cudaEventCreate(&b) != cudaSuccess) {
                cudaEventDestroy(a);
                return;
            }
            ctx->events.emplace_back(a, b);
        }
        on = cudaEventRecord(ctx->events[ctx->used].first, st) == cudaSuccess;
    }
    void stop()
    {
        if (on && cudaEventRecord(ctx->events[ctx->used].second, st) == cudaSuccess)
            ++ctx->used;
        on = false;
    }
};

int launched(const char* what, cudaError_t e)
{
    if (e != cudaSuccess)
        return cuda_fail(what, e);
    g_error.clear();
    return MAKO_OK;
}

} // namespace

extern "C" {

const char* mako_attn_last_error(void) { return g_error.c_str(); }

int mako_attn_version(void) { return MAKO_ATTN_VERSION; }

int mako_attn_create(int device, mako_attn_ctx** out)
{
    if (!out)
        return fail(MAKO_EINVAL, "null output pointer");
    *out = nullptr;
    int n = 0;
    cudaError_t e = cudaGetDeviceCount(&n);
    if (e != cudaSuccess)
        return cuda_fail("cudaGetDeviceCount", e);
    if (device < 0 || device >= n)
        return fail(MAKO_EINVAL, "device %d of %d", device, n);
    cudaDeviceProp prop;
    if ((e = cudaGetDeviceProperties(&prop, device)) != cudaSuccess)
        return cuda_fail("cudaGetDeviceProperties", e);
    auto* ctx = new (std::nothrow) mako_attn_ctx;
    if (!ctx)
        return fail(MAKO_ENOMEM, "context");
    ctx->device = device;
    ctx->num_sms = prop.multiProcessorCount;
    ctx->cc_major = prop.major;
    {
        DeviceGuard dg(device);
        if ((e = cudaMalloc(&ctx->err, sizeof(int))) != cudaSuccess ||
            (e = cudaMemset(ctx->err, 0, sizeof(int))) != cudaSuccess) {
            if (ctx->err)
                cudaFree(ctx->err);
            delete ctx;
            return cuda_fail("context error flag", e);
        }
    }
    *out = ctx;
    g_error.clear();
    return MAKO_OK;
}

int mako_attn_destroy(mako_attn_ctx* ctx)
{
    if (!ctx)
        return MAKO_OK;
    int rc = MAKO_OK;
    {
        DeviceGuard dg(ctx->device);
        if (ctx->err)
            cudaFree(ctx->err);
        for (auto& ev : ctx->events) {
            cudaEventDestroy(ev.first);
            cudaEventDestroy(ev.second);
        }
        for (auto& kv : ctx->scratch)
            if (kv.second.ptr) {
                cudaError_t e = cudaFree(kv.second.ptr);
                if (e != cudaSuccess && rc == MAKO_OK)
                    rc = cuda_fail("scratch free", e);
            }
    }
    delete ctx;
    return rc;
}

int mako_attn_set_option(mako_attn_ctx* ctx, int option, int64_t value)
{
    if (!ctx)
        return fail(MAKO_EINVAL, "null context");
    switch (option) {
    case MAKO_OPT_PREFILL_KERNEL:
        if (value < 0 || value > 2)
            return fail(MAKO_EINVAL, "prefill kernel %lld (0 auto, 1 mma.sync, 2 tcgen05)", (long long)value);
        ctx->prefill_kernel = int(value);
        return MAKO_OK;
    case MAKO_OPT_DECODE_ROUTE:
        ctx->decode_route = value != 0;
        return MAKO_OK;
    case MAKO_OPT_KERNEL_TIMING:
        ctx->timing = value != 0;
        return MAKO_OK;
    case MAKO_OPT_OUTPUT_16BIT:
        ctx->out16 = value != 0;
        return MAKO_OK;
    case MAKO_OPT_GRID_CTAS:
        if (value < 0 || value > (int64_t(1) << 20))
            return fail(MAKO_EINVAL, "grid CTAs %lld (0: one per SM)", (long long)value);
        ctx->grid_ctas = int(value);
        return MAKO_OK;
    case MAKO_OPT_DECODE_CHUNK:
        if (value < 0 || value % 64 || value > (int64_t(1) << 30))
            return fail(MAKO_EINVAL, "decode chunk %lld (0 or a multiple of 64)", (long long)value);
        ctx->decode_chunk = uint32_t(value);
        return MAKO_OK;
    default:
        return fail(MAKO_EINVAL, "option %d", option);
    }
}

int mako_attn_launches(mako_attn_ctx* ctx, uint64_t* out)
{
    if (!ctx || !out)
        return fail(MAKO_EINVAL, "null argument");
    *out = ctx->launches;
    return MAKO_OK;
}

int mako_attn_kernel_times(mako_attn_ctx* ctx, float* ms, uint32_t cap, uint32_t* n)
{
    if (!ctx || !n || (cap && !ms))
        return fail(MAKO_EINVAL, "null argument");
    DeviceGuard dg(ctx->device);
    uint32_t k = 0;
    for (size_t i = 0; i < ctx->used; ++i) {
        float t = 0.0f;
        cudaError_t e = cudaEventSynchronize(ctx->events[i].second);
        if (e == cudaSuccess)
            e = cudaEventElapsedTime(&t, ctx->events[i].first, ctx->events[i].second);
        if (e != cudaSuccess) {
            ctx->used = 0;
            return cuda_fail("kernel times", e);
        }
        if (k < cap)
            ms[k] = t;
        ++k;
    }
    ctx->used = 0;
    *n = k;
    return MAKO_OK;
}

int mako_attn_device_error(mako_attn_ctx* ctx, int* out)
{
    if (!ctx || !out)
        return fail(MAKO_EINVAL, "null argument");
    DeviceGuard dg(ctx->device);
    int v = 0;
    cudaError_t e = cudaMemcpy(&v, ctx->err, sizeof(int), cudaMemcpyDeviceToHost);
    if (e != cudaSuccess)
        return cuda_fail("read device error flag", e);
    if (v && (e = cudaMemset(ctx->err, 0, sizeof(int))) != cudaSuccess)
        return cuda_fail("reset device error flag", e);
    *out = v;
    return MAKO_OK;
}

int mako_attention(mako_attn_ctx* ctx, void* stream, int dtype, const void* q, const void* k, const void* v, float* o,
                   uint32_t n_q, uint32_t q_pad, uint32_t n_k, uint32_t k_pad, uint32_t heads, uint32_t kv_heads,
                   uint32_t q_pos0, uint32_t block, uint32_t dim, uint32_t width)
{
    if (int rc = check_ctx(ctx, dtype))
        return rc;
    if (dim != 64 && dim != 128 && dim != 256)
        return fail(MAKO_EINVAL, "attention: heads of %u", dim);
    if (width == 0)
        width = heads * dim;
    if (!heads || !kv_heads || heads % kv_heads)
        return fail(MAKO_EINVAL, "attention: %u heads over %u kv heads", heads, kv_heads);
    if (q_pad % 64 || q_pad < n_q || k_pad < n_k)
        return fail(MAKO_EINVAL, "attention: q_pad %u (a multiple of 64, at least n_q %u), k_pad %u (at least n_k %u)",
                    q_pad, n_q, k_pad, n_k);
    if (width < heads * dim)
        return fail(MAKO_EINVAL, "attention: o rows of %u floats for %u heads of %u", width, heads, dim);
    if (!q || !k || !v || !o || !aligned16(q) || !aligned16(k) || !aligned16(v) || !aligned16(o))
        return fail(MAKO_EINVAL, "attention: null or unaligned tensor (16-byte alignment)");
    // the prefill kernels store o rows 16 bytes at a time: rows keep o's alignment
    if (!(n_q == 1 && ctx->decode_route) && width % (ctx->out16 ? 8 : 4))
        return fail(MAKO_EINVAL, "attention: o row width %u (a multiple of %d)", width, ctx->out16 ? 8 : 4);
    if (n_q == 0)
        return MAKO_OK;
    DeviceGuard dg(ctx->device);
    if (dg.err != cudaSuccess)
        return cuda_fail("set device", dg.err);
    auto st = static_cast<cudaStream_t>(stream);
    if (n_q == 1 && ctx->decode_route) {
        // One query: the keys it sees are a prefix [0, len) (mask predicate at pos = q_pos0).
        const uint32_t len = q_pos0 >= block ? n_k : (n_k < q_pos0 + 1 ? n_k : q_pos0 + 1);
        mako::DecodeParams p{};
        p.q = q;
        p.k = k;
        p.v = v;
        p.o = o;
        p.kv_len = nullptr;
        p.len = len;
        p.q_bstride = 0;
        p.q_hstride = uint64_t(q_pad) * dim;
        p.k_bstride = 0;
        p.k_hstride = uint64_t(k_pad) * dim;
        p.o_bstride = width;
        p.o_type = out_type(ctx, dtype);
        p.batch = 1;
        p.heads = heads;
        p.kv_heads = kv_heads;
        p.scale = 1.0f / sqrtf(float(dim));
        mako::decode_plan(len, 1, kv_heads, heads, ctx->num_sms, ctx->decode_chunk, &p.chunk, &p.n_splits);
        void *op, *mlp;
        if (int rc = scratch(ctx, "dec_o", size_t(heads) * p.n_splits * dim * 4, &op))
            return rc;
        if (int rc = scratch(ctx, "dec_ml", size_t(heads) * p.n_splits * 8, &mlp))
            return rc;
        p.o_part = static_cast<float*>(op);
        p.ml_part = static_cast<float2*>(mlp);
        ctx->launches += 2;
        KernelTimer t(ctx, st);
        cudaError_t e = mako::launch_decode_split(p, dtype, int(dim), st);
        t.stop();
        if (e != cudaSuccess)
            return cuda_fail("attention (decode splits)", e);
        return launched("attention (decode combine)", mako::launch_decode_combine(p, int(dim), st));
    }
    mako::AttnParams p{};
    p.num_sms = ctx->persistent_ctas();
    p.q = q;
    p.k = k;
    p.v = v;
    p.o = o;
    p.n_q = n_q;
    p.q_pad = q_pad;
    p.n_k = n_k;
    p.k_pad = k_pad;
    p.heads = heads;
    p.kv_heads = kv_heads;
    p.q_pos0 = q_pos0;
    p.block = block;
    p.width = width;
    p.o_type = out_type(ctx, dtype);
    p.scale = 1.0f / sqrtf(float(dim));
    // The tcgen05 kernels are the path; the mma.sync kernels run only when asked for (MAKO_OPT_PREFILL_KERNEL 1, the
    // baseline the tests and benchmarks compare against), never as a silent substitute on another device.
    if (ctx->prefill_kernel != 1 && ctx->cc_major != 10)
        return fail(MAKO_ENOTSUP, "attention: the tcgen05 kernels need sm_100 (sm_%d)", ctx->cc_major * 10);
    if (ctx->prefill_kernel != 1) {
        void *v16 = nullptr, *vmax = nullptr, *vinv = nullptr;
        if (dtype == MAKO_BF16) {
            if (int rc = scratch(ctx, "v16", size_t(kv_heads) * k_pad * dim * 2, &v16))
                return rc;
            if (int rc = scratch(ctx, "vmax", size_t(kv_heads) * 4, &vmax))
                return rc;
            if (int rc = scratch(ctx, "vinv", size_t(kv_heads) * 4, &vinv))
                return rc;
            cudaError_t e = mako::launch_v_to_f16(v, v16, static_cast<uint32_t*>(vmax), static_cast<float*>(vinv),
                                                  dim, kv_heads, k_pad, n_k, nullptr, ctx->num_sms, st);
            if (e != cudaSuccess)
                return cuda_fail("attention (V to fp16)", e);
            ctx->launches += 2;
        }
        ctx->launches += 1;
        KernelTimer t(ctx, st);
        cudaError_t e = dim == 256 ? mako::launch_attn_tc256(p, dtype, v16, static_cast<const float*>(vinv), ctx->err, st)
                                   : mako::launch_attn_tc(p, dtype, int(dim), v16, static_cast<const float*>(vinv),
                                                          ctx->err, st);
        t.stop();
        return launched("attention (tcgen05)", e);
    }
    ctx->launches += 1;
    KernelTimer t(ctx, st);
    cudaError_t e = mako::launch_attn_mma(p, dtype, dim, false, false, st);
    t.stop();
    return launched("attention", e);
}

int mako_attention_decode(mako_attn_ctx* ctx, void* stream, int dtype, const void* q, const void* k, const void* v,
                          float* o, uint32_t batch, const int32_t* kv_len, uint32_t max_kv_len, uint32_t heads,
                          uint32_t kv_heads, uint32_t dim, uint32_t k_stride)
{
    if (int rc = check_ctx(ctx, dtype))
        return rc;
    if (dim != 64 && dim != 128 && dim != 256)
        return fail(MAKO_EINVAL, "decode: heads of %u", dim);
    if (!heads || !kv_heads || heads % kv_heads)
        return fail(MAKO_EINVAL, "decode: %u heads over %u kv heads", heads, kv_heads);
    if (max_kv_len > k_stride)
        return fail(MAKO_EINVAL, "decode: max_kv_len %u beyond the cache's %u rows", max_kv_len, k_stride);
    if (!q || !k || !v || !o || !kv_len || !aligned16(q) || !aligned16(k) || !aligned16(v) || !aligned16(o))
        return fail(MAKO_EINVAL, "decode: null or unaligned tensor (16-byte alignment)");
    if (batch == 0)
        return MAKO_OK;
    DeviceGuard dg(ctx->device);
    if (dg.err != cudaSuccess)
        return cuda_fail("set device", dg.err);
    mako::DecodeParams p{};
    p.q = q;
    p.k = k;
    p.v = v;
    p.o = o;
    p.kv_len = kv_len;
    p.len = max_kv_len;
    p.q_bstride = uint64_t(heads) * dim;
    p.q_hstride = dim;
    p.k_hstride = uint64_t(k_stride) * dim;
    p.k_bstride = uint64_t(kv_heads) * p.k_hstride;
    p.o_bstride = uint64_t(heads) * dim;
    p.o_type = out_type(ctx, dtype);
    p.batch = batch;
    p.heads = heads;
    p.kv_heads = kv_heads;
    p.scale = 1.0f / sqrtf(float(dim));
    mako::decode_plan(max_kv_len, batch, kv_heads, heads, ctx->num_sms, ctx->decode_chunk, &p.chunk, &p.n_splits);
    void *op, *mlp;
    if (int rc = scratch(ctx, "dec_o", size_t(batch) * heads * p.n_splits * dim * 4, &op))
        return rc;
    if (int rc = scratch(ctx, "dec_ml", size_t(batch) * heads * p.n_splits * 8, &mlp))
        return rc;
    p.o_part = static_cast<float*>(op);
    p.ml_part = static_cast<float2*>(mlp);
    ctx->launches += 2;
    auto st = static_cast<cudaStream_t>(stream);
    KernelTimer t(ctx, st);
    cudaError_t e = mako::launch_decode_split(p, dtype, int(dim), st);
    t.stop();
    if (e != cudaSuccess)
        return cuda_fail("decode (splits)", e);
    return launched("decode (combine)", mako::launch_decode_combine(p, int(dim), st));
}

int mako_cube_select(mako_attn_ctx* ctx, void* stream, int dtype, const void* q, const void* k, uint32_t heads,
                     uint32_t q_pad, uint32_t k_pad, uint32_t n_cubes, const uint32_t* cnt, uint32_t topk,
                     uint16_t** sel, uint16_t** nsel, uint32_t local, uint32_t stride)
{
    if (int rc = check_ctx(ctx, dtype))
        return rc;
    if (n_cubes > 4096 || !topk || (local != 0 && local != 1 && local != 3))
        return fail(MAKO_EINVAL, "cube_select: %u cubes, top %u, local %u", n_cubes, topk, local);
    if (uint64_t(n_cubes) * 64 > q_pad || uint64_t(n_cubes) * 64 > k_pad)
        return fail(MAKO_EINVAL, "cube_select: %u cubes of 64 rows beyond q_pad %u / k_pad %u", n_cubes, q_pad, k_pad);
    if (!q || !k || !cnt || !sel || !nsel || !aligned16(q) || !aligned16(k))
        return fail(MAKO_EINVAL, "cube_select: null or unaligned argument");
    DeviceGuard dg(ctx->device);
    if (dg.err != cudaSuccess)
        return cuda_fail("set device", dg.err);
    const uint32_t kk = topk < n_cubes ? topk : n_cubes;
    mako::CubeParams p{};
    void *qp, *kp, *sc, *s, *ns;
    const size_t nc = n_cubes ? n_cubes : 1;
    if (int rc = scratch(ctx, "c_qp", size_t(heads) * nc * 128 * 4, &qp))
        return rc;
    if (int rc = scratch(ctx, "c_kp", size_t(heads) * nc * 128 * 4, &kp))
        return rc;
    if (int rc = scratch(ctx, "c_sc", size_t(heads) * nc * nc * 4, &sc))
        return rc;
    if (int rc = scratch(ctx, "c_sel", size_t(heads) * nc * (kk ? kk : 1) * 2, &s))
        return rc;
    if (int rc = scratch(ctx, "c_nsel", size_t(heads) * nc * 2, &ns))
        return rc;
    p.q = q;
    p.k = k;
    p.cnt = cnt;
    p.qp = static_cast<float*>(qp);
    p.kp = static_cast<float*>(kp);
    p.sc = static_cast<float*>(sc);
    p.sel = static_cast<uint16_t*>(s);
    p.nsel = static_cast<uint16_t*>(ns);
    p.heads = heads;
    p.q_pad = q_pad;
    p.k_pad = k_pad;
    p.n_cubes = n_cubes;
    p.topk = topk;
    p.local = local;
    p.stride = stride;
    *sel = p.sel;
    *nsel = p.nsel;
    ctx->launches += n_cubes ? 3 : 0;
    return launched("cube_select", mako::launch_cube_select(p, dtype, static_cast<cudaStream_t>(stream)));
}

namespace {

int sparse_common(mako_attn_ctx* ctx, void* stream, int dtype, mako::AttnParams& p, bool sel_i32)
{
    if (p.width % (ctx->out16 ? 8 : 4))  // o rows are stored 16 bytes at a time
        return fail(MAKO_EINVAL, "attention_sparse: o row width %u (a multiple of %d)", p.width, ctx->out16 ? 8 : 4);
    DeviceGuard dg(ctx->device);
    if (dg.err != cudaSuccess)
        return cuda_fail("set device", dg.err);
    p.scale = 1.0f / sqrtf(128.0f);
    p.o_type = out_type(ctx, dtype);
    auto st = static_cast<cudaStream_t>(stream);
    if (ctx->prefill_kernel != 1 && ctx->cc_major != 10)
        return fail(MAKO_ENOTSUP, "attention_sparse: the tcgen05 kernel needs sm_100 (sm_%d)", ctx->cc_major * 10);
    if (ctx->prefill_kernel != 1) {
        void *v16 = nullptr, *vmax = nullptr, *vinv = nullptr;
        if (dtype == MAKO_BF16) {
            if (int rc = scratch(ctx, "v16", size_t(p.kv_heads) * p.k_pad * 128 * 2, &v16))
                return rc;
            if (int rc = scratch(ctx, "vmax", size_t(p.kv_heads) * 4, &vmax))
                return rc;
            if (int rc = scratch(ctx, "vinv", size_t(p.kv_heads) * 4, &vinv))
                return rc;
            cudaError_t e = mako::launch_v_to_f16(p.v, v16, static_cast<uint32_t*>(vmax), static_cast<float*>(vinv),
                                                  128, p.kv_heads, p.k_pad, p.k_pad, p.valid, ctx->num_sms, st);
            if (e != cudaSuccess)
                return cuda_fail("attention_sparse (V to fp16)", e);
            ctx->launches += 2;
        }
        ctx->launches += 1;
        KernelTimer t(ctx, st);
        cudaError_t e = mako::launch_attn_tc_sparse(p, dtype, sel_i32, v16, static_cast<const float*>(vinv), ctx->err,
                                                    st);
        t.stop();
        return launched("attention_sparse (tcgen05)", e);
    }
    ctx->launches += 1;
    KernelTimer t(ctx, st);
    cudaError_t e = mako::launch_attn_mma(p, dtype, 128, true, sel_i32, st);
    t.stop();
    return launched("attention_sparse", e);
}

} // namespace

int mako_attention_sparse(mako_attn_ctx* ctx, void* stream, int dtype, const void* q, const void* k, const void* v,
                          float* o, uint32_t n_q, uint32_t q_pad, uint32_t n_k, uint32_t k_pad, uint32_t heads,
                          uint32_t kv_heads, uint32_t width, uint32_t n_cubes, uint32_t topk, uint32_t dense0,
                          uint32_t dense1, const uint16_t* sel, const uint16_t* nsel, const uint8_t* valid,
                          const int32_t* map)
{
    if (int rc = check_ctx(ctx, dtype))
        return rc;
    if (q_pad % 64 || k_pad % 128 || dense0 % 32)
        return fail(MAKO_EINVAL, "attention_sparse: q_pad a multiple of 64, k_pad of 128, the dense rows from a "
                                 "multiple of 32");
    if (!heads || !kv_heads || heads % kv_heads)
        return fail(MAKO_EINVAL, "attention_sparse: %u heads over %u kv heads", heads, kv_heads);
    if (q_pad < n_q || k_pad < n_k || dense0 > dense1 || dense1 > k_pad || uint64_t(n_cubes) * 64 > q_pad ||
        uint64_t(n_cubes) * 64 > k_pad || width < heads * 128)
        return fail(MAKO_EINVAL, "attention_sparse: rows n_q %u q_pad %u n_k %u k_pad %u dense [%u, %u) cubes %u width %u",
                    n_q, q_pad, n_k, k_pad, dense0, dense1, n_cubes, width);
    if (!q || !k || !v || !o || !valid || !map || (n_cubes && (!sel || !nsel)) || !aligned16(q) || !aligned16(k) ||
        !aligned16(v) || !aligned16(o) || !aligned16(valid))
        return fail(MAKO_EINVAL, "attention_sparse: null or unaligned argument");
    if (n_q == 0)
        return MAKO_OK;
    mako::AttnParams p{};
    p.num_sms = ctx->persistent_ctas();
    p.q = q;
    p.k = k;
    p.v = v;
    p.o = o;
    p.n_q = n_q;
    p.q_pad = q_pad;
    p.n_k = n_k;
    p.k_pad = k_pad;
    p.heads = heads;
    p.kv_heads = kv_heads;
    p.width = width;
    p.n_cubes = n_cubes;
    p.max_sel = topk < n_cubes ? topk : n_cubes;
    p.dense0 = dense0;
    p.dense1 = dense1;
    p.sel = sel;
    p.nsel = nsel;
    p.valid = valid;
    p.map = map;
    return sparse_common(ctx, stream, dtype, p, false);
}

int mako_attention_block_sparse(mako_attn_ctx* ctx, void* stream, int dtype, const void* q, const void* k,
                                const void* v, float* o, uint32_t n, uint32_t heads, uint32_t kv_heads,
                                const int32_t* lists, const int32_t* counts, uint32_t max_list)
{
    if (int rc = check_ctx(ctx, dtype))
        return rc;
    if (n % 64 || !heads || !kv_heads || heads % kv_heads)
        return fail(MAKO_EINVAL, "block_sparse: %u rows (a multiple of 64), %u heads over %u kv heads", n, heads,
                    kv_heads);
    if (!q || !k || !v || !o || !lists || !counts || !aligned16(q) || !aligned16(k) || !aligned16(v) || !aligned16(o))
        return fail(MAKO_EINVAL, "block_sparse: null or unaligned argument");
    if (n == 0)
        return MAKO_OK;
    mako::AttnParams p{};
    p.num_sms = ctx->persistent_ctas();
    p.q = q;
    p.k = k;
    p.v = v;
    p.o = o;
    p.n_q = n;
    p.q_pad = n;
    p.n_k = n;
    p.k_pad = n;
    p.heads = heads;
    p.kv_heads = kv_heads;
    p.width = heads * 128;
    p.n_cubes = n / 64;
    p.max_sel = max_list;
    p.dense0 = n;
    p.dense1 = n;
    p.sel = lists;
    p.nsel = counts;
    p.valid = nullptr;
    p.map = nullptr;
    return sparse_common(ctx, stream, dtype, p, true);
}

} // extern "C"

// ---- head-tile producers --------------------------------------------------------------------------------------------

namespace {

int heads_common(mako_attn_ctx* ctx, void* stream, int dtype, mako::HeadsParams& p, const char* what)
{
    if (int rc = check_ctx(ctx, dtype))
        return rc;
    if (!p.x || !p.y || (p.rope && !p.cs) || (p.eps > 0.0f && !p.w) || !aligned16(p.y))
        return fail(MAKO_EINVAL, "%s: null argument or unaligned tile (16-byte alignment)", what);
    if (uint64_t(p.row0) + p.rows > p.n_pad)
        return fail(MAKO_EINVAL, "%s: rows %u + %u beyond n_pad %u", what, p.row0, p.rows, p.n_pad);
    if (!(p.eps >= 0.0f))
        return fail(MAKO_EINVAL, "%s: eps %g", what, double(p.eps));
    if (p.rows == 0 || p.heads == 0)
        return MAKO_OK;
    DeviceGuard dg(ctx->device);
    if (dg.err != cudaSuccess)
        return cuda_fail("set device", dg.err);
    p.vec4 = ((reinterpret_cast<uintptr_t>(p.x) & 15) == 0 && p.ld % 4 == 0 && p.col0 % 4 == 0 && p.stride % 4 == 0)
                 ? 1u
                 : 0u;
    ctx->launches += 1;
    auto st = static_cast<cudaStream_t>(stream);
    KernelTimer t(ctx, st);
    cudaError_t e = mako::launch_heads(p, dtype, st);
    t.stop();
    return launched(what, e);
}

int clear_rows(void* y, int dtype, uint32_t dim, uint32_t n_pad, uint32_t from, uint32_t heads, cudaStream_t st)
{
    if (from >= n_pad || heads == 0)
        return MAKO_OK;
    (void)dtype;  // both element types are 2 bytes
    const size_t pitch = size_t(n_pad) * dim * 2;
    cudaError_t e = cudaMemset2DAsync(static_cast<char*>(y) + size_t(from) * dim * 2, pitch, 0,
                                      size_t(n_pad - from) * dim * 2, heads, st);
    return e == cudaSuccess ? MAKO_OK : cuda_fail("heads_clear", e);
}

} // namespace

extern "C" {

int mako_heads(mako_attn_ctx* ctx, void* stream, int dtype, const float* x, uint32_t ld, uint32_t col0,
               uint32_t heads, uint32_t T, uint32_t n_pad, const float* cs, uint32_t rope, void* y)
{
    if (rope > 2)
        return fail(MAKO_EINVAL, "heads: rope %u (0 none, 1 halves, 2 adjacent pairs)", rope);
    if (T > n_pad)
        return fail(MAKO_EINVAL, "heads: %u rows beyond n_pad %u", T, n_pad);
    mako::HeadsParams p{};
    p.x = x;
    p.cs = cs;
    p.y = y;
    p.ld = ld;
    p.col0 = col0;
    p.stride = 128;
    p.dim = 128;
    p.rot = 128;
    p.rope = rope;
    p.rows = T;
    p.heads = heads;
    p.n_pad = n_pad;
    p.cs_row = 64;
    if (int rc = heads_common(ctx, stream, dtype, p, "heads"))
        return rc;
    if (T < n_pad && heads && y) {
        DeviceGuard dg(ctx->device);
        return clear_rows(y, dtype, 128, n_pad, T, heads, static_cast<cudaStream_t>(stream));
    }
    return MAKO_OK;
}

int mako_heads_norm(mako_attn_ctx* ctx, void* stream, int dtype, const float* x, uint32_t ld, uint32_t col0,
                    uint32_t heads, uint32_t T, uint32_t n_pad, const float* cs, uint32_t rope, const float* w,
                    float eps, uint32_t row0, void* y)
{
    if (rope > 2)
        return fail(MAKO_EINVAL, "heads_norm: rope %u (0 none, 1 halves, 2 adjacent pairs)", rope);
    if (!(eps > 0.0f))
        return fail(MAKO_EINVAL, "heads_norm: eps %g (positive)", double(eps));
    mako::HeadsParams p{};
    p.x = x;
    p.cs = cs;
    p.w = w;
    p.y = y;
    p.ld = ld;
    p.col0 = col0;
    p.stride = 128;
    p.dim = 128;
    p.rot = 128;
    p.rope = rope;
    p.rows = T;
    p.heads = heads;
    p.n_pad = n_pad;
    p.row0 = row0;
    p.cs_row = 64;
    p.eps = eps;
    return heads_common(ctx, stream, dtype, p, "heads_norm");
}

int mako_heads_partial(mako_attn_ctx* ctx, void* stream, int dtype, const float* x, uint32_t ld, uint32_t col0,
                       uint32_t stride, uint32_t dim, uint32_t rot, uint32_t heads, uint32_t T, uint32_t n_pad,
                       const float* cs, const float* w, float eps, void* y, const int32_t* map)
{
    // the reference's check and message (src/models/runtime.cpp:248-249), and rot within the head
    if (dim > 256 || dim % 32 || rot % 2 || dim == 0)
        return fail(MAKO_EINVAL, "heads_partial: heads of %u with %u rotated", dim, rot);
    if (rot > dim)
        return fail(MAKO_EINVAL, "heads_partial: %u rotated of a head of %u", rot, dim);
    if (T > n_pad)
        return fail(MAKO_EINVAL, "heads_partial: %u rows beyond n_pad %u", T, n_pad);
    mako::HeadsParams p{};
    p.x = x;
    p.cs = cs;
    p.w = w;
    p.map = map;
    p.y = y;
    p.ld = ld;
    p.col0 = col0;
    p.stride = stride;
    p.dim = dim;
    p.rot = rot;
    p.rope = rot ? 1u : 0u;
    p.rows = T;
    p.heads = heads;
    p.n_pad = n_pad;
    p.cs_row = rot / 2;
    p.eps = w ? eps : 0.0f;  // the reference normalises only when w is given
    if (w && !(eps > 0.0f))
        return fail(MAKO_EINVAL, "heads_partial: eps %g with a norm weight", double(eps));
    return heads_common(ctx, stream, dtype, p, "heads_partial");
}

int mako_proj(mako_attn_ctx* ctx, void* stream, int dtype, const void* w, const void* x, float* y, uint32_t T,
              uint32_t k, uint32_t n, uint32_t ldy)
{
    if (int rc = check_ctx(ctx, dtype))
        return rc;
    if (k % 64)  // the reference's own limit for its BF16 GEMM (src/gpu/runtime.cpp:178-179)
        return fail(MAKO_EINVAL, "BF16 %ux%u: k must be a multiple of 64", k, n);
    if (ldy == 0)
        ldy = n;
    if (ldy < n || !w || !x || !y || !aligned16(w) || !aligned16(x) || !aligned16(y) || ldy % 4)
        return fail(MAKO_EINVAL, "proj: null or unaligned tensor, or row stride %u under %u (16-byte aligned rows)", ldy,
                    n);
    if (ctx->cc_major != 10)
        return fail(MAKO_ENOTSUP, "proj: the tcgen05 GEMM needs sm_100 (sm_%d)", ctx->cc_major * 10);
    if (T == 0 || n == 0)
        return MAKO_OK;
    DeviceGuard dg(ctx->device);
    if (dg.err != cudaSuccess)
        return cuda_fail("set device", dg.err);
    mako::ProjParams p{};
    p.x = x;
    p.w = w;
    p.y = y;
    p.T = T;
    p.k = k;
    p.n = n;
    p.ldy = ldy;
    p.num_sms = ctx->persistent_ctas();
    auto st = static_cast<cudaStream_t>(stream);
    ctx->launches += 1;
    KernelTimer t(ctx, st);
    cudaError_t e = mako::launch_proj_gemm(p, dtype, ctx->err, st);
    t.stop();
    return launched("proj", e);
}

int mako_heads_clear(mako_attn_ctx* ctx, void* stream, int dtype, void* y, uint32_t dim, uint32_t n_pad, uint32_t from,
                     uint32_t heads)
{
    if (int rc = check_ctx(ctx, dtype))
        return rc;
    if (!y || !dim)
        return fail(MAKO_EINVAL, "heads_clear: null tile or zero width");
    DeviceGuard dg(ctx->device);
    if (dg.err != cudaSuccess)
        return cuda_fail("set device", dg.err);
    int rc = clear_rows(y, dtype, dim, n_pad, from, heads, static_cast<cudaStream_t>(stream));
    if (rc == MAKO_OK)
        g_error.clear();
    return rc;
}

} // extern "C"

// ---- multi-GPU ------------------------------------------------------------------------------------------------------

struct mako_attn_group {
    mako_attn_ctx* ctx = nullptr;
    uint32_t rank = 0, n_ranks = 1, rows_cap = 0;
    void* area = nullptr;                     // this rank's exchange area
    void* peer[MAKO_MAX_RANKS] = {};          // every rank's area as this process addresses it
    bool connected = false;
    bool mapped = false;                      // peers opened through IPC (closed on destroy)
    uint32_t epoch = 0;                       // collective calls so far (flags carry the call's number)
};

namespace {

static_assert(sizeof(cudaIpcMemHandle_t) == sizeof(mako_ipc_handle), "IPC handle size");
static_assert(MAKO_MAX_RANKS == mako::kMaxRanks, "rank limit");

mako::XchgParams xchg_params(mako_attn_group* g)
{
    mako::XchgParams x{};
    for (uint32_t r = 0; r < g->n_ranks; ++r)
        x.area[r] = static_cast<unsigned char*>(g->peer[r]);
    x.n_ranks = g->n_ranks;
    x.rank = g->rank;
    // 0 is the flags' initial value, never a call's number; after 0xFFFFFFFF (odd) comes 2 (even), so consecutive
    // calls keep alternating halves of the exchange area's parity double buffer across the wrap.
    if (++g->epoch == 0)
        g->epoch = 2;
    x.epoch = g->epoch;
    x.rows_cap = g->rows_cap;
    x.err = g->ctx->err;
    return x;
}

int check_group(mako_attn_group* g, int dtype)
{
    if (!g)
        return fail(MAKO_EINVAL, "null group");
    if (!g->connected)
        return fail(MAKO_EINVAL, "group not connected (mako_group_connect)");
    return check_ctx(g->ctx, dtype);
}

} // namespace

extern "C" {

int mako_peer_alloc(mako_attn_ctx* ctx, size_t bytes, void** ptr, mako_ipc_handle* handle)
{
    if (!ctx || !ptr || !handle || !bytes)
        return fail(MAKO_EINVAL, "peer_alloc: null argument or zero bytes");
    *ptr = nullptr;
    DeviceGuard dg(ctx->device);
    if (dg.err != cudaSuccess)
        return cuda_fail("set device", dg.err);
    void* p = nullptr;
    cudaError_t e = cudaMalloc(&p, bytes);
    if (e != cudaSuccess) {
        cudaGetLastError();
        return fail(MAKO_ENOMEM, "peer_alloc: %zu bytes: %s", bytes, cudaGetErrorString(e));
    }
    cudaIpcMemHandle_t h;
    if ((e = cudaIpcGetMemHandle(&h, p)) != cudaSuccess) {
        cudaFree(p);
        return cuda_fail("peer_alloc: cudaIpcGetMemHandle", e);
    }
    std::memcpy(handle->bytes, &h, sizeof(h));
    *ptr = p;
    g_error.clear();
    return MAKO_OK;
}

int mako_peer_free(mako_attn_ctx* ctx, void* ptr)
{
    if (!ctx)
        return fail(MAKO_EINVAL, "peer_free: null context");
    if (!ptr)
        return MAKO_OK;
    DeviceGuard dg(ctx->device);
    cudaError_t e = cudaFree(ptr);
    return e == cudaSuccess ? (g_error.clear(), MAKO_OK) : cuda_fail("peer_free", e);
}

int mako_peer_open(mako_attn_ctx* ctx, const mako_ipc_handle* handle, void** ptr)
{
    if (!ctx || !handle || !ptr)
        return fail(MAKO_EINVAL, "peer_open: null argument");
    *ptr = nullptr;
    DeviceGuard dg(ctx->device);
    if (dg.err != cudaSuccess)
        return cuda_fail("set device", dg.err);
    cudaIpcMemHandle_t h;
    std::memcpy(&h, handle->bytes, sizeof(h));
    cudaError_t e = cudaIpcOpenMemHandle(ptr, h, cudaIpcMemLazyEnablePeerAccess);
    if (e != cudaSuccess) {
        *ptr = nullptr;
        cudaGetLastError();
        return cuda_fail("peer_open: cudaIpcOpenMemHandle", e);
    }
    g_error.clear();
    return MAKO_OK;
}

int mako_peer_close(mako_attn_ctx* ctx, void* ptr)
{
    if (!ctx)
        return fail(MAKO_EINVAL, "peer_close: null context");
    if (!ptr)
        return MAKO_OK;
    DeviceGuard dg(ctx->device);
    cudaError_t e = cudaIpcCloseMemHandle(ptr);
    return e == cudaSuccess ? (g_error.clear(), MAKO_OK) : cuda_fail("peer_close", e);
}

int mako_group_create(mako_attn_ctx* ctx, uint32_t rank, uint32_t n_ranks, uint32_t max_rows, mako_attn_group** out,
                      mako_ipc_handle* handle)
{
    if (!ctx || !out || !handle)
        return fail(MAKO_EINVAL, "group_create: null argument");
    *out = nullptr;
    if (n_ranks == 0 || n_ranks > MAKO_MAX_RANKS || rank >= n_ranks)
        return fail(MAKO_EINVAL, "group_create: rank %u of %u (at most %d ranks)", rank, n_ranks, MAKO_MAX_RANKS);
    if (max_rows == 0 || max_rows > (1u << 20))
        return fail(MAKO_EINVAL, "group_create: max_rows %u (1 .. 2^20)", max_rows);
    auto* g = new (std::nothrow) mako_attn_group;
    if (!g)
        return fail(MAKO_ENOMEM, "group");
    g->ctx = ctx;
    g->rank = rank;
    g->n_ranks = n_ranks;
    g->rows_cap = max_rows;
    const size_t bytes = mako::xchg_bytes(max_rows);
    if (int rc = mako_peer_alloc(ctx, bytes, &g->area, handle)) {
        delete g;
        return rc;
    }
    {
        DeviceGuard dg(ctx->device);
        cudaError_t e = cudaMemset(g->area, 0, bytes);
        if (e == cudaSuccess)
            e = cudaDeviceSynchronize();  // zeroed before any peer can map and signal into it
        if (e != cudaSuccess) {
            cudaFree(g->area);
            delete g;
            return cuda_fail("group_create: clear", e);
        }
    }
    g->peer[rank] = g->area;
    *out = g;
    g_error.clear();
    return MAKO_OK;
}

int mako_group_connect(mako_attn_group* g, const mako_ipc_handle* handles)
{
    if (!g || !handles)
        return fail(MAKO_EINVAL, "group_connect: null argument");
    if (g->connected)
        return fail(MAKO_EINVAL, "group_connect: already connected");
    for (uint32_t r = 0; r < g->n_ranks; ++r) {
        if (r == g->rank)
            continue;
        if (int rc = mako_peer_open(g->ctx, &handles[r], &g->peer[r])) {
            for (uint32_t s = 0; s < r; ++s)
                if (s != g->rank && g->peer[s]) {
                    mako_peer_close(g->ctx, g->peer[s]);
                    g->peer[s] = nullptr;
                }
            return rc;
        }
    }
    g->connected = true;
    g->mapped = true;
    g_error.clear();
    return MAKO_OK;
}

int mako_group_connect_ptrs(mako_attn_group* g, void* const* areas)
{
    if (!g || !areas)
        return fail(MAKO_EINVAL, "group_connect_ptrs: null argument");
    if (g->connected)
        return fail(MAKO_EINVAL, "group_connect_ptrs: already connected");
    for (uint32_t r = 0; r < g->n_ranks; ++r)
        if (r != g->rank && (!areas[r] || !aligned16(areas[r])))
            return fail(MAKO_EINVAL, "group_connect_ptrs: area of rank %u null or unaligned", r);
    for (uint32_t r = 0; r < g->n_ranks; ++r)
        if (r != g->rank)
            g->peer[r] = areas[r];
    g->connected = true;
    g_error.clear();
    return MAKO_OK;
}

int mako_group_area(mako_attn_group* g, void** area, size_t* bytes)
{
    if (!g || !area || !bytes)
        return fail(MAKO_EINVAL, "group_area: null argument");
    *area = g->area;
    *bytes = mako::xchg_bytes(g->rows_cap);
    return MAKO_OK;
}

int mako_group_destroy(mako_attn_group* g)
{
    if (!g)
        return MAKO_OK;
    int rc = MAKO_OK;
    {
        DeviceGuard dg(g->ctx->device);
        cudaDeviceSynchronize();  // no kernel of ours still signals through the mappings
        for (uint32_t r = 0; r < g->n_ranks && g->mapped; ++r)
            if (r != g->rank && g->peer[r]) {
                cudaError_t e = cudaIpcCloseMemHandle(g->peer[r]);
                if (e != cudaSuccess && rc == MAKO_OK)
                    rc = cuda_fail("group_destroy: close", e);
            }
        if (g->area) {
            cudaError_t e = cudaFree(g->area);
            if (e != cudaSuccess && rc == MAKO_OK)
                rc = cuda_fail("group_destroy: free", e);
        }
    }
    delete g;
    return rc;
}

int mako_attention_gather(mako_attn_group* g, void* stream, int dtype, const void* q, const void* k, const void* v,
                          float* const* o_ranks, uint32_t n_q, uint32_t q_pad, uint32_t n_k, uint32_t k_pad,
                          uint32_t heads, uint32_t kv_heads, uint32_t head0, uint32_t q_pos0, uint32_t block,
                          uint32_t width)
{
    if (int rc = check_group(g, dtype))
        return rc;
    mako_attn_ctx* ctx = g->ctx;
    if (ctx->cc_major != 10)
        return fail(MAKO_ENOTSUP, "attention_gather: the tcgen05 kernel needs sm_100 (sm_%d)", ctx->cc_major * 10);
    if (ctx->out16)
        return fail(MAKO_ENOTSUP, "attention_gather: o is fp32 in the sharded forms (MAKO_OPT_OUTPUT_16BIT is set)");
    if (width % 4)
        return fail(MAKO_EINVAL, "attention_gather: o row width %u (a multiple of 4)", width);
    if (!heads || !kv_heads || heads % kv_heads)
        return fail(MAKO_EINVAL, "attention_gather: %u heads over %u kv heads", heads, kv_heads);
    if (q_pad % 64 || q_pad < n_q || k_pad < n_k)
        return fail(MAKO_EINVAL, "attention_gather: q_pad %u (a multiple of 64, at least n_q %u), k_pad %u (at least "
                                 "n_k %u)", q_pad, n_q, k_pad, n_k);
    if (uint64_t(head0 + heads) * 128 > width)
        return fail(MAKO_EINVAL, "attention_gather: heads [%u, %u) of 128 beyond o rows of %u floats", head0,
                    head0 + heads, width);
    if (!q || !k || !v || !o_ranks || !aligned16(q) || !aligned16(k) || !aligned16(v))
        return fail(MAKO_EINVAL, "attention_gather: null or unaligned tensor (16-byte alignment)");
    for (uint32_t r = 0; r < g->n_ranks; ++r)
        if (!o_ranks[r] || !aligned16(o_ranks[r]))
            return fail(MAKO_EINVAL, "attention_gather: o of rank %u null or unaligned", r);
    DeviceGuard dg(ctx->device);
    if (dg.err != cudaSuccess)
        return cuda_fail("set device", dg.err);
    auto st = static_cast<cudaStream_t>(stream);
    mako::AttnParams p{};
    p.num_sms = ctx->persistent_ctas();
    p.q = q;
    p.k = k;
    p.v = v;
    p.o = o_ranks[g->rank];
    p.n_q = n_q;
    p.q_pad = q_pad;
    p.n_k = n_k;
    p.k_pad = k_pad;
    p.heads = heads;
    p.kv_heads = kv_heads;
    p.q_pos0 = q_pos0;
    p.block = block;
    p.width = width;
    p.scale = 1.0f / sqrtf(128.0f);
    p.n_od = g->n_ranks;
    p.head0 = head0;
    for (uint32_t r = 0; r < g->n_ranks; ++r)  // own copy first: the local store is the cheap one
        p.od[r] = o_ranks[(g->rank + r) % g->n_ranks];
    void *v16 = nullptr, *vmax = nullptr, *vinv = nullptr;
    if (dtype == MAKO_BF16) {
        if (int rc = scratch(ctx, "v16", size_t(kv_heads) * k_pad * 128 * 2, &v16))
            return rc;
        if (int rc = scratch(ctx, "vmax", size_t(kv_heads) * 4, &vmax))
            return rc;
        if (int rc = scratch(ctx, "vinv", size_t(kv_heads) * 4, &vinv))
            return rc;
        cudaError_t e = mako::launch_v_to_f16(v, v16, static_cast<uint32_t*>(vmax), static_cast<float*>(vinv),
                                              128, kv_heads, k_pad, n_k, nullptr, ctx->num_sms, st);
        if (e != cudaSuccess)
            return cuda_fail("attention_gather (V to fp16)", e);
        ctx->launches += 2;
    }
    const mako::XchgParams x = xchg_params(g);
    cudaError_t e = mako::launch_group_barrier(x, 0, st);
    if (e != cudaSuccess)
        return cuda_fail("attention_gather (enter barrier)", e);
    if (n_q) {
        KernelTimer t(ctx, st);
        e = mako::launch_attn_tc(p, dtype, 128, v16, static_cast<const float*>(vinv), ctx->err, st);
        t.stop();
        if (e != cudaSuccess)
            return cuda_fail("attention_gather (tcgen05)", e);
    }
    ctx->launches += n_q ? 3 : 2;
    return launched("attention_gather (done barrier)", mako::launch_group_barrier(x, 1, st));
}

int mako_attention_decode_kv_sharded(mako_attn_group* g, void* stream, int dtype, const void* q, const void* k,
                                     const void* v, float* o, uint32_t batch, const int32_t* kv_len,
                                     uint32_t max_kv_len, uint32_t heads, uint32_t kv_heads, uint32_t dim,
                                     uint32_t k_stride)
{
    if (int rc = check_group(g, dtype))
        return rc;
    mako_attn_ctx* ctx = g->ctx;
    if (ctx->out16)
        return fail(MAKO_ENOTSUP, "decode_kv_sharded: o is fp32 in the sharded forms (MAKO_OPT_OUTPUT_16BIT is set)");
    if (dim != 64 && dim != 128 && dim != 256)
        return fail(MAKO_EINVAL, "decode_kv_sharded: heads of %u", dim);
    if (!heads || !kv_heads || heads % kv_heads)
        return fail(MAKO_EINVAL, "decode_kv_sharded: %u heads over %u kv heads", heads, kv_heads);
    if (max_kv_len > k_stride)
        return fail(MAKO_EINVAL, "decode_kv_sharded: max_kv_len %u beyond the cache's %u rows", max_kv_len, k_stride);
    if (uint64_t(batch) * heads > g->rows_cap)
        return fail(MAKO_EINVAL, "decode_kv_sharded: %u sequences x %u heads beyond the group's %u rows", batch, heads,
                    g->rows_cap);
    if (!q || !k || !v || !o || !kv_len || !aligned16(q) || !aligned16(k) || !aligned16(v) || !aligned16(o))
        return fail(MAKO_EINVAL, "decode_kv_sharded: null or unaligned tensor (16-byte alignment)");
    if (batch == 0)
        return MAKO_OK;
    DeviceGuard dg(ctx->device);
    if (dg.err != cudaSuccess)
        return cuda_fail("set device", dg.err);
    mako::DecodeParams p{};
    p.q = q;
    p.k = k;
    p.v = v;
    p.o = o;
    p.kv_len = kv_len;
    p.len = max_kv_len;
    p.q_bstride = uint64_t(heads) * dim;
    p.q_hstride = dim;
    p.k_hstride = uint64_t(k_stride) * dim;
    p.k_bstride = uint64_t(kv_heads) * p.k_hstride;
    p.o_bstride = uint64_t(heads) * dim;
    p.batch = batch;
    p.heads = heads;
    p.kv_heads = kv_heads;
    p.scale = 1.0f / sqrtf(float(dim));
    p.keep_partials = 1;
    mako::decode_plan(max_kv_len, batch, kv_heads, heads, ctx->num_sms, ctx->decode_chunk, &p.chunk, &p.n_splits);
    void *op, *mlp;
    if (int rc = scratch(ctx, "dec_o", size_t(batch) * heads * p.n_splits * dim * 4, &op))
        return rc;
    if (int rc = scratch(ctx, "dec_ml", size_t(batch) * heads * p.n_splits * 8, &mlp))
        return rc;
    p.o_part = static_cast<float*>(op);
    p.ml_part = static_cast<float2*>(mlp);
    auto st = static_cast<cudaStream_t>(stream);
    KernelTimer t(ctx, st);
    cudaError_t e = mako::launch_decode_split(p, dtype, int(dim), st);
    t.stop();
    if (e != cudaSuccess)
        return cuda_fail("decode_kv_sharded (splits)", e);
    ctx->launches += 2;
    return launched("decode_kv_sharded (exchange)", mako::launch_decode_xchg(p, xchg_params(g), int(dim), st));
}

} // extern "C"
