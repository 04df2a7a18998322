// Split-KV decode: one query row per (sequence, head) attending keys [0, len) of its sequence's cache.  The reference
// has no decode kernel (a decode token there is attention() with n_q = 1, q_pos0 = len - 1, causal:
// src/models/runtime.cpp:262-273, src/kernels/ops.metal:242-270); this is the same maths laid out for an HBM-bound
// read of the whole cache.
//
// Kernel 1 (decode_split_kernel): one CTA per (split of `chunk` keys, kv head, sequence) serves the q heads of that
// kv head's GQA group (up to 16 a CTA) from one read of K and V.  64-key tiles of K and V stream through a 3-stage
// cp.async ring of 128-bit loads into XOR-swizzled shared memory; each of the 4 warps takes 16 keys of a tile on
// mma.sync (the group's q rows padded to 16), keeps its own running softmax and accumulator, and the warps merge at
// the end into one partial (o unnormalised, max, sum) per (sequence, head, split); a sequence with one split writes
// o directly.
// Kernel 2 (decode_combine_kernel): the log-sum-exp merge of a row's splits into o, launched as a programmatic
// dependent of kernel 1 so that its launch overlaps kernel 1's last wave.
#include "common.cuh"
#include "kernels.h"
#include "mako_attn.h"

#include <mutex>
#include <type_traits>

namespace mako {
namespace {

constexpr int DBN = 64, DNT = 128, DST = 3, QR = 16;
constexpr uint64_t kMaxSplits = 1024;

// Keys of sequence b: its kv_len entry (<= 0: none) capped at max_kv_len, so that a length beyond the split plan's
// reach is cut at max_kv_len and every kernel of a call agrees on the same split count; without kv_len, p.len.
__device__ __forceinline__ uint32_t seq_keys(const DecodeParams& p, uint32_t b)
{
    if (!p.kv_len)
        return p.len;
    const int32_t l = p.kv_len[b];
    return l > 0 ? min(uint32_t(l), p.len) : 0u;
}

template <int D, typename T>
__global__ void __launch_bounds__(DNT, 2) decode_split_kernel(const DecodeParams p)
{
    constexpr int ROWB = D * 2, CH = D / 8, KS = D / 16, TILE = DBN * ROWB;
    constexpr bool SPLIT = !std::is_same<T, __half>::value;
    extern __shared__ __align__(128) uint8_t smem[];
    const uint32_t sQ = smem_u32(smem), sK = sQ + QR * ROWB, sV = sK + DST * TILE;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, g = lane >> 2, tq = lane & 3, mi = lane >> 3;
    const uint32_t group = p.heads / p.kv_heads, rb = (group + QR - 1) / QR;
    const uint32_t b = blockIdx.z, kvh = blockIdx.y / rb, rblk = blockIdx.y % rb, split = blockIdx.x;
    asm volatile("griddepcontrol.launch_dependents;\n" ::: "memory");  // the combine may be scheduled now
    const uint32_t L = seq_keys(p, b);
    const uint32_t start = split * p.chunk;
    const uint32_t h0 = kvh * group + rblk * QR, nrows = min(uint32_t(QR), group - rblk * QR);
    if (start >= L) {
        if (L == 0 && split == 0 && !p.keep_partials)  // no key: the rows are 0
            for (uint32_t i = tid; i < nrows * D; i += DNT)
                out_store1(p.o, uint64_t(b) * p.o_bstride + uint64_t(h0 + i / D) * D + i % D, 0.0f, p.o_type);
        return;
    }
    const uint32_t end = min(L, start + p.chunk);
    const T* qg = static_cast<const T*>(p.q) + uint64_t(b) * p.q_bstride;
    const T* kg = static_cast<const T*>(p.k) + uint64_t(b) * p.k_bstride + uint64_t(kvh) * p.k_hstride;
    const T* vg = static_cast<const T*>(p.v) + uint64_t(b) * p.k_bstride + uint64_t(kvh) * p.k_hstride;

    for (int i = tid; i < QR * CH; i += DNT) {
        const uint32_t r = i / CH, c = i % CH;
        const bool ok = r < nrows;
        cp_async16(sQ + swz(r, c, ROWB), qg + (ok ? uint64_t(h0 + r) * p.q_hstride + c * 8 : 0), ok);
    }
    cp_async_commit();
    const uint32_t nt = (end - start + DBN - 1) / DBN;
    auto load = [&](uint32_t t) {
        const uint32_t st = t % DST, j0 = start + t * DBN;
        for (int i = tid; i < DBN * CH; i += DNT) {
            const uint32_t r = i / CH, c = i % CH, j = j0 + r;
            const bool ok = j < end;
            const uint64_t off = ok ? uint64_t(j) * D + c * 8 : 0;
            cp_async16(sK + st * TILE + swz(r, c, ROWB), kg + off, ok);
            cp_async16(sV + st * TILE + swz(r, c, ROWB), vg + off, ok);
        }
    };
#pragma unroll
    for (int t = 0; t < DST - 1; ++t) {
        if (uint32_t(t) < nt)
            load(t);
        cp_async_commit();
    }

    uint32_t qa[KS][4];
    float acc[D / 8][4];
#pragma unroll
    for (int i = 0; i < D / 8; ++i)
        acc[i][0] = acc[i][1] = acc[i][2] = acc[i][3] = 0.0f;
    float m[2] = {-INFINITY, -INFINITY}, l[2] = {0.0f, 0.0f};
    const float scale = p.scale * kLog2e;

    for (uint32_t t = 0; t < nt; ++t) {
        cp_async_wait<DST - 2>();
        __syncthreads();
        if (t == 0) {
#pragma unroll
            for (int ks = 0; ks < KS; ++ks)
                ldsm_x4(qa[ks], sQ + swz((mi & 1) * 8 + (lane & 7), ks * 2 + (mi >> 1), ROWB));
        }
        if (t + DST - 1 < nt)
            load(t + DST - 1);
        cp_async_commit();
        const uint32_t kst = sK + (t % DST) * TILE, vst = sV + (t % DST) * TILE;
        const uint32_t kr = warp * 16;  // this warp's 16 keys of the tile

        float s[2][4] = {{0.0f, 0.0f, 0.0f, 0.0f}, {0.0f, 0.0f, 0.0f, 0.0f}};
#pragma unroll
        for (int ks = 0; ks < KS; ++ks) {
            uint32_t kb[4];
            ldsm_x4(kb, kst + swz(kr + (mi >> 1) * 8 + (lane & 7), ks * 2 + (mi & 1), ROWB));
            mma16816(s[0], qa[ks], kb[0], kb[1], T());
            mma16816(s[1], qa[ks], kb[2], kb[3], T());
        }
        const uint32_t jb = start + t * DBN + kr;
        float mx[2] = {-INFINITY, -INFINITY};
#pragma unroll
        for (int n = 0; n < 2; ++n)
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                const uint32_t j = jb + n * 8 + 2 * tq + (e & 1);
                const float x = j < end ? s[n][e] * scale : -INFINITY;
                s[n][e] = x;
                mx[e >> 1] = fmaxf(mx[e >> 1], x);
            }
        float f[2];
#pragma unroll
        for (int r = 0; r < 2; ++r) {
            mx[r] = fmaxf(mx[r], __shfl_xor_sync(0xffffffffu, mx[r], 1));
            mx[r] = fmaxf(mx[r], __shfl_xor_sync(0xffffffffu, mx[r], 2));
            const float mn = fmaxf(m[r], mx[r]);
            f[r] = mn == -INFINITY ? 1.0f : ex2(m[r] - mn);
            m[r] = mn;
            l[r] *= f[r];
        }
#pragma unroll
        for (int i = 0; i < D / 8; ++i) {
            acc[i][0] *= f[0];
            acc[i][1] *= f[0];
            acc[i][2] *= f[1];
            acc[i][3] *= f[1];
        }
#pragma unroll
        for (int n = 0; n < 2; ++n)
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                const float mm = m[e >> 1];
                const float pe = mm == -INFINITY ? 0.0f : ex2(s[n][e] - mm);
                s[n][e] = pe;
                l[e >> 1] += pe;
            }
        uint32_t pa[4], pl[4];
        if (!SPLIT) {
            pa[0] = Elem<__half>::pack(s[0][0], s[0][1]);
            pa[1] = Elem<__half>::pack(s[0][2], s[0][3]);
            pa[2] = Elem<__half>::pack(s[1][0], s[1][1]);
            pa[3] = Elem<__half>::pack(s[1][2], s[1][3]);
        } else {
            const float* src[4] = {&s[0][0], &s[0][2], &s[1][0], &s[1][2]};
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                const __nv_bfloat16 h0 = __float2bfloat16_rn(src[i][0]), h1 = __float2bfloat16_rn(src[i][1]);
                pa[i] = Elem<__nv_bfloat16>::pack(__bfloat162float(h0), __bfloat162float(h1));
                pl[i] = Elem<__nv_bfloat16>::pack(src[i][0] - __bfloat162float(h0), src[i][1] - __bfloat162float(h1));
            }
        }
#pragma unroll
        for (int dp = 0; dp < D / 16; ++dp) {
            uint32_t vb[4];
            ldsm_x4_t(vb, vst + swz(kr + (mi & 1) * 8 + (lane & 7), dp * 2 + (mi >> 1), ROWB));
            mma16816(acc[2 * dp], pa, vb[0], vb[1], T());
            mma16816(acc[2 * dp + 1], pa, vb[2], vb[3], T());
            if (SPLIT) {
                mma16816(acc[2 * dp], pl, vb[0], vb[1], T());
                mma16816(acc[2 * dp + 1], pl, vb[2], vb[3], T());
            }
        }
    }
    cp_async_wait<0>();
    __syncthreads();  // the stage ring is reused below for the warps' merge

    // Merge the four warps: rows g and g + 8 of each warp's state into shared memory, then per row.
    float* sm = reinterpret_cast<float*>(smem + QR * ROWB);  // [4][2][QR] (m, l) then [4][QR][D] o
    float* so = sm + 4 * 2 * QR;
#pragma unroll
    for (int r = 0; r < 2; ++r) {
        l[r] += __shfl_xor_sync(0xffffffffu, l[r], 1);
        l[r] += __shfl_xor_sync(0xffffffffu, l[r], 2);
        if (tq == 0) {
            sm[(warp * 2 + 0) * QR + g + 8 * r] = m[r];
            sm[(warp * 2 + 1) * QR + g + 8 * r] = l[r];
        }
#pragma unroll
        for (int i = 0; i < D / 8; ++i)
            *reinterpret_cast<float2*>(so + (warp * QR + g + 8 * r) * D + i * 8 + 2 * tq) =
                make_float2(acc[i][2 * r], acc[i][2 * r + 1]);
    }
    __syncthreads();
    const uint32_t ns = (L + p.chunk - 1) / p.chunk;  // this sequence's splits
    for (uint32_t i = tid; i < nrows * D; i += DNT) {
        const uint32_t r = i / D, d = i % D;
        float M = -INFINITY;
#pragma unroll
        for (int w = 0; w < 4; ++w)
            M = fmaxf(M, sm[(w * 2) * QR + r]);
        float Ls = 0.0f, O = 0.0f;
#pragma unroll
        for (int w = 0; w < 4; ++w) {
            const float mw = sm[(w * 2) * QR + r];
            const float fw = mw == -INFINITY ? 0.0f : ex2(mw - M);
            Ls += sm[(w * 2 + 1) * QR + r] * fw;
            O += so[(w * QR + r) * D + d] * fw;
        }
        if (ns == 1 && !p.keep_partials) {
            out_store1(p.o, uint64_t(b) * p.o_bstride + uint64_t(h0 + r) * D + d, Ls > 0.0f ? O / Ls : 0.0f, p.o_type);
        } else {
            const uint64_t row = (uint64_t(b) * p.heads + h0 + r) * p.n_splits + split;
            p.o_part[row * D + d] = O;
            if (d == 0)
                p.ml_part[row] = make_float2(M, Ls);
        }
    }
}

// One CTA per (head, sequence), one thread per output value; the splits' weights 2^(m_s - M) go through shared
// memory so each thread's loop is a stream of independent loads.
template <int D>
__global__ void __launch_bounds__(D) decode_combine_kernel(const DecodeParams p)
{
    asm volatile("griddepcontrol.wait;\n" ::: "memory");  // kernel 1's writes are visible from here on
    __shared__ float w[kMaxSplits];
    __shared__ float tot;
    const uint32_t h = blockIdx.x, b = blockIdx.y, d = threadIdx.x;
    const uint32_t L = seq_keys(p, b);
    const uint32_t ns = min((L + p.chunk - 1) / p.chunk, p.n_splits);
    if (ns <= 1)  // written by kernel 1 (one split, or no key)
        return;
    const uint64_t row0 = (uint64_t(b) * p.heads + h) * p.n_splits;
    float M = -INFINITY;
    for (uint32_t s = d; s < ns; s += D)
        M = fmaxf(M, p.ml_part[row0 + s].x);
    __shared__ float red[D / 32];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1)
        M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, o));
    if ((d & 31) == 0)
        red[d >> 5] = M;
    __syncthreads();
    M = red[0];
#pragma unroll
    for (int i = 1; i < D / 32; ++i)
        M = fmaxf(M, red[i]);
    float ls = 0.0f;
    for (uint32_t s = d; s < ns; s += D) {
        const float2 ml = p.ml_part[row0 + s];
        const float f = ml.x == -INFINITY ? 0.0f : ex2(ml.x - M);
        w[s] = f;
        ls += ml.y * f;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1)
        ls += __shfl_xor_sync(0xffffffffu, ls, o);
    __syncthreads();
    if ((d & 31) == 0)
        red[d >> 5] = ls;
    __syncthreads();
    if (d == 0) {
        float t = 0.0f;
#pragma unroll
        for (int i = 0; i < D / 32; ++i)
            t += red[i];
        tot = t;
    }
    __syncthreads();
    const float* src = p.o_part + row0 * D + d;
    float acc[8] = {0.0f, 0.0f, 0.0f, 0.0f, 0.0f, 0.0f, 0.0f, 0.0f};
    uint32_t s = 0;
    for (; s + 8 <= ns; s += 8) {
#pragma unroll
        for (int u = 0; u < 8; ++u)
            acc[u] += src[uint64_t(s + u) * D] * w[s + u];
    }
    for (; s < ns; ++s)
        acc[0] += src[uint64_t(s) * D] * w[s];
    const float O = ((acc[0] + acc[1]) + (acc[2] + acc[3])) + ((acc[4] + acc[5]) + (acc[6] + acc[7]));
    out_store1(p.o, uint64_t(b) * p.o_bstride + uint64_t(h) * D + d, tot > 0.0f ? O / tot : 0.0f, p.o_type);
}

template <int D, typename T>
cudaError_t launch_dec(const DecodeParams& p, cudaStream_t st)
{
    constexpr int smem = (QR + 2 * DST * DBN) * D * 2;
    static_assert((4 * 2 * QR + 4 * QR * D) * 4 <= 2 * DST * DBN * D * 2, "merge buffer fits the stage ring");
    auto kern = decode_split_kernel<D, T>;
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e != cudaSuccess)
        return e;
    const uint32_t group = p.heads / p.kv_heads, rb = (group + QR - 1) / QR;
    kern<<<dim3(p.n_splits, p.kv_heads * rb, p.batch), DNT, smem, st>>>(p);
    if ((e = cudaGetLastError()) != cudaSuccess)
        return e;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(p.heads, p.batch);
    cfg.blockDim = dim3(D);
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, decode_combine_kernel<D>, p);
}

template <int D, typename T>
cudaError_t launch_split_only(const DecodeParams& p, cudaStream_t st)
{
    constexpr int smem = (QR + 2 * DST * DBN) * D * 2;
    auto kern = decode_split_kernel<D, T>;
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e != cudaSuccess)
        return e;
    const uint32_t group = p.heads / p.kv_heads, rb = (group + QR - 1) / QR;
    kern<<<dim3(p.n_splits, p.kv_heads * rb, p.batch), DNT, smem, st>>>(p);
    return cudaGetLastError();
}

__device__ __forceinline__ void st_release_sys(uint32_t* ptr, uint32_t v)
{
    asm volatile("st.release.sys.global.u32 [%0], %1;\n" ::"l"(ptr), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* ptr)
{
    uint32_t v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];\n" : "=r"(v) : "l"(ptr) : "memory");
    return v;
}
constexpr long long kXchgWaitLimit = 1ll << 31;  // clock cycles (~1 s) before a wait on a peer gives up

// One CTA per (head, sequence), one thread per output value.  Phase 1 merges this rank's splits (as
// decode_combine_kernel, but keeping the unnormalised sum and its maximum); phase 2 stores that row into slot `rank`
// of every rank's area and releases the row's flag there; phase 3 waits until every rank's row has arrived in this
// rank's area (bounded) and merges them by log-sum-exp into o.  The area is double-buffered by epoch parity: a rank
// one call ahead writes the other half, and it cannot get two calls ahead because its own phase 3 waits for ours.
template <int D>
__global__ void __launch_bounds__(D) decode_xchg_kernel(const DecodeParams p, const XchgParams x)
{
    asm volatile("griddepcontrol.wait;\n" ::: "memory");
    __shared__ float w[kMaxSplits];
    __shared__ float red[D / 32];
    __shared__ float tot;
    __shared__ int timed_out;
    const uint32_t h = blockIdx.x, b = blockIdx.y, d = threadIdx.x;
    const uint32_t row = b * p.heads + h, par = x.epoch & 1u;
    const uint32_t L = seq_keys(p, b);
    const uint32_t ns = min((L + p.chunk - 1) / p.chunk, p.n_splits);
    const uint64_t row0 = (uint64_t(b) * p.heads + h) * p.n_splits;
    if (d == 0)
        timed_out = 0;

    // ---- phase 1: this rank's splits
    float M = -INFINITY;
    for (uint32_t s = d; s < ns; s += D)
        M = fmaxf(M, p.ml_part[row0 + s].x);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1)
        M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, o));
    if ((d & 31) == 0)
        red[d >> 5] = M;
    __syncthreads();
    M = red[0];
#pragma unroll
    for (int i = 1; i < D / 32; ++i)
        M = fmaxf(M, red[i]);
    float ls = 0.0f;
    for (uint32_t s = d; s < ns; s += D) {
        const float2 ml = p.ml_part[row0 + s];
        const float f = ml.x == -INFINITY ? 0.0f : ex2(ml.x - M);
        w[s] = f;
        ls += ml.y * f;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1)
        ls += __shfl_xor_sync(0xffffffffu, ls, o);
    __syncthreads();
    if ((d & 31) == 0)
        red[d >> 5] = ls;
    __syncthreads();
    if (d == 0) {
        float t = 0.0f;
#pragma unroll
        for (int i = 0; i < D / 32; ++i)
            t += red[i];
        tot = t;
    }
    __syncthreads();
    float O = 0.0f;
    for (uint32_t s = 0; s < ns; ++s)
        O += p.o_part[(row0 + s) * D + d] * w[s];
    const float Ls = tot;

    // ---- phase 2: push (O, M, Ls) into slot `rank` of every rank's area, then release the row's flags
    const uint64_t xoff = xchg_rows_offset(x.rows_cap);
    const uint64_t slot = ((uint64_t(par) * kMaxRanks + x.rank) * x.rows_cap + row) * kXchgStride;
    for (uint32_t g = 0; g < x.n_ranks; ++g) {
        float* dst = reinterpret_cast<float*>(x.area[g] + xoff) + slot;
        dst[d] = O;
        if (d == 0)
            *reinterpret_cast<float2*>(dst + D) = make_float2(M, Ls);
    }
    __syncthreads();
    const uint64_t fslot = (uint64_t(par) * kMaxRanks + x.rank) * x.rows_cap + row;
    if (d < x.n_ranks) {
        asm volatile("fence.acq_rel.sys;\n" ::: "memory");
        st_release_sys(reinterpret_cast<uint32_t*>(x.area[d] + 256) + fslot, x.epoch);
    }

    // ---- phase 3: every rank's row in this rank's area, merged
    if (d < x.n_ranks) {
        const uint32_t* f = reinterpret_cast<const uint32_t*>(x.area[x.rank] + 256) +
                            (uint64_t(par) * kMaxRanks + d) * x.rows_cap + row;
        if (ld_acquire_sys(f) != x.epoch) {
            const long long t0 = clock64();
            while (ld_acquire_sys(f) != x.epoch)
                if (clock64() - t0 > kXchgWaitLimit) {
                    timed_out = 1;
                    atomicExch(x.err, 31);
                    break;
                }
        }
    }
    __syncthreads();
    const float* mine = reinterpret_cast<const float*>(x.area[x.rank] + xoff);
    float Mg = -INFINITY;
    for (uint32_t g = 0; g < x.n_ranks; ++g)
        Mg = fmaxf(Mg, __ldcg(mine + ((uint64_t(par) * kMaxRanks + g) * x.rows_cap + row) * kXchgStride + D));
    float T = 0.0f, Og = 0.0f;
    for (uint32_t g = 0; g < x.n_ranks; ++g) {
        const float* src = mine + ((uint64_t(par) * kMaxRanks + g) * x.rows_cap + row) * kXchgStride;
        const float mg = __ldcg(src + D);
        const float f = mg == -INFINITY ? 0.0f : ex2(mg - Mg);
        T += __ldcg(src + D + 1) * f;
        Og += __ldcg(src + d) * f;
    }
    p.o[uint64_t(b) * p.o_bstride + uint64_t(h) * D + d] = (T > 0.0f && !timed_out) ? Og / T : 0.0f;
}

// Barrier over the group: thread g releases this rank's flag in rank g's area, then waits for rank g's flag in ours.
__global__ void group_barrier_kernel(const XchgParams x, uint32_t kind)
{
    const uint32_t g = threadIdx.x, par = x.epoch & 1u;
    if (g >= x.n_ranks)
        return;
    asm volatile("fence.acq_rel.sys;\n" ::: "memory");
    st_release_sys(reinterpret_cast<uint32_t*>(x.area[g]) + (par * 2 + kind) * kMaxRanks + x.rank, x.epoch);
    const uint32_t* f = reinterpret_cast<const uint32_t*>(x.area[x.rank]) + (par * 2 + kind) * kMaxRanks + g;
    if (ld_acquire_sys(f) != x.epoch) {
        const long long t0 = clock64();
        while (ld_acquire_sys(f) != x.epoch)
            if (clock64() - t0 > kXchgWaitLimit) {
                atomicExch(x.err, 30);
                break;
            }
    }
}

} // namespace

cudaError_t launch_decode_split(const DecodeParams& p, int dtype, int dim, cudaStream_t st)
{
    if (p.batch == 0 || p.heads == 0)
        return cudaSuccess;
    const bool bf = dtype == kBF16;
    switch (dim) {
    case 64:
        return bf ? launch_split_only<64, __nv_bfloat16>(p, st) : launch_split_only<64, __half>(p, st);
    case 128:
        return bf ? launch_split_only<128, __nv_bfloat16>(p, st) : launch_split_only<128, __half>(p, st);
    case 256:
        return bf ? launch_split_only<256, __nv_bfloat16>(p, st) : launch_split_only<256, __half>(p, st);
    default:
        return cudaErrorInvalidValue;
    }
}

cudaError_t launch_decode_combine(const DecodeParams& p, int dim, cudaStream_t st)
{
    if (p.batch == 0 || p.heads == 0)
        return cudaSuccess;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(p.heads, p.batch);
    cfg.blockDim = dim3(dim);
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    switch (dim) {
    case 64:
        return cudaLaunchKernelEx(&cfg, decode_combine_kernel<64>, p);
    case 128:
        return cudaLaunchKernelEx(&cfg, decode_combine_kernel<128>, p);
    case 256:
        return cudaLaunchKernelEx(&cfg, decode_combine_kernel<256>, p);
    default:
        return cudaErrorInvalidValue;
    }
}

cudaError_t launch_decode_xchg(const DecodeParams& p, const XchgParams& x, int dim, cudaStream_t st)
{
    if (p.batch == 0 || p.heads == 0)
        return cudaSuccess;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(p.heads, p.batch);
    cfg.blockDim = dim3(dim);
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    switch (dim) {
    case 64:
        return cudaLaunchKernelEx(&cfg, decode_xchg_kernel<64>, p, x);
    case 128:
        return cudaLaunchKernelEx(&cfg, decode_xchg_kernel<128>, p, x);
    case 256:
        return cudaLaunchKernelEx(&cfg, decode_xchg_kernel<256>, p, x);
    default:
        return cudaErrorInvalidValue;
    }
}

cudaError_t launch_group_barrier(const XchgParams& x, uint32_t kind, cudaStream_t st)
{
    group_barrier_kernel<<<1, 32, 0, st>>>(x, kind);
    return cudaGetLastError();
}

void decode_plan(uint32_t max_len, uint32_t batch, uint32_t kv_heads, uint32_t heads, int num_sms, uint32_t chunk_opt,
                 uint32_t* chunk, uint32_t* n_splits)
{
    // About 8 splits of the longest sequence's length an SM (the hardware scheduler back-fills freed SMs), each of
    // 256 to 2048 keys: fewer, longer splits cost fewer CTA starts and partial rows.  Measured on config 2 (batch 8,
    // 16-30K keys) and its 262144-key single sequence: 1664 and 1792 keys a split ran the split kernel 2.7% and 1.4%
    // faster than 1024; 512 or fewer keys were slower.
    const uint32_t group = heads / kv_heads, rb = (group + QR - 1) / QR;
    const uint64_t rows = uint64_t(max_len) * batch * kv_heads * rb;
    const uint64_t target = uint64_t(num_sms > 0 ? num_sms : 148) * 8;
    uint64_t c = (rows + target - 1) / target;
    c = (c + DBN - 1) / DBN * DBN;
    c = c < 256 ? 256 : (c > 2048 ? 2048 : c);
    if (chunk_opt)
        c = chunk_opt;
    if (uint64_t(max_len) > c * kMaxSplits)  // the combine's weight table holds kMaxSplits splits a row
        c = (uint64_t(max_len) + kMaxSplits - 1) / kMaxSplits;
    c = (c + DBN - 1) / DBN * DBN;
    *chunk = uint32_t(c);
    *n_splits = max_len ? uint32_t((max_len + c - 1) / c) : 1u;
}

cudaError_t launch_decode(const DecodeParams& p, int dtype, int dim, cudaStream_t st)
{
    if (p.batch == 0 || p.heads == 0)
        return cudaSuccess;
    const bool bf = dtype == kBF16;
    switch (dim) {
    case 64:
        return bf ? launch_dec<64, __nv_bfloat16>(p, st) : launch_dec<64, __half>(p, st);
    case 128:
        return bf ? launch_dec<128, __nv_bfloat16>(p, st) : launch_dec<128, __half>(p, st);
    case 256:
        return bf ? launch_dec<256, __nv_bfloat16>(p, st) : launch_dec<256, __half>(p, st);
    default:
        return cudaErrorInvalidValue;
    }
}

} // namespace mako

// ---- decode without device allocation ------------------------------------------------------------------------------
//
// Some callers cannot call cudaMalloc: a process whose device memory is entirely committed to another owner (a fixed
// pre-reserved pool, or memory borrowed under a lending protocol such as mako's lender / borrower, which must not
// grow outside its loan), or a latency-critical loop that cannot accept cudaMalloc / cudaFree synchronising the
// device.  mako_attention_decode_noalloc serves them: the split-KV partials live in the static device array below
// instead of context scratch, so a call allocates nothing and needs no context.

namespace {

// The partials of one call: o [batch][heads][n_splits][dim] fp32, then (max, sum) [batch][heads][n_splits].  Every
// GPU that loads this library holds this array until the process exits.
constexpr size_t kNoAllocScratchBytes = size_t(4) << 20;
static __device__ __align__(256) unsigned char g_decode_scratch[kNoAllocScratchBytes];

constexpr int kMaxDevices = 64;
std::mutex g_scratch_mutex;
void* g_scratch_addr[kMaxDevices] = {};

// The array's device address on `device` (current), looked up once per device.  In host code the array's name is
// only a host-side stand-in, never a usable device address.  The address belongs to the device's primary context:
// cudaDeviceReset destroys that context, so a process that resets a device must not call the entry point on that
// device again (the remembered address would be stale).
int scratch_address(int device, void** out)
{
    std::lock_guard<std::mutex> lock(g_scratch_mutex);
    if (!g_scratch_addr[device]) {
        void* p = nullptr;
        const cudaError_t e = cudaGetSymbolAddress(&p, g_decode_scratch);
        if (e != cudaSuccess || !p)
            return mako::set_error(MAKO_ECUDA, "decode_noalloc: address of the static scratch on device %d: %s", device,
                                   cudaGetErrorString(e));
        g_scratch_addr[device] = p;
    }
    *out = g_scratch_addr[device];
    return MAKO_OK;
}

} // namespace

extern "C" int mako_attention_decode_noalloc(void* stream, int dtype, const void* q, const void* k, const void* v,
                                             float* o, uint32_t batch, const int32_t* kv_len, uint32_t max_kv_len,
                                             uint32_t heads, uint32_t kv_heads, uint32_t dim, uint32_t k_stride)
{
    using mako::set_error;
    if (dtype != MAKO_F16 && dtype != MAKO_BF16)
        return set_error(MAKO_EINVAL, "decode_noalloc: element type %d", dtype);
    if (dim != 64 && dim != 128 && dim != 256)
        return set_error(MAKO_EINVAL, "decode_noalloc: heads of %u", dim);
    if (!heads || !kv_heads || heads % kv_heads)
        return set_error(MAKO_EINVAL, "decode_noalloc: %u heads over %u kv heads", heads, kv_heads);
    if (max_kv_len > k_stride)
        return set_error(MAKO_EINVAL, "decode_noalloc: max_kv_len %u beyond the cache's %u rows", max_kv_len, k_stride);
    auto aligned = [](const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; };
    if (!q || !k || !v || !o || !kv_len || !aligned(q) || !aligned(k) || !aligned(v) || !aligned(o))
        return set_error(MAKO_EINVAL, "decode_noalloc: null or unaligned tensor (16-byte alignment)");
    if (batch == 0)
        return MAKO_OK;
    int device = 0, sms = 148;
    cudaError_t e = cudaGetDevice(&device);
    if (e != cudaSuccess || device < 0 || device >= kMaxDevices)
        return set_error(MAKO_ECUDA, "decode_noalloc: current device: %s", cudaGetErrorString(e));
    if ((e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device)) != cudaSuccess)
        return set_error(MAKO_ECUDA, "decode_noalloc: SM count: %s", cudaGetErrorString(e));

    // The split plan of mako_attention_decode, with larger chunks when its partials would not fit the array.
    uint32_t chunk, n_splits;
    mako::decode_plan(max_kv_len, batch, kv_heads, heads, sms, 0, &chunk, &n_splits);
    // Layout in the array: o partials [batch][heads][n_splits][dim] fp32, then (max, sum) [batch][heads][n_splits].
    // With dim >= 64 the o block is a whole number of 256-byte lines, so the (max, sum) block needs no padding and a
    // split of every row costs exactly per_split bytes.
    const uint64_t per_split = uint64_t(batch) * heads * (uint64_t(dim) * 4 + 8);
    const uint64_t ns_max = kNoAllocScratchBytes / per_split;  // the most splits a row whose partials fit
    if (ns_max == 0)
        return set_error(MAKO_EINVAL,
                         "decode_noalloc: %u sequences x %u heads of %u need %llu bytes of partials, beyond the %zu-byte "
                         "static scratch (use mako_attention_decode)",
                         batch, heads, dim, (unsigned long long)per_split, kNoAllocScratchBytes);
    if (n_splits > ns_max) {  // the smallest multiple of 64 keys a split that needs no more than ns_max splits
        chunk = uint32_t(((uint64_t(max_kv_len) + ns_max - 1) / ns_max + 63) / 64 * 64);
        n_splits = (max_kv_len + chunk - 1) / chunk;
    }
    void* base = nullptr;
    if (int rc = scratch_address(device, &base))
        return rc;

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
    p.chunk = chunk;
    p.n_splits = n_splits;
    p.scale = 1.0f / sqrtf(float(dim));
    // Every partial the combine reads is written by the same call first, so nothing in the array needs clearing.
    const size_t o_bytes = size_t(batch) * heads * n_splits * dim * 4;
    p.o_part = static_cast<float*>(base);
    p.ml_part = reinterpret_cast<float2*>(static_cast<unsigned char*>(base) + o_bytes);
    if ((e = mako::launch_decode(p, dtype, int(dim), static_cast<cudaStream_t>(stream))) != cudaSuccess)
        return set_error(MAKO_ECUDA, "decode_noalloc: %s (%s)", cudaGetErrorString(e), cudaGetErrorName(e));
    mako::clear_error();
    return MAKO_OK;
}
