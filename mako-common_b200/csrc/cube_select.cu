// cube_select (TransformerRuntime::cube_select, src/models/runtime.cpp:286-303): for block-sparse attention over
// 64-row cubes, per head and query cube the `topk` key cubes whose mean-pooled k best matches the cube's mean-pooled q.
//
//   cube_pool   (ops.metal:927-939)  mean over a cube's 64 rows (all summed, invalid rows are zero) / cnt[c]
//   cube_scores (ops.metal:942-955)  sc[h][qc][kc] = qp . kp
//   cube_topk   (ops.metal:959-1027) the local cubes first, then the largest scores, ties to the smaller index
//               (here: a bitonic sort of packed (score, index) keys, one CTA per query cube and head)
//
// The fp32 arithmetic is pinned to one order so that the selection is reproducible bit for bit (the CPU oracle
// restates it): a sequential sum over the 64 rows then one IEEE division; per score s += ((q0 k0 + q1 k1) + q2 k2)
// + q3 k3 over d in fours.  __fmul_rn / __fadd_rn keep the compiler from fusing any of it into FMAs.
#include "common.cuh"
#include "kernels.h"

namespace mako {
namespace {

constexpr int CD = 128;  // head width of the sparse path (kHeadDim, src/models/runtime.hpp:34)

template <typename T>
__global__ void __launch_bounds__(CD) cube_pool_kernel(const CubeParams p)
{
    const uint32_t c = blockIdx.x, h = blockIdx.y, which = blockIdx.z, d = threadIdx.x;
    const T* x = static_cast<const T*>(which ? p.k : p.q);
    const uint32_t pad = which ? p.k_pad : p.q_pad;
    const T* src = x + (uint64_t(h) * pad + uint64_t(c) * 64) * CD + d;
    float s = 0.0f;
#pragma unroll 8
    for (int r = 0; r < 64; ++r)
        s = __fadd_rn(s, Elem<T>::to_f(src[uint64_t(r) * CD]));
    const uint32_t n = p.cnt[c];
    (which ? p.kp : p.qp)[(uint64_t(h) * p.n_cubes + c) * CD + d] = n ? __fdiv_rn(s, float(n)) : 0.0f;
}

// A 32 x 32 block of (query cube, key cube) scores: thread (ty, tx) scores query cubes 4 ty .. 4 ty + 3 against key
// cube tx.
__global__ void __launch_bounds__(256) cube_scores_kernel(const CubeParams p)
{
    __shared__ float sq[32][CD + 4], sk[32][CD + 4];
    const uint32_t h = blockIdx.z, qb = blockIdx.y * 32, kb = blockIdx.x * 32, tid = threadIdx.x;
    const uint32_t n = p.n_cubes;
    for (uint32_t i = tid; i < 32 * CD / 4; i += 256) {
        const uint32_t r = i / (CD / 4), c4 = i % (CD / 4);
        const float4 zero = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
        const float4 a = qb + r < n ? reinterpret_cast<const float4*>(p.qp + (uint64_t(h) * n + qb + r) * CD)[c4] : zero;
        const float4 b = kb + r < n ? reinterpret_cast<const float4*>(p.kp + (uint64_t(h) * n + kb + r) * CD)[c4] : zero;
        *reinterpret_cast<float4*>(&sq[r][c4 * 4]) = a;
        *reinterpret_cast<float4*>(&sk[r][c4 * 4]) = b;
    }
    __syncthreads();
    const uint32_t tx = tid & 31, ty = tid >> 5;
    float s[4] = {0.0f, 0.0f, 0.0f, 0.0f};
#pragma unroll 4
    for (int d = 0; d < CD; d += 4) {
        const float4 k4 = *reinterpret_cast<const float4*>(&sk[tx][d]);
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const float4 q4 = *reinterpret_cast<const float4*>(&sq[ty * 4 + i][d]);
            float t = __fmul_rn(q4.x, k4.x);
            t = __fadd_rn(t, __fmul_rn(q4.y, k4.y));
            t = __fadd_rn(t, __fmul_rn(q4.z, k4.z));
            t = __fadd_rn(t, __fmul_rn(q4.w, k4.w));
            s[i] = __fadd_rn(s[i], t);
        }
    }
    const uint32_t kc = kb + tx;
    if (kc >= n)
        return;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const uint32_t qc = qb + ty * 4 + i;
        if (qc < n)
            p.sc[(uint64_t(h) * n + qc) * n + kc] = s[i];
    }
}

// ---- top-k by sorting -------------------------------------------------------------------------------------------
//
// The selection rule (what the reference's cube_topk produces, ops.metal:959-1027, and what the oracle restates):
// the `local` cubes first; then, one pick at a time, the largest score not yet picked, ties to the smaller index;
// a score of -inf or NaN is never picked, and once nothing above -inf is left every further pick is cube 0.
// Equivalently: the candidates (scores above -inf, not a local pick) in descending (score, -index) order, then 0s.
// Here one CTA per (query cube, head) packs each candidate into a 64-bit key -- an order-preserving image of the
// score above the complemented index, so that the key order is exactly that order and all keys differ -- gives every
// other entry the key 0 (below any candidate), sorts the row's keys in shared memory with a bitonic network and
// reads the picks off the front.

constexpr uint32_t kTopkMaxCubes = 4096;  // the reference's bound (runtime.cpp:290)
constexpr uint32_t kTopkThreads = 256;

// Larger floats map to larger unsigned images; -0 maps as +0, since the selection's `>` treats them as equal.
__device__ __forceinline__ uint32_t order_image(float f)
{
    const uint32_t b = f == 0.0f ? 0u : __float_as_uint(f);
    return (b >> 31) ? ~b : (b | 0x80000000u);
}

__global__ void __launch_bounds__(kTopkThreads) cube_topk_kernel(const CubeParams p)
{
    __shared__ unsigned long long key[kTopkMaxCubes];
    const uint32_t qc = blockIdx.x, h = blockIdx.y, n = p.n_cubes, tid = threadIdx.x;
    const uint32_t k = min(p.topk, n);  // >= 1
    // The local option's forced entries, in this order: the query cube; with local 3 also the cube `stride` before
    // it and the cube `stride` after it, each when inside [0, n); no more than k in all (n: none).  Every thread
    // derives the same list.
    uint32_t nf = 0, f0 = n, f1 = n, f2 = n;
    if (p.local >= 1)
        f0 = qc, nf = 1;
    if (p.local == 3) {
        if (qc >= p.stride && nf < k)
            f1 = qc - p.stride, ++nf;
        if (qc + p.stride < n && nf < k)
            f2 = qc + p.stride, ++nf;
    }
    uint32_t width = 2;  // the sorted length: a power of two covering the row
    while (width < n)
        width <<= 1;
    const float* row = p.sc + (uint64_t(h) * n + qc) * n;
    for (uint32_t i = tid; i < width; i += kTopkThreads) {
        unsigned long long kv = 0ull;
        if (i < n) {
            const float s = row[i];
            const bool is_forced = i == f0 || i == f1 || i == f2;
            if (s > -INFINITY && !is_forced)  // false for NaN too
                kv = (static_cast<unsigned long long>(order_image(s)) << 32) | (0xFFFFFFFFu - i);
        }
        key[i] = kv;
    }
    __syncthreads();
    // Bitonic sort, descending: blocks of `size` alternate direction until the last merge.
    for (uint32_t size = 2; size <= width; size <<= 1)
        for (uint32_t half = size >> 1; half > 0; half >>= 1) {
            for (uint32_t t = tid; t < width / 2; t += kTopkThreads) {
                const uint32_t i = 2 * t - (t & (half - 1)), j = i + half;
                const unsigned long long a = key[i], b = key[j];
                if ((a < b) == ((i & size) == 0)) {
                    key[i] = b;
                    key[j] = a;
                }
            }
            __syncthreads();
        }
    uint16_t* out = p.sel + (uint64_t(h) * n + qc) * k;
    for (uint32_t i = tid; i < k; i += kTopkThreads) {
        uint32_t c;
        if (i < nf)
            c = i == 0 ? f0 : (i == 1 ? (f1 < n ? f1 : f2) : f2);
        else {
            const unsigned long long kv = key[i - nf];
            c = kv ? 0xFFFFFFFFu - uint32_t(kv) : 0u;
        }
        out[i] = uint16_t(c);
    }
    if (tid == 0)
        p.nsel[uint64_t(h) * n + qc] = uint16_t(k);
}

} // namespace

cudaError_t launch_cube_select(const CubeParams& p, int dtype, cudaStream_t st)
{
    if (p.heads == 0 || p.n_cubes == 0)
        return cudaSuccess;
    if (dtype == kBF16)
        cube_pool_kernel<__nv_bfloat16><<<dim3(p.n_cubes, p.heads, 2), CD, 0, st>>>(p);
    else
        cube_pool_kernel<__half><<<dim3(p.n_cubes, p.heads, 2), CD, 0, st>>>(p);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess)
        return e;
    const uint32_t nb = (p.n_cubes + 31) / 32;
    cube_scores_kernel<<<dim3(nb, nb, p.heads), 256, 0, st>>>(p);
    if ((e = cudaGetLastError()) != cudaSuccess)
        return e;
    cube_topk_kernel<<<dim3(p.n_cubes, p.heads), 256, 0, st>>>(p);
    return cudaGetLastError();
}

} // namespace mako
