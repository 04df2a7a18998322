// cube_select (TransformerRuntime::cube_select, src/models/runtime.cpp:286-303): for block-sparse attention over
// 64-row cubes, per head and query cube the `topk` key cubes whose mean-pooled k best matches the cube's mean-pooled q.
//
//   cube_pool   (ops.metal:927-939)  mean over a cube's 64 rows (all summed, invalid rows are zero) / cnt[c]
//   cube_scores (ops.metal:942-955)  sc[h][qc][kc] = qp . kp
//   cube_topk   (ops.metal:959-1027) the local cubes first, then the largest scores, ties to the smaller index
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

// One CTA of 256 per (query cube, head); at most 4096 cubes (the reference's bound).
__global__ void __launch_bounds__(256) cube_topk_kernel(const CubeParams p)
{
    __shared__ float scores[4096];
    __shared__ float best_v[8];
    __shared__ uint32_t best_i[8];
    __shared__ uint32_t n_local;
    const uint32_t qc = blockIdx.x, h = blockIdx.y, n = p.n_cubes, tid = threadIdx.x, lane = tid & 31, wid = tid >> 5;
    const float* row = p.sc + (uint64_t(h) * n + qc) * n;
    for (uint32_t i = tid; i < n; i += 256)
        scores[i] = row[i];
    const uint32_t k = min(p.topk, n);
    uint16_t* out = p.sel + (uint64_t(h) * n + qc) * k;
    __syncthreads();
    uint32_t it = 0;
    if (p.local) {
        if (tid == 0) {
            const uint32_t picks[3] = {qc, qc >= p.stride ? qc - p.stride : n, qc + p.stride < n ? qc + p.stride : n};
            uint32_t c = 0;
            for (uint32_t j = 0; j < p.local && c < k; ++j)
                if (picks[j] < n) {
                    out[c++] = uint16_t(picks[j]);
                    scores[picks[j]] = -INFINITY;
                }
            n_local = c;
        }
        __syncthreads();
        it = n_local;
    }
    for (; it < k; ++it) {
        float v = -INFINITY;
        uint32_t idx = 0;
        for (uint32_t i = tid; i < n; i += 256)
            if (scores[i] > v) {
                v = scores[i];
                idx = i;
            }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            const float ov = __shfl_xor_sync(0xffffffffu, v, o);
            const uint32_t oi = __shfl_xor_sync(0xffffffffu, idx, o);
            if (ov > v || (ov == v && oi < idx)) {
                v = ov;
                idx = oi;
            }
        }
        if (lane == 0) {
            best_v[wid] = v;
            best_i[wid] = idx;
        }
        __syncthreads();
        if (tid == 0) {
            float bv = best_v[0];
            uint32_t bi = best_i[0];
            for (int j = 1; j < 8; ++j)
                if (best_v[j] > bv || (best_v[j] == bv && best_i[j] < bi)) {
                    bv = best_v[j];
                    bi = best_i[j];
                }
            out[it] = uint16_t(bi);
            scores[bi] = -INFINITY;
        }
        __syncthreads();
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
