// Head-tile producers: the 16-bit [heads][n_pad][dim] tiles every attention call reads, made from fp32 projection
// rows, RMS-normed per head and rotated by RoPE angles on the way -- TransformerRuntime::heads, heads_norm and
// heads_partial (src/models/runtime.cpp:215-260; kernels heads_half, heads_norm_half, heads_partial,
// src/kernels/ops.metal:11-43,371-408,577-613) -- and heads_clear (ops.metal:45-52).
//
// HBM-bound: a warp takes one output row of up to 8 heads, each lane dim / 32 consecutive values of each (128-bit
// loads for 128-wide heads, the 8 heads' loads in flight together, the row's angles and the norm weights read once);
// a head's sum of squares is a warp reduction (the row's heads reduce interleaved); rotation partners (i with
// i + rot / 2, or 2i with 2i + 1) come from the same lane, a shuffle, or a per-warp shared-memory copy of the row when
// the pairing crosses lanes unevenly.
#include "kernels.h"

#include <cuda_bf16.h>
#include <cuda_fp16.h>

namespace mako {
namespace {

// Warps (rows) a CTA.  One: every warp is scheduled on its own, so a slot frees the moment its row is stored and the
// small k and v calls (1.7 waves of rows) end on a warp-sized tail rather than a CTA-sized one (0.1170 against 0.1218
// ms for a step of config 3's six calls with 4-warp CTAs).
constexpr int HW = 1;

template <typename T>
__device__ __forceinline__ T to16(float v);
template <>
__device__ __forceinline__ __half to16<__half>(float v)
{
    return __float2half_rn(v);
}
template <>
__device__ __forceinline__ __nv_bfloat16 to16<__nv_bfloat16>(float v)
{
    return __float2bfloat16_rn(v);
}

#ifndef MAKO_HEADS_HPW
#define MAKO_HEADS_HPW 8
#endif
// heads a warp takes of its row: their loads are in flight together, and the row's angles and the norm weights are
// read once for all of them
constexpr int HPW = MAKO_HEADS_HPW;

// VPL values a lane as 16-bit, packed into as few stores as the width allows.
template <int VPL, typename T>
__device__ __forceinline__ void store16(T* dst, const float (&v)[VPL])
{
    if (VPL % 4 == 0) {
#pragma unroll
        for (int k = 0; k < VPL; k += 4) {
            uint2 w;
            T a[4] = {to16<T>(v[k]), to16<T>(v[k + 1]), to16<T>(v[k + 2]), to16<T>(v[k + 3])};
            memcpy(&w, a, 8);
            *reinterpret_cast<uint2*>(dst + k) = w;
        }
    } else if (VPL % 2 == 0) {
#pragma unroll
        for (int k = 0; k < VPL; k += 2) {
            T a[2] = {to16<T>(v[k]), to16<T>(v[k + 1])};
            uint32_t w;
            memcpy(&w, a, 4);
            *reinterpret_cast<uint32_t*>(dst + k) = w;
        }
    } else {
#pragma unroll
        for (int k = 0; k < VPL; ++k)
            dst[k] = to16<T>(v[k]);
    }
}

// The (cos, sin) angle of each of this lane's values (value i < rot pairs with i +- rot / 2 and takes angle
// i mod rot / 2; adjacent pairs 2i, 2i + 1 take angle i), loaded with the row's values so that both round trips to
// memory overlap; (1, 0) past rot.
template <int VPL>
__device__ __forceinline__ void load_angles(const HeadsParams& p, const float2* cs, int lane, float2 (&ang)[VPL])
{
    const uint32_t half = p.rot / 2;
#pragma unroll
    for (int k = 0; k < VPL; ++k) {
        const uint32_t i = lane * VPL + k;
        ang[k] = make_float2(1.0f, 0.0f);
        if (p.rope == 2)
            ang[k] = __ldg(cs + i / 2);
        else if (i < p.rot)
            ang[k] = __ldg(cs + (i < half ? i : i - half));
    }
}

// The rest of row r (model row t) once the values of its nh heads from h0 are in registers: RMS norm, rotation and
// the 16-bit stores (zeros for t < 0).  ang: the angles of this lane's values (load_angles), wv: their norm
// weights, buf: dim floats of per-warp scratch, used when rotation partners cross lanes unevenly.
template <int VPL, int NH, typename T>
__device__ __forceinline__ void row_out(const HeadsParams& p, int32_t t, uint32_t r, uint32_t h0, uint32_t nh,
                                        float (&v)[NH][VPL], const float (&wv)[VPL], const float2 (&ang)[VPL],
                                        float* buf, int lane)
{
    T* const y0 = static_cast<T*>(p.y) + (uint64_t(h0) * p.n_pad + p.row0 + r) * p.dim + lane * VPL;
    const uint64_t ystep = uint64_t(p.n_pad) * p.dim;
    if (t < 0) {  // a row the map leaves empty is zero
        float z[VPL];
#pragma unroll
        for (int k = 0; k < VPL; ++k)
            z[k] = 0.0f;
        for (uint32_t j = 0; j < nh; ++j)
            store16<VPL, T>(y0 + j * ystep, z);
        return;
    }
    // the sign of the partner's term: -s for the first of a pair, +s for the second
    float cc[VPL], sn[VPL];
    const uint32_t half = p.rot / 2;
    if (p.rope) {
#pragma unroll
        for (int k = 0; k < VPL; ++k) {
            const uint32_t i = lane * VPL + k;
            const bool first = p.rope == 2 ? (i & 1) == 0 : i < half;
            cc[k] = ang[k].x;
            sn[k] = first ? -ang[k].y : ang[k].y;
        }
    }
    // Every step runs over all NH heads at once (heads past nh hold zeros and are not stored), so the heads' shuffle
    // chains overlap instead of following one another.
#pragma unroll
    for (int j = 0; j < NH; ++j)
        if (uint32_t(j) >= nh)
#pragma unroll
            for (int k = 0; k < VPL; ++k)
                v[j][k] = 0.0f;
    if (p.eps > 0.0f) {  // RMS norm over each head, times w
        float ss[NH];
#pragma unroll
        for (int j = 0; j < NH; ++j) {
            ss[j] = 0.0f;
#pragma unroll
            for (int k = 0; k < VPL; ++k)
                ss[j] = fmaf(v[j][k], v[j][k], ss[j]);
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1)
#pragma unroll
            for (int j = 0; j < NH; ++j)
                ss[j] += __shfl_xor_sync(0xffffffffu, ss[j], o);
#pragma unroll
        for (int j = 0; j < NH; ++j) {
            const float inv = rsqrtf(ss[j] / float(p.dim) + p.eps);
#pragma unroll
            for (int k = 0; k < VPL; ++k)
                v[j][k] *= inv * wv[k];
        }
    }
    if (p.rope) {
        // rotation partners: within the lane (adjacent pairs, even VPL), a fixed lane away (halves whose offset is a
        // whole number of lanes), or through shared memory otherwise
        const bool in_lane = p.rope == 2 && VPL % 2 == 0;
        const bool by_shfl = p.rope == 1 && half % VPL == 0;
        const int hl = int(half / VPL), src = lane < hl ? lane + hl : lane - hl;
        // x' = x c - y s for the first of a pair, y' = y c + x s for the second (sn carries the sign)
        if (in_lane) {
#pragma unroll
            for (int j = 0; j < NH; ++j)
#pragma unroll
                for (int k = 0; k < VPL; k += 2) {
                    const float a = v[j][k], b = v[j][k + 1];
                    v[j][k] = fmaf(a, cc[k], b * sn[k]);
                    v[j][k + 1] = fmaf(b, cc[k + 1], a * sn[k + 1]);
                }
        } else if (by_shfl) {
            // the partner of this lane's value k is value k of lane src, read before either is rewritten
#pragma unroll
            for (int j = 0; j < NH; ++j)
#pragma unroll
                for (int k = 0; k < VPL; ++k) {
                    const float q = __shfl_sync(0xffffffffu, v[j][k], src);
                    if (lane * VPL + k < p.rot)
                        v[j][k] = fmaf(v[j][k], cc[k], q * sn[k]);
                }
        } else {
#pragma unroll
            for (int j = 0; j < NH; ++j) {
                float* const hb = buf;
                __syncwarp();
#pragma unroll
                for (int k = 0; k < VPL; ++k)
                    hb[lane * VPL + k] = v[j][k];
                __syncwarp();
#pragma unroll
                for (int k = 0; k < VPL; ++k) {
                    const uint32_t i = lane * VPL + k;
                    const uint32_t pi = p.rope == 2 ? (i ^ 1) : (i < half ? i + half : i - half);
                    const float q = pi < p.dim ? hb[pi] : 0.0f;
                    if (p.rope == 2 || i < p.rot)
                        v[j][k] = fmaf(v[j][k], cc[k], q * sn[k]);
                }
            }
        }
    }
#pragma unroll
    for (int j = 0; j < NH; ++j)
        if (uint32_t(j) < nh)
            store16<VPL, T>(y0 + j * ystep, v[j]);
}

template <int VPL, typename T>
__global__ void __launch_bounds__(HW * 32, (VPL <= 4 ? 32 : 16) / HW) heads_kernel(const HeadsParams p)
{
    __shared__ float row_buf[HW][VPL * 32];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t r = blockIdx.x * HW + warp, h0 = blockIdx.y * HPW;
    if (r >= p.rows)
        return;
    const uint32_t nh = min(uint32_t(HPW), p.heads - h0);
    const int32_t t = p.map ? p.map[r] : int32_t(r);
    float v[HPW][VPL];
    float wv[VPL];
    float2 ang[VPL];
    if (t >= 0) {
        // all the warp's heads of this row in flight at once
        const float* const x0 = p.x + uint64_t(t) * p.ld + p.col0 + uint64_t(h0) * p.stride + lane * VPL;
#pragma unroll
        for (int j = 0; j < HPW; ++j) {
            if (uint32_t(j) < nh) {
                if (VPL % 4 == 0 && p.vec4) {
#pragma unroll
                    for (int k = 0; k < VPL; k += 4) {
                        const float4 w = __ldg(reinterpret_cast<const float4*>(x0 + j * p.stride + k));
                        v[j][k] = w.x;
                        v[j][k + 1] = w.y;
                        v[j][k + 2] = w.z;
                        v[j][k + 3] = w.w;
                    }
                } else {
#pragma unroll
                    for (int k = 0; k < VPL; ++k)
                        v[j][k] = __ldg(x0 + j * p.stride + k);
                }
            }
        }
        if (p.eps > 0.0f)
#pragma unroll
            for (int k = 0; k < VPL; ++k)
                wv[k] = __ldg(p.w + lane * VPL + k);
        if (p.rope)
            load_angles<VPL>(p, reinterpret_cast<const float2*>(p.cs) + uint64_t(t) * p.cs_row, lane, ang);
    }
    row_out<VPL, HPW, T>(p, t, r, h0, nh, v, wv, ang, row_buf[warp], lane);
}

template <typename T>
cudaError_t launch_heads_t(const HeadsParams& p, cudaStream_t st)
{
    const dim3 grid((p.rows + HW - 1) / HW, (p.heads + HPW - 1) / HPW);
    switch (p.dim / 32) {
    case 1:
        heads_kernel<1, T><<<grid, HW * 32, 0, st>>>(p);
        break;
    case 2:
        heads_kernel<2, T><<<grid, HW * 32, 0, st>>>(p);
        break;
    case 3:
        heads_kernel<3, T><<<grid, HW * 32, 0, st>>>(p);
        break;
    case 4:
        heads_kernel<4, T><<<grid, HW * 32, 0, st>>>(p);
        break;
    case 5:
        heads_kernel<5, T><<<grid, HW * 32, 0, st>>>(p);
        break;
    case 6:
        heads_kernel<6, T><<<grid, HW * 32, 0, st>>>(p);
        break;
    case 7:
        heads_kernel<7, T><<<grid, HW * 32, 0, st>>>(p);
        break;
    case 8:
        heads_kernel<8, T><<<grid, HW * 32, 0, st>>>(p);
        break;
    default:
        return cudaErrorInvalidValue;
    }
    return cudaGetLastError();
}

} // namespace

cudaError_t launch_heads(const HeadsParams& p, int dtype, cudaStream_t st)
{
    if (p.rows == 0 || p.heads == 0)
        return cudaSuccess;
    return dtype == kBF16 ? launch_heads_t<__nv_bfloat16>(p, st) : launch_heads_t<__half>(p, st);
}

} // namespace mako
