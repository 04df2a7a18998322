// Device helpers shared by the attention kernels: 16-bit element traits, cp.async, ldmatrix, mma.sync, ex2.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <stdint.h>

namespace mako {

constexpr float kLog2e = 1.4426950408889634f;

__device__ __forceinline__ uint32_t smem_u32(const void* p) { return uint32_t(__cvta_generic_to_shared(p)); }

// ---- output element type (o_type: 0 fp32, 1 fp16, 2 bf16; the 16-bit types round to nearest even) ----------------

__device__ __forceinline__ uint32_t out_pack2(float a, float b, uint32_t o_type)
{
    if (o_type == 1) {
        __half2 v = __floats2half2_rn(a, b);
        return *reinterpret_cast<uint32_t*>(&v);
    }
    __nv_bfloat162 v = __floats2bfloat162_rn(a, b);
    return *reinterpret_cast<uint32_t*>(&v);
}
// o[i] = v
__device__ __forceinline__ void out_store1(void* o, uint64_t i, float v, uint32_t o_type)
{
    if (o_type == 0)
        static_cast<float*>(o)[i] = v;
    else if (o_type == 1)
        static_cast<__half*>(o)[i] = __float2half_rn(v);
    else
        static_cast<__nv_bfloat16*>(o)[i] = __float2bfloat16_rn(v);
}
// o[i], o[i + 1] = a, b (i even)
__device__ __forceinline__ void out_store2(void* o, uint64_t i, float a, float b, uint32_t o_type)
{
    if (o_type == 0)
        *reinterpret_cast<float2*>(static_cast<float*>(o) + i) = make_float2(a, b);
    else
        *reinterpret_cast<uint32_t*>(static_cast<uint16_t*>(o) + i) = out_pack2(a, b, o_type);
}
// o[i .. i + 32) = r[0 .. 32) (fp32 bits) * s, i a multiple of 8 and o 16-byte aligned: 128-bit stores
__device__ __forceinline__ void st_global_v8(void* d, const uint32_t (&w)[8])
{
    asm volatile("st.global.v8.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8};\n" ::"l"(d), "r"(w[0]), "r"(w[1]), "r"(w[2]),
                 "r"(w[3]), "r"(w[4]), "r"(w[5]), "r"(w[6]), "r"(w[7])
                 : "memory");
}

// 32 consecutive output values of one row (r[k] * s), fp32 or 16-bit.  32-byte stores (whole sectors) where the row
// slice is 32-byte aligned, else 16-byte stores: a warp's 32 rows are 32 scattered slices, so fewer, fuller stores
// cost less.
__device__ __forceinline__ void out_store32(void* o, uint64_t i, const uint32_t (&r)[32], float s, uint32_t o_type)
{
    if (o_type == 0) {
        float* d = static_cast<float*>(o) + i;
        if ((reinterpret_cast<uintptr_t>(d) & 31) == 0) {
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                uint32_t w[8];
#pragma unroll
                for (int k = 0; k < 8; ++k)
                    w[k] = __float_as_uint(__uint_as_float(r[8 * e + k]) * s);
                st_global_v8(d + 8 * e, w);
            }
            return;
        }
#pragma unroll
        for (int e = 0; e < 8; ++e)
            *reinterpret_cast<float4*>(d + 4 * e) =
                make_float4(__uint_as_float(r[4 * e]) * s, __uint_as_float(r[4 * e + 1]) * s,
                            __uint_as_float(r[4 * e + 2]) * s, __uint_as_float(r[4 * e + 3]) * s);
        return;
    }
    uint16_t* d = static_cast<uint16_t*>(o) + i;
    if ((reinterpret_cast<uintptr_t>(d) & 31) == 0) {
#pragma unroll
        for (int e = 0; e < 2; ++e) {
            uint32_t w[8];
#pragma unroll
            for (int k = 0; k < 8; ++k)
                w[k] = out_pack2(__uint_as_float(r[16 * e + 2 * k]) * s, __uint_as_float(r[16 * e + 2 * k + 1]) * s,
                                 o_type);
            st_global_v8(d + 16 * e, w);
        }
        return;
    }
#pragma unroll
    for (int e = 0; e < 4; ++e) {
        uint32_t w[4];
#pragma unroll
        for (int k = 0; k < 4; ++k)
            w[k] = out_pack2(__uint_as_float(r[8 * e + 2 * k]) * s, __uint_as_float(r[8 * e + 2 * k + 1]) * s, o_type);
        *reinterpret_cast<uint4*>(d + 8 * e) = make_uint4(w[0], w[1], w[2], w[3]);
    }
}

// 16 bytes global -> shared, zero-filled when !pred (nothing is read then).
__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src, bool pred)
{
    const int n = pred ? 16 : 0;
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;\n" ::"r"(dst), "l"(src), "r"(n) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;\n" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait()
{
    asm volatile("cp.async.wait_group %0;\n" ::"n"(N) : "memory");
}

__device__ __forceinline__ void ldsm_x4(uint32_t (&r)[4], uint32_t addr)
{
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];\n"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
                 : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t (&r)[4], uint32_t addr)
{
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];\n"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
                 : "r"(addr));
}

// Element traits: the 16-bit type, its mma.sync spelling, packing two floats.
template <typename T>
struct Elem;
template <>
struct Elem<__half> {
    static __device__ __forceinline__ uint32_t pack(float lo, float hi)
    {
        __half2 h = __floats2half2_rn(lo, hi);
        return *reinterpret_cast<uint32_t*>(&h);
    }
    static __device__ __forceinline__ float to_f(__half x) { return __half2float(x); }
};
template <>
struct Elem<__nv_bfloat16> {
    static __device__ __forceinline__ uint32_t pack(float lo, float hi)
    {
        __nv_bfloat162 h = __floats2bfloat162_rn(lo, hi);
        return *reinterpret_cast<uint32_t*>(&h);
    }
    static __device__ __forceinline__ float to_f(__nv_bfloat16 x) { return __bfloat162float(x); }
};

// D += A (16x16, row) * B (16x8, col), fp32 accumulate.
__device__ __forceinline__ void mma16816(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1, __half)
{
    asm volatile("mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
                 "{%0,%1,%2,%3};\n"
                 : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
                 : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
__device__ __forceinline__ void mma16816(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1,
                                         __nv_bfloat16)
{
    asm volatile("mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
                 "{%0,%1,%2,%3};\n"
                 : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
                 : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// 2^x with the hardware's approximate exponential (PTX ex2.approx.ftz.f32); 2^-inf = 0.
__device__ __forceinline__ float ex2(float x)
{
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;\n" : "=f"(y) : "f"(x));
    return y;
}

// Byte offset of 16-byte chunk `c` of row `r` in a tile whose rows are `row_bytes` long, the chunks XOR-swizzled
// by the row's low three bits so that ldmatrix over 8 consecutive rows touches 8 distinct bank groups.
__device__ __forceinline__ uint32_t swz(uint32_t r, uint32_t c, uint32_t row_bytes)
{
    return r * row_bytes + ((c ^ (r & 7)) << 4);
}

} // namespace mako
