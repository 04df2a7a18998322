// The output projection that consumes the attention's output, on sm_100a tensor cores: y[t][j] = sum_i x[t][i] w[j][i]
// for 16-bit x [T][k] (the attention's o in its 16-bit form, MAKO_OPT_OUTPUT_16BIT) and 16-bit w [n][k] of the same
// type, fp32 accumulate, fp32 y [T][ldy].  The reference runs this as Runtime::proj on a BF16 or F16 matrix
// (src/gpu/runtime.cpp:164-190: x rounded to 16 bits by to_bf16, then its GEMM), called right after the attention
// (src/models/h3.cpp:366, src/models/qwen_text.cpp:312).
//
// A persistent grid (one CTA per SM) walks 128 x 256 output tiles, row block by row block (a block of x stays in L2
// while the tiles of w pass over it).  Warp 0 loads x and w tiles of 64 k-values by TMA (128-byte swizzle) into a
// 4-stage ring; warp 1's elected thread issues tcgen05 UMMA (M 128, N 256, K 16, both operands K-major in shared
// memory) into one of two 256-column TMEM accumulators; warps 4-7 (one thread per tile row) read a finished
// accumulator and store its rows while the tensor core fills the other.  Every wait is bounded; a timeout records a
// code in the context's error flag and the CTA unwinds.
#include "common.cuh"
#include "kernels.h"
#include "tc100.cuh"

#include <cudaTypedefs.h>

namespace mako {
namespace {

using namespace tc;

constexpr uint32_t GM = 128, GN = 256, GK = 64, GSTAGES = 4, GNT = 256;
constexpr uint32_t GA_BYTES = GM * GK * 2, GB_BYTES = GN * GK * 2, GSTAGE = GA_BYTES + GB_BYTES;
constexpr uint32_t G_BAR = GSTAGES * GSTAGE;
constexpr uint32_t G_SMEM = G_BAR + 256 + 1024;  // + barriers + alignment slack
constexpr long long G_WAIT = 1ll << 31;          // clock cycles (~1 s) before a wait gives up

struct __align__(64) GemmParams {
    CUtensorMap tx, tw;  // x [T][k] and w [n][k], boxes of 64 k-values x 128 (x) or 256 (w) rows
    float* y;
    int* err;
    uint32_t T, k, n, ldy, fmt, tiles_n, n_tiles;
};

__device__ __forceinline__ void tma_load_2d(uint32_t dst, const CUtensorMap* map, uint32_t bar, int c0, int c1)
{
    asm volatile("cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
                 " [%0], [%1, {%3, %4}], [%2];\n" ::"r"(dst),
                 "l"(reinterpret_cast<uint64_t>(map)), "r"(bar), "r"(c0), "r"(c1)
                 : "memory");
}

__global__ void __launch_bounds__(GNT, 1) proj_gemm_kernel(const __grid_constant__ GemmParams p)
{
    extern __shared__ uint8_t smem_raw[];
    const uint32_t raw = smem_u32(smem_raw);
    const uint32_t base = (raw + 1023u) & ~1023u;
    const uint32_t sB = base + G_BAR;
    auto full = [&](uint32_t s) { return sB + 8 * s; };
    auto empty = [&](uint32_t s) { return sB + 32 + 8 * s; };
    auto acc_full = [&](uint32_t b) { return sB + 64 + 8 * b; };
    auto acc_empty = [&](uint32_t b) { return sB + 80 + 8 * b; };
    const uint32_t mma_done = sB + 96, tmem_slot = sB + 104;
    volatile uint32_t* tmem_slot_ptr = reinterpret_cast<volatile uint32_t*>(smem_raw + (tmem_slot - raw));
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t kb_n = p.k / GK;  // k-steps per tile

    if (threadIdx.x == 0) {
        for (uint32_t s = 0; s < GSTAGES; ++s) {
            mbar_init(full(s), 1);
            mbar_init(empty(s), 1);
        }
        for (uint32_t b = 0; b < 2; ++b) {
            mbar_init(acc_full(b), 1);
            mbar_init(acc_empty(b), 4);  // one arrival per epilogue warp
        }
        mbar_init(mma_done, 1);
        fence_barrier_init();
    }
    if (warp == 1) {
        tmem_alloc(tmem_slot, 512);
        tmem_relinquish();
    }
    fence_before();
    __syncthreads();
    fence_after();
    const uint32_t tmem = *tmem_slot_ptr;

    if (warp == 0 && lane == 0) {
        // ---------------- TMA producer ----------------
        tma_prefetch_desc(&p.tx);
        tma_prefetch_desc(&p.tw);
        bool ok = true;
        uint32_t g = 0;  // k-steps loaded so far (ring stage and phase)
        for (uint32_t tile = blockIdx.x; tile < p.n_tiles && ok; tile += gridDim.x) {
            const int m0 = int((tile / p.tiles_n) * GM), n0 = int((tile % p.tiles_n) * GN);
            for (uint32_t kb = 0; kb < kb_n; ++kb, ++g) {
                const uint32_t s = g % GSTAGES, ph = (g / GSTAGES) & 1;
                if (g >= GSTAGES && !mbar_wait(empty(s), ph ^ 1, G_WAIT)) {
                    ok = false;
                    break;
                }
                const uint32_t sa = base + s * GSTAGE;
                mbar_expect_tx(full(s), GSTAGE);
                tma_load_2d(sa, &p.tx, full(s), int(kb * GK), m0);
                tma_load_2d(sa + GA_BYTES, &p.tw, full(s), int(kb * GK), n0);
            }
        }
        if (!ok)
            atomicExch(p.err, 21);
        // our copies in flight land before the CTA leaves (already so on the normal path)
        for (uint32_t i = g > GSTAGES ? g - GSTAGES : 0; i < g; ++i)
            mbar_wait(full(i % GSTAGES), (i / GSTAGES) & 1, G_WAIT);
    } else if (warp == 1 && lane == 0) {
        // ---------------- UMMA issuer ----------------
        const uint32_t idesc = idesc_f16(p.fmt, p.fmt, 0, 0, GM, GN);
        bool ok = true;
        uint32_t g = 0, a = 0;  // k-steps consumed, tiles accumulated
        for (uint32_t tile = blockIdx.x; tile < p.n_tiles && ok; tile += gridDim.x, ++a) {
            const uint32_t b = a & 1;
            if (a >= 2 && !(ok = mbar_wait(acc_empty(b), ((a - 2) >> 1) & 1, G_WAIT)))
                break;
            fence_after();
            for (uint32_t kb = 0; kb < kb_n; ++kb, ++g) {
                const uint32_t s = g % GSTAGES;
                if (!(ok = mbar_wait(full(s), (g / GSTAGES) & 1, G_WAIT)))
                    break;
                fence_after();
                const uint32_t sa = base + s * GSTAGE;
#pragma unroll
                for (uint32_t ks = 0; ks < GK / 16; ++ks)
                    umma_ss(tmem + b * GN, sdesc(sa + ks * 32, 16, 1024), sdesc(sa + GA_BYTES + ks * 32, 16, 1024),
                            idesc, (kb | ks) != 0);
                umma_commit(empty(s));  // the stage is free once these products have read it
            }
            if (ok)
                umma_commit(acc_full(b));
        }
        if (!ok)
            atomicExch(p.err, 22);
        umma_commit(mma_done);  // every MMA issued above has finished before TMEM is freed
        mbar_wait(mma_done, 0, G_WAIT);
    } else if (warp >= 4) {
        // ---------------- epilogue: tile row `row` ----------------
        const uint32_t row = (warp & 3) * 32 + lane, tl = tmem + (((warp & 3) * 32) << 16);
        bool ok = true;
        uint32_t a = 0;
        for (uint32_t tile = blockIdx.x; tile < p.n_tiles && ok; tile += gridDim.x, ++a) {
            const uint32_t b = a & 1;
            ok = __all_sync(0xffffffffu, mbar_wait(acc_full(b), (a >> 1) & 1, G_WAIT));
            if (!ok)
                break;
            fence_after();
            const uint32_t t = (tile / p.tiles_n) * GM + row, n0 = (tile % p.tiles_n) * GN;
            float* const yrow = p.y + uint64_t(t) * p.ldy;
#pragma unroll 1
            for (uint32_t c = 0; c < GN / 32; ++c) {
                uint32_t r[32];
                tmem_ld32(tl + b * GN + c * 32, r);
                tmem_wait_ld();
                reg_fence(r);
                const uint32_t j0 = n0 + c * 32;
                if (t >= p.T || j0 >= p.n)
                    continue;
                if (j0 + 32 <= p.n) {
                    out_store32(yrow, j0, r, 1.0f, 0);
                } else {
                    for (uint32_t e = 0; j0 + e < p.n; ++e)
                        yrow[j0 + e] = __uint_as_float(r[e]);
                }
            }
            fence_before();
            __syncwarp();
            if (lane == 0)
                mbar_arrive(acc_empty(b));
        }
        if (!ok && lane == 0)
            atomicExch(p.err, 23);
    }
    __syncwarp();
    fence_before();
    __syncthreads();
    if (warp == 1) {
        fence_after();
        tmem_dealloc(tmem, 512);
    }
}

// [rows][k] 16-bit matrix as a TMA source: boxes of 64 k-values (128 bytes, the 128-byte swizzle) x box_rows rows.
bool rows_map(CUtensorMap* map, const void* ptr, bool bf16, uint32_t k, uint32_t rows, uint32_t box_rows)
{
    auto enc = tensor_map_encoder();
    if (!enc)
        return false;
    cuuint64_t dims[2] = {k, rows};
    cuuint64_t strides[1] = {uint64_t(k) * 2};
    cuuint32_t box[2] = {GK, box_rows};
    cuuint32_t estr[2] = {1, 1};
    return enc(map, bf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2,
               const_cast<void*>(ptr), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
               CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
               CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

} // namespace

cudaError_t launch_proj_gemm(const ProjParams& a, int dtype, int* err, cudaStream_t st)
{
    if (a.T == 0 || a.n == 0)
        return cudaSuccess;
    GemmParams p;
    const bool bf = dtype == kBF16;
    if (!rows_map(&p.tx, a.x, bf, a.k, a.T, GM) || !rows_map(&p.tw, a.w, bf, a.k, a.n, GN))
        return cudaErrorInvalidValue;
    p.y = a.y;
    p.err = err;
    p.T = a.T;
    p.k = a.k;
    p.n = a.n;
    p.ldy = a.ldy;
    p.fmt = bf ? 1u : 0u;
    p.tiles_n = (a.n + GN - 1) / GN;
    p.n_tiles = ((a.T + GM - 1) / GM) * p.tiles_n;
    cudaError_t e = cudaFuncSetAttribute(proj_gemm_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, G_SMEM);
    if (e != cudaSuccess)
        return e;
    const uint32_t sms = a.num_sms ? a.num_sms : 148;
    proj_gemm_kernel<<<p.n_tiles < sms ? p.n_tiles : sms, GNT, G_SMEM, st>>>(p);
    return cudaGetLastError();
}

} // namespace mako
