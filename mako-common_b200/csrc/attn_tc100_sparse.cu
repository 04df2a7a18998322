// Block-sparse attention on sm_100a tensor cores: TransformerRuntime::attention_sparse (src/models/runtime.cpp:305-317,
// kernel flash_attn_sparse_128, src/kernels/ops.metal:1039-1185) for 128-wide heads.
//
// The reference's unit is a 64-row query cube with its own list of 64-row key cubes, but full-rate UMMA tiles are
// 128 rows.  A 128-row tile here holds two query cubes and walks their lists in lockstep: pass k loads cube A's k-th
// key cube into key rows 0-63 and cube B's k-th into rows 64-127, so S = Q K^T is block-diagonal -- rows of cube A
// see only keys 0-63, rows of cube B only 64-127 -- and the softmax computes only the 64 useful columns of each row,
// writing zeros into the other half of P.  Then the tile's dense passes ([dense0, dense1), shared by both cubes) and
// the query rows after the cubes (every valid key below n_k) run as full 128-key tiles.  A list shorter than its
// partner's is padded with empty passes; an entry >= n_cubes is skipped.  Masking per key: valid[key] and the pass's
// key range (ops.metal:1109); output row r goes to o row map[r], dropped when < 0 (ops.metal:1174-1184).
//
// CTA: two such tiles (A, B) with their own single-stage K and V buffers (the two tiles' loads and products
// interleave), warp 0 TMA (K / V as 64-row boxes so each half can come from anywhere), warp 1 the UMMA issuer
// (whichever product of either tile is ready), warps 4-7 / 8-11 the softmax of tile A / B, one row per thread.
// TMEM as the dense kernel: S_A, S_B, O_A, O_B.  Precision, bounded waits and the error flag as the dense kernel.
#include "common.cuh"
#include "kernels.h"
#include "tc100.cuh"

#include <cudaTypedefs.h>

namespace mako {
namespace {

using namespace tc;

constexpr int SD = 128, SNT = 384;
constexpr uint32_t QBOX = 128 * 64 * 2;  // a 128-row x 64-value box: 16 KB
constexpr uint32_t HBOX = 64 * 64 * 2;   // a 64-row x 64-value box: 8 KB
constexpr uint32_t STILE = 2 * QBOX;     // 128 rows x 128 values
constexpr uint32_t S_Q = 0, S_K = 2 * STILE, S_V = 4 * STILE, S_BAR = 6 * STILE;
constexpr uint32_t S_TOTAL = S_BAR + 256 + 1024;
constexpr long long S_WAIT_LIMIT = 1ll << 31;

struct __align__(64) SpParams {
    CUtensorMap tq;      // q, 128-row boxes
    CUtensorMap tk, tv;  // k and v (or the fp16 copy of v), 64-row boxes
    float* o;
    int* err;
    const float* vinv;
    const void* sel;
    const void* nsel;
    const uint8_t* valid;
    const int32_t* map;
    uint32_t sel_i32, qk_fmt;
    uint32_t n_q, q_pad, n_k, k_pad, heads, kv_heads, width, n_cubes, max_sel, dense0, dense1;
    uint32_t tiles_cube, tiles_total;
    float scale_log2;
};

struct TileInfo {
    uint32_t active, cube, row0, ncp, np;  // cube passes, all passes
    uint32_t cube_id[2], ns[2];
};

__device__ __forceinline__ uint32_t list_entry(const SpParams& p, const void* base, uint64_t i)
{
    return p.sel_i32 ? uint32_t(static_cast<const int32_t*>(base)[i]) : uint32_t(static_cast<const uint16_t*>(base)[i]);
}

__device__ __forceinline__ TileInfo tile_info(const SpParams& p, uint32_t u, uint32_t h)
{
    TileInfo t{};
    if (u >= p.tiles_total)
        return t;
    t.active = 1;
    if (u < p.tiles_cube) {
        t.cube = 1;
        t.row0 = u * 128;
        for (uint32_t hh = 0; hh < 2; ++hh) {
            const uint32_t c = 2 * u + hh;
            t.cube_id[hh] = c;
            uint32_t n = 0;
            if (c < p.n_cubes) {
                const int64_t raw = p.sel_i32 ? int64_t(static_cast<const int32_t*>(p.nsel)[uint64_t(h) * p.n_cubes + c])
                                              : int64_t(static_cast<const uint16_t*>(p.nsel)[uint64_t(h) * p.n_cubes + c]);
                n = raw <= 0 ? 0u : (raw < int64_t(p.max_sel) ? uint32_t(raw) : p.max_sel);
            }
            t.ns[hh] = n;
        }
        t.ncp = max(t.ns[0], t.ns[1]);
        t.np = t.ncp + (p.dense1 > p.dense0 ? (p.dense1 - p.dense0 + 127) / 128 : 0);
    } else {
        t.row0 = p.n_cubes * 64 + (u - p.tiles_cube) * 128;
        t.np = (p.n_k + 127) / 128;
    }
    return t;
}

// Key rows of pass `pi`, half `hh` (tile rows 64 hh .. 64 hh + 63 of K / V): they start at j0; keys j < hi are in
// range.  Cube passes: the half belongs to one query cube (empty: hi = j0 = 0).  Other passes: 128 consecutive keys.
__device__ __forceinline__ void pass_keys(const SpParams& p, const TileInfo& t, uint32_t h, uint32_t pi, uint32_t hh,
                                          uint32_t& j0, uint32_t& hi)
{
    if (t.cube && pi < t.ncp) {
        if (pi < t.ns[hh]) {
            const uint32_t c =
                list_entry(p, p.sel, (uint64_t(h) * p.n_cubes + t.cube_id[hh]) * p.max_sel + pi);
            if (c < p.n_cubes) {
                j0 = c * 64;
                hi = j0 + 64;
                return;
            }
        }
        j0 = 0;
        hi = 0;
        return;
    }
    const uint32_t base = t.cube ? p.dense0 + (pi - t.ncp) * 128 : pi * 128;
    j0 = base + 64 * hh;
    hi = t.cube ? p.dense1 : p.n_k;
}

__device__ __forceinline__ uint32_t pack_half2s(float lo, float hi)
{
    __half2 v = __floats2half2_rn(lo, hi);
    return *reinterpret_cast<uint32_t*>(&v);
}

__global__ void __launch_bounds__(SNT, 1) attn_tc_sparse_kernel(const __grid_constant__ SpParams p)
{
    extern __shared__ uint8_t smem_raw[];
    const uint32_t raw = smem_u32(smem_raw);
    const uint32_t base = (raw + 1023u) & ~1023u;
    const uint32_t sB = base + S_BAR;
    const uint32_t q_full = sB;
    auto k_full = [&](uint32_t x) { return sB + 8 + 8 * x; };
    auto k_empty = [&](uint32_t x) { return sB + 24 + 8 * x; };
    auto v_full = [&](uint32_t x) { return sB + 40 + 8 * x; };
    auto v_empty = [&](uint32_t x) { return sB + 56 + 8 * x; };
    auto s_full = [&](uint32_t x) { return sB + 72 + 8 * x; };
    auto p_full = [&](uint32_t x) { return sB + 88 + 8 * x; };
    auto pv_done = [&](uint32_t x) { return sB + 104 + 8 * x; };
    const uint32_t mma_done = sB + 120, tmem_slot = sB + 128;
    volatile uint32_t* tmem_slot_ptr = reinterpret_cast<volatile uint32_t*>(smem_raw + (tmem_slot - raw));

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t h = blockIdx.y, kvh = h / (p.heads / p.kv_heads);
    const uint32_t pair = gridDim.x - 1 - blockIdx.x;  // the row tiles after the cubes (all keys) first
    TileInfo ti[2] = {tile_info(p, 2 * pair, h), tile_info(p, 2 * pair + 1, h)};

    if (threadIdx.x == 0) {
        mbar_init(q_full, 1);
        for (uint32_t x = 0; x < 2; ++x) {
            mbar_init(k_full(x), 1);
            mbar_init(k_empty(x), 1);
            mbar_init(v_full(x), 1);
            mbar_init(v_empty(x), 1);
            mbar_init(s_full(x), 1);
            mbar_init(p_full(x), 128);
            mbar_init(pv_done(x), 1);
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

    if (warp == 0) {
        // ---------------- TMA producer ----------------
        if (lane == 0) {
            tma_prefetch_desc(&p.tq);
            tma_prefetch_desc(&p.tk);
            tma_prefetch_desc(&p.tv);
            const uint32_t nq = ti[0].active + ti[1].active;
            mbar_expect_tx(q_full, nq * STILE);
            for (uint32_t x = 0; x < 2; ++x)
                if (ti[x].active)
                    for (int dh = 0; dh < 2; ++dh)
                        tma_load_3d(base + S_Q + x * STILE + dh * QBOX, &p.tq, q_full, dh * 64, ti[x].row0, h);
            uint32_t kn[2] = {0, 0}, vn[2] = {0, 0};
            bool ok = true;
            long long idle_since = clock64();
            auto load = [&](const CUtensorMap* map, uint32_t dst, uint32_t bar, uint32_t x, uint32_t pi) {
                mbar_expect_tx(bar, STILE);
                for (uint32_t hh = 0; hh < 2; ++hh) {
                    uint32_t j0, hi;
                    pass_keys(p, ti[x], h, pi, hh, j0, hi);
                    for (int dh = 0; dh < 2; ++dh)
                        tma_load_3d(dst + dh * QBOX + hh * HBOX, map, bar, dh * 64, int(j0), kvh);
                }
            };
            while (ok && (kn[0] < ti[0].np || vn[0] < ti[0].np || kn[1] < ti[1].np || vn[1] < ti[1].np)) {
                bool progressed = false;
                for (uint32_t x = 0; x < 2; ++x) {
                    if (kn[x] < ti[x].np && (kn[x] == 0 || mbar_try_wait(k_empty(x), (kn[x] - 1) & 1))) {
                        load(&p.tk, base + S_K + x * STILE, k_full(x), x, kn[x]);
                        ++kn[x];
                        progressed = true;
                    }
                    if (vn[x] < ti[x].np && (vn[x] == 0 || mbar_try_wait(v_empty(x), (vn[x] - 1) & 1))) {
                        load(&p.tv, base + S_V + x * STILE, v_full(x), x, vn[x]);
                        ++vn[x];
                        progressed = true;
                    }
                }
                if (progressed)
                    idle_since = clock64();
                else if (clock64() - idle_since > S_WAIT_LIMIT)
                    ok = false;
            }
            if (!ok)
                atomicExch(p.err, 11);
            // Our copies in flight land before the CTA leaves (already so on the normal path).
            mbar_wait(q_full, 0, S_WAIT_LIMIT);
            for (uint32_t x = 0; x < 2; ++x) {
                if (kn[x])
                    mbar_wait(k_full(x), (kn[x] - 1) & 1, S_WAIT_LIMIT);
                if (vn[x])
                    mbar_wait(v_full(x), (vn[x] - 1) & 1, S_WAIT_LIMIT);
            }
        }
    } else if (warp == 1) {
        // ---------------- UMMA issuer ----------------
        if (lane == 0 && (ti[0].np || ti[1].np)) {
            const uint32_t idesc_qk = idesc_f16(p.qk_fmt, p.qk_fmt, 0, 0, 128, 128);
            const uint32_t idesc_pv = idesc_f16(0, 0, 0, 1, 128, SD);
            auto qk = [&](uint32_t x) {
#pragma unroll
                for (uint32_t ks = 0; ks < SD / 16; ++ks) {
                    const uint32_t off = (ks >> 2) * QBOX + (ks & 3) * 32;
                    umma_ss(tmem + x * 128, sdesc(base + S_Q + x * STILE + off, 16, 1024),
                            sdesc(base + S_K + x * STILE + off, 16, 1024), idesc_qk, ks > 0);
                }
            };
            auto pv = [&](uint32_t x, bool acc) {
#pragma unroll
                for (uint32_t kk = 0; kk < 8; ++kk)
                    umma_ts(tmem + 256 + x * 128, tmem + x * 128 + kk * 8,
                            sdesc(base + S_V + x * STILE + kk * 2048, QBOX, 1024), idesc_pv, acc || kk > 0);
            };
            bool ok = mbar_wait(q_full, 0, S_WAIT_LIMIT);
            uint32_t qn[2] = {0, 0}, pn[2] = {0, 0};
            long long idle_since = clock64();
            while (ok && (pn[0] < ti[0].np || pn[1] < ti[1].np)) {
                bool progressed = false;
#pragma unroll
                for (uint32_t x = 0; x < 2; ++x) {
                    const uint32_t i = qn[x];
                    // QK_X(i): K_X(i) landed and PV_X(i-1) finished (it read the P this overwrites)
                    if (i < ti[x].np && pn[x] == i && mbar_try_wait(k_full(x), i & 1) &&
                        (i == 0 || mbar_try_wait(pv_done(x), (i - 1) & 1))) {
                        fence_after();
                        qk(x);
                        umma_commit(s_full(x));
                        umma_commit(k_empty(x));
                        qn[x] = i + 1;
                        progressed = true;
                    }
                    const uint32_t j = pn[x];
                    // PV_X(j): P_X(j) written and V_X(j) landed
                    if (j < qn[x] && mbar_try_wait(p_full(x), j & 1) && mbar_try_wait(v_full(x), j & 1)) {
                        fence_after();
                        pv(x, j > 0);
                        umma_commit(pv_done(x));
                        umma_commit(v_empty(x));
                        pn[x] = j + 1;
                        progressed = true;
                    }
                }
                if (progressed)
                    idle_since = clock64();
                else if (clock64() - idle_since > S_WAIT_LIMIT)
                    ok = false;
            }
            if (!ok)
                atomicExch(p.err, 12);
            umma_commit(mma_done);
            mbar_wait(mma_done, 0, S_WAIT_LIMIT);
        }
    } else if (warp >= 4) {
        // ---------------- softmax (and epilogue) of tile X ----------------
        const uint32_t x = (warp - 4) >> 2, ql = (warp & 3) * 32, row = ql + lane, hr = ql >> 6;
        const TileInfo& t = ti[x];
        const uint32_t tl = tmem + (ql << 16);
        const uint32_t colS = x * 128, colO = 256 + x * 128;
        const float scale = p.scale_log2;
        const uint64_t scale2 = pack2(scale, scale);
        float m = -INFINITY, l = 0.0f;
        bool ok = true;
        for (uint32_t i = 0; i < t.np; ++i) {
            ok = __all_sync(0xffffffffu, mbar_wait(s_full(x), i & 1, S_WAIT_LIMIT));
            if (!ok)
                break;
            fence_after();
            const bool half = t.cube && i < t.ncp;  // this row sees only its cube's 64 keys
            uint32_t r[4][32];
            uint32_t j0, hi;
            if (half) {
                pass_keys(p, t, h, i, hr, j0, hi);
                tmem_ld32(tl + colS + 64 * hr, r[0]);
                tmem_ld32(tl + colS + 64 * hr + 32, r[1]);
                tmem_wait_ld();
                reg_fence(r[0]);
                reg_fence(r[1]);
                if (hi < j0 + 64 || p.valid) {
#pragma unroll
                    for (int c = 0; c < 64; ++c) {
                        const uint32_t jj = j0 + c;
                        if (jj >= hi || (p.valid && !p.valid[jj]))
                            r[c >> 5][c & 31] = 0xFF800000u;
                    }
                }
            } else {
                pass_keys(p, t, h, i, 0, j0, hi);
#pragma unroll
                for (int c = 0; c < 4; ++c)
                    tmem_ld32(tl + colS + c * 32, r[c]);
                tmem_wait_ld();
#pragma unroll
                for (int c = 0; c < 4; ++c)
                    reg_fence(r[c]);
                if (hi < j0 + 128 || p.valid) {
#pragma unroll
                    for (int c = 0; c < 128; ++c) {
                        const uint32_t jj = j0 + c;
                        if (jj >= hi || (p.valid && !p.valid[jj]))
                            r[c >> 5][c & 31] = 0xFF800000u;
                    }
                }
            }
            const int ncol = half ? 64 : 128;
            float mq[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
#pragma unroll
            for (int c = 0; c < 128; c += 8) {
                if (c < ncol) {
#pragma unroll
                    for (int s = 0; s < 4; ++s)
                        mq[s] = max3f(mq[s], __uint_as_float(r[(c + 2 * s) >> 5][(c + 2 * s) & 31]),
                                      __uint_as_float(r[(c + 2 * s + 1) >> 5][(c + 2 * s + 1) & 31]));
                }
            }
            const float mx = fmaxf(fmaxf(mq[0], mq[1]), fmaxf(mq[2], mq[3])) * scale;
            float f = 1.0f;
            bool resc = false;
            if (mx > m + 8.0f) {
                f = m == -INFINITY ? 0.0f : ex2(m - mx);
                m = mx;
                l *= f;
                resc = true;
            }
            const float mneg = m == -INFINITY ? 0.0f : -m;
            const uint64_t mneg2 = pack2(mneg, mneg);
            uint32_t pk[2][32];
            uint64_t sum2[2] = {pack2(0.0f, 0.0f), pack2(0.0f, 0.0f)};
#pragma unroll
            for (int c = 0; c < 64; ++c) {
                if (2 * c < ncol) {
                    const uint64_t xv = pack2(__uint_as_float(r[(2 * c) >> 5][(2 * c) & 31]),
                                              __uint_as_float(r[(2 * c + 1) >> 5][(2 * c + 1) & 31]));
                    float a, b;
                    unpack2(ffma2(xv, scale2, mneg2), a, b);
                    a = ex2(a);
                    b = ex2(b);
                    sum2[c & 1] = fadd2(sum2[c & 1], pack2(a, b));
                    pk[c >> 5][c & 31] = pack_half2s(a, b);
                } else {
                    pk[c >> 5][c & 31] = 0u;
                }
            }
            {
                float s0, s1, s2, s3;
                unpack2(sum2[0], s0, s1);
                unpack2(sum2[1], s2, s3);
                l += (s0 + s1) + (s2 + s3);
            }
            if (half) {
                // P of this row's cube sits at packed columns 32 hr .. 32 hr + 31, zeros in the other cube's half
                if (hr == 0) {
                    tmem_st32(tl + colS, pk[0]);
                    tmem_st32(tl + colS + 32, pk[1]);
                } else {
                    tmem_st32(tl + colS, pk[1]);
                    tmem_st32(tl + colS + 32, pk[0]);
                }
            } else {
                tmem_st32(tl + colS, pk[0]);
                tmem_st32(tl + colS + 32, pk[1]);
            }
            if (__any_sync(0xffffffffu, resc && i > 0)) {
                const float g = resc ? f : 1.0f;
#pragma unroll
                for (int c = 0; c < 4; ++c) {
                    uint32_t o[32];
                    tmem_ld32(tl + colO + c * 32, o);
                    tmem_wait_ld();
                    reg_fence(o);
#pragma unroll
                    for (int k = 0; k < 32; ++k)
                        o[k] = __float_as_uint(__uint_as_float(o[k]) * g);
                    tmem_st32(tl + colO + c * 32, o);
                }
            }
            tmem_wait_st();
            fence_before();
            mbar_arrive(p_full(x));
        }
        if (ok && t.np > 0) {
            ok = __all_sync(0xffffffffu, mbar_wait(pv_done(x), (t.np - 1) & 1, S_WAIT_LIMIT));
            fence_after();
        }
        if (!ok && lane == 0)
            atomicExch(p.err, 13);
        // Store: rows below n_q that belong to this tile (a cube tile's half past the last cube is another tile's).
        const uint32_t grow = t.row0 + row;
        bool store = t.active && grow < p.n_q && (!t.cube || t.cube_id[hr] < p.n_cubes);
        int64_t dst = grow;
        if (store && p.map) {
            dst = p.map[grow];
            store = dst >= 0;
        }
        const float inv = (l > 0.0f ? 1.0f / l : 0.0f) * (p.vinv ? p.vinv[kvh] : 1.0f);
        float* orow = p.o + uint64_t(dst) * p.width + uint64_t(h) * SD;
#pragma unroll
        for (int c = 0; c < 4; ++c) {
            uint32_t o[32];
            if (ok && t.np > 0) {
                tmem_ld32(tl + colO + c * 32, o);
                tmem_wait_ld();
                reg_fence(o);
            } else {
#pragma unroll
                for (int k = 0; k < 32; ++k)
                    o[k] = 0u;
            }
            if (store) {
#pragma unroll
                for (int k = 0; k < 8; ++k)
                    *reinterpret_cast<float4*>(orow + c * 32 + k * 4) =
                        make_float4(__uint_as_float(o[4 * k]) * inv, __uint_as_float(o[4 * k + 1]) * inv,
                                    __uint_as_float(o[4 * k + 2]) * inv, __uint_as_float(o[4 * k + 3]) * inv);
            }
        }
    }
    __syncwarp();
    fence_before();
    __syncthreads();
    if (warp == 1) {
        fence_after();
        tmem_dealloc(tmem, 512);
    }
}

PFN_cuTensorMapEncodeTiled_v12000 encode_sp()
{
    static PFN_cuTensorMapEncodeTiled_v12000 fn = [] {
        void* f = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &f, cudaEnableDefault, &q) != cudaSuccess ||
            q != cudaDriverEntryPointSuccess)
            return static_cast<PFN_cuTensorMapEncodeTiled_v12000>(nullptr);
        return reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(f);
    }();
    return fn;
}

bool map_rows(CUtensorMap* map, const void* ptr, bool bf16, uint32_t rows, uint32_t heads, uint32_t box_rows)
{
    auto enc = encode_sp();
    if (!enc)
        return false;
    cuuint64_t dims[3] = {SD, rows, heads};
    cuuint64_t strides[2] = {uint64_t(SD) * 2, uint64_t(rows) * SD * 2};
    cuuint32_t box[3] = {64, box_rows, 1};
    cuuint32_t estr[3] = {1, 1, 1};
    return enc(map, bf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3,
               const_cast<void*>(ptr), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
               CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
               CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

} // namespace

cudaError_t launch_attn_tc_sparse(const AttnParams& a, int dtype, bool sel_i32, const void* v16, const float* vinv,
                                  int* err, cudaStream_t st)
{
    if (a.n_q == 0 || a.heads == 0)
        return cudaSuccess;
    SpParams p;
    const bool bf = dtype == kBF16;
    if (!map_rows(&p.tq, a.q, bf, a.q_pad, a.heads, 128) || !map_rows(&p.tk, a.k, bf, a.k_pad, a.kv_heads, 64) ||
        !map_rows(&p.tv, bf ? v16 : a.v, false, a.k_pad, a.kv_heads, 64))
        return cudaErrorInvalidValue;
    p.o = a.o;
    p.err = err;
    p.vinv = bf ? vinv : nullptr;
    p.sel = a.sel;
    p.nsel = a.nsel;
    p.valid = a.valid;
    p.map = a.map;
    p.sel_i32 = sel_i32 ? 1u : 0u;
    p.qk_fmt = bf ? 1u : 0u;
    p.n_q = a.n_q;
    p.q_pad = a.q_pad;
    p.n_k = a.n_k;
    p.k_pad = a.k_pad;
    p.heads = a.heads;
    p.kv_heads = a.kv_heads;
    p.width = a.width;
    p.n_cubes = a.n_cubes;
    p.max_sel = a.max_sel;
    p.dense0 = a.dense0;
    p.dense1 = a.dense1;
    p.tiles_cube = (a.n_cubes + 1) / 2;
    const uint32_t rest = a.n_q > a.n_cubes * 64 ? a.n_q - a.n_cubes * 64 : 0;
    p.tiles_total = p.tiles_cube + (rest + 127) / 128;
    p.scale_log2 = a.scale * kLog2e;
    cudaError_t e = cudaFuncSetAttribute(attn_tc_sparse_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, S_TOTAL);
    if (e != cudaSuccess)
        return e;
    const uint32_t pairs = (p.tiles_total + 1) / 2;
    if (pairs == 0)
        return cudaSuccess;
    attn_tc_sparse_kernel<<<dim3(pairs, a.heads), SNT, S_TOTAL, st>>>(p);
    return cudaGetLastError();
}

} // namespace mako
