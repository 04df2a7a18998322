// Flash attention on mma.sync (m16n8k16) tensor cores for every head width the reference supports (64, 128, 256):
// the dense form (TransformerRuntime::attention, src/models/runtime.cpp:262-273; kernels flash_attn_coop /
// flash_attn_sg, src/kernels/ops.metal:106-369) and the block-sparse form (attention_sparse, runtime.cpp:305-317;
// flash_attn_sparse_128, ops.metal:1039-1185).
//
// A CTA takes 64 query rows of one head (the reference's tile, kAttnRows), four warps of 16 rows each, and streams
// 64-key blocks of K and V through a double-buffered, XOR-swizzled shared-memory tile filled by cp.async.  Scores
// stay in registers; the running softmax is in base 2 with the reference's lazy rescale: a row's reference maximum
// moves only when a score passes it by 8, so exp2 stays within 256 (ops.metal:303-316).  P goes to the P.V product
// as fp16 for fp16 inputs; for bf16 inputs P is split into bf16 hi + lo parts (two products) so the rounding of P
// costs ~2^-16 instead of bf16's 2^-8.  The output is fp32 [rows][width] at column h * dim, zero for rows that see
// no key (ops.metal:355).
#include "common.cuh"
#include "kernels.h"

#include <type_traits>

namespace mako {
namespace {

constexpr int BM = 64, BN = 64, NT = 128;

template <int D, typename T, bool SPARSE, typename S>
__global__ void __launch_bounds__(NT) attn_mma_kernel(const AttnParams p)
{
    constexpr int ROWB = D * 2, CH = D / 8, KS = D / 16;
    constexpr bool QREG = D <= 128;  // Q fragments held in registers (D 256 re-reads them from shared memory)
    constexpr bool SPLIT = sizeof(T) == 2 && !std::is_same<T, __half>::value;
    extern __shared__ __align__(128) uint8_t smem[];
    const uint32_t sQ = smem_u32(smem), sK = sQ + BM * ROWB, sV = sK + 2 * BN * ROWB;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, g = lane >> 2, tq = lane & 3, mi = lane >> 3;
    const uint32_t tile = blockIdx.x, h = blockIdx.y, q0 = tile * BM;
    if (q0 >= p.n_q)
        return;
    const uint32_t kvh = h / (p.heads / p.kv_heads);
    const T* qg = static_cast<const T*>(p.q) + (uint64_t(h) * p.q_pad + q0) * D;
    const T* kg = static_cast<const T*>(p.k) + uint64_t(kvh) * p.k_pad * D;
    const T* vg = static_cast<const T*>(p.v) + uint64_t(kvh) * p.k_pad * D;

    // The pass list: dense -- 64-key blocks up to the tile's last visible key (ops.metal:269-270); sparse -- a cube
    // tile's selected cubes then its dense rows [dense0, dense1), a later tile every key below n_k (ops.metal:1079-1098).
    uint32_t nb, ns = 0;
    bool cube = false;
    const S* my_sel = nullptr;
    if (SPARSE) {
        cube = tile < p.n_cubes;
        if (cube) {
            const int64_t cnt = int64_t(static_cast<const S*>(p.nsel)[uint64_t(h) * p.n_cubes + tile]);
            ns = cnt <= 0 ? 0u : (cnt < int64_t(p.max_sel) ? uint32_t(cnt) : p.max_sel);
            my_sel = static_cast<const S*>(p.sel) + (uint64_t(h) * p.n_cubes + tile) * p.max_sel;
            nb = ns + (p.dense1 > p.dense0 ? (p.dense1 - p.dense0 + BN - 1) / BN : 0);
        } else {
            nb = (p.n_k + BN - 1) / BN;
        }
    } else {
        const uint32_t last = p.q_pos0 + min(q0 + BM, p.n_q) - 1;
        const uint32_t n_keys = last >= p.block ? p.n_k : min(p.n_k, last + 1);
        nb = (n_keys + BN - 1) / BN;
    }
    auto block_range = [&](uint32_t b, uint32_t& j0, uint32_t& hi) {
        if (!SPARSE) {
            j0 = b * BN;
            hi = p.n_k;
        } else if (cube && b < ns) {
            const uint32_t c = uint32_t(my_sel[b]);
            j0 = c < p.n_cubes ? c * BN : 0;
            hi = c < p.n_cubes ? j0 + BN : 0;  // an out-of-range entry is skipped (nothing visible)
        } else if (cube) {
            j0 = p.dense0 + (b - ns) * BN;
            hi = min(j0 + BN, p.dense1);
        } else {
            j0 = b * BN;
            hi = min(j0 + BN, p.n_k);
        }
    };
    auto load_kv = [&](uint32_t b, int stage) {
        uint32_t j0, hi;
        block_range(b, j0, hi);
        const uint32_t dk = sK + stage * BN * ROWB, dv = sV + stage * BN * ROWB;
        for (int i = tid; i < BN * CH; i += NT) {
            const uint32_t r = i / CH, c = i % CH, row = j0 + r;
            const bool ok = row < p.k_pad;
            const uint64_t off = ok ? uint64_t(row) * D + c * 8 : 0;
            cp_async16(dk + swz(r, c, ROWB), kg + off, ok);
            cp_async16(dv + swz(r, c, ROWB), vg + off, ok);
        }
    };
    for (int i = tid; i < BM * CH; i += NT)
        cp_async16(sQ + swz(i / CH, i % CH, ROWB), qg + uint64_t(i / CH) * D + (i % CH) * 8, true);
    cp_async_commit();
    if (nb > 0)
        load_kv(0, 0);
    cp_async_commit();

    const uint32_t wr0 = warp * 16;
    uint32_t qa[QREG ? KS : 1][4];
    float acc[D / 8][4];
#pragma unroll
    for (int i = 0; i < D / 8; ++i)
        acc[i][0] = acc[i][1] = acc[i][2] = acc[i][3] = 0.0f;
    float m[2] = {-INFINITY, -INFINITY}, l[2] = {0.0f, 0.0f};
    const float scale = p.scale * kLog2e;
    const uint32_t P0 = p.q_pos0 + q0;                    // the tile's first position
    const uint32_t pos_g = P0 + wr0 + g;                  // this lane's rows: pos_g, pos_g + 8

    for (uint32_t b = 0; b < nb; ++b) {
        const int st = b & 1;
        if (b + 1 < nb)
            load_kv(b + 1, st ^ 1);
        cp_async_commit();
        cp_async_wait<1>();
        __syncthreads();
        if (QREG && b == 0) {
#pragma unroll
            for (int ks = 0; ks < KS; ++ks)
                ldsm_x4(qa[QREG ? ks : 0], sQ + swz(wr0 + (mi & 1) * 8 + (lane & 7), ks * 2 + (mi >> 1), ROWB));
        }
        uint32_t j0, hi;
        block_range(b, j0, hi);
        const uint32_t kst = sK + st * BN * ROWB, vst = sV + st * BN * ROWB;

        // S = Q K^T for this warp's 16 rows x 64 keys.
        float s[8][4];
#pragma unroll
        for (int i = 0; i < 8; ++i)
            s[i][0] = s[i][1] = s[i][2] = s[i][3] = 0.0f;
#pragma unroll
        for (int ks = 0; ks < KS; ++ks) {
            uint32_t a[4];
            if (QREG) {
#pragma unroll
                for (int i = 0; i < 4; ++i)
                    a[i] = qa[QREG ? ks : 0][i];
            } else {
                ldsm_x4(a, sQ + swz(wr0 + (mi & 1) * 8 + (lane & 7), ks * 2 + (mi >> 1), ROWB));
            }
#pragma unroll
            for (int np = 0; np < 4; ++np) {
                uint32_t kb[4];
                ldsm_x4(kb, kst + swz(np * 16 + (mi >> 1) * 8 + (lane & 7), ks * 2 + (mi & 1), ROWB));
                mma16816(s[2 * np], a, kb[0], kb[1], T());
                mma16816(s[2 * np + 1], a, kb[2], kb[3], T());
            }
        }

        // Scale, mask, running maximum (lazy, +8) and the exponentials.
        bool plain;
        if (!SPARSE)  // rows at or past `block` see every key below n_k; earlier rows the keys up to their position
            plain = j0 + BN <= p.n_k && (P0 >= p.block || j0 + BN - 1 <= P0);
        else
            plain = hi >= j0 + BN && p.valid == nullptr;
        float mx[2] = {-INFINITY, -INFINITY};
#pragma unroll
        for (int nt = 0; nt < 8; ++nt)
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                float x = s[nt][e] * scale;
                if (!plain) {
                    const uint32_t j = j0 + nt * 8 + 2 * tq + (e & 1);
                    bool vis;
                    if (!SPARSE) {
                        const uint32_t pos = pos_g + 8 * (e >> 1);
                        vis = j < p.n_k && (j <= pos || (pos >= p.block && j >= p.block));
                    } else {
                        vis = j < hi && (p.valid == nullptr || p.valid[j] != 0);
                    }
                    if (!vis)
                        x = -INFINITY;
                }
                s[nt][e] = x;
                mx[e >> 1] = fmaxf(mx[e >> 1], x);
            }
#pragma unroll
        for (int r = 0; r < 2; ++r) {
            mx[r] = fmaxf(mx[r], __shfl_xor_sync(0xffffffffu, mx[r], 1));
            mx[r] = fmaxf(mx[r], __shfl_xor_sync(0xffffffffu, mx[r], 2));
        }
        float f[2] = {1.0f, 1.0f};
        bool rescale = false;
#pragma unroll
        for (int r = 0; r < 2; ++r)
            if (mx[r] > m[r] + 8.0f) {
                f[r] = m[r] == -INFINITY ? 0.0f : ex2(m[r] - mx[r]);
                m[r] = mx[r];
                l[r] *= f[r];
                rescale = true;
            }
        if (rescale) {
#pragma unroll
            for (int i = 0; i < D / 8; ++i) {
                acc[i][0] *= f[0];
                acc[i][1] *= f[0];
                acc[i][2] *= f[1];
                acc[i][3] *= f[1];
            }
        }
#pragma unroll
        for (int nt = 0; nt < 8; ++nt)
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                const float mm = m[e >> 1];
                const float pe = mm == -INFINITY ? 0.0f : ex2(s[nt][e] - mm);
                s[nt][e] = pe;
                l[e >> 1] += pe;
            }

        // O += P V, 16 keys a step.
#pragma unroll
        for (int kk = 0; kk < 4; ++kk) {
            uint32_t pa[4], pl[4];
            if (!SPLIT) {
                pa[0] = Elem<__half>::pack(s[2 * kk][0], s[2 * kk][1]);
                pa[1] = Elem<__half>::pack(s[2 * kk][2], s[2 * kk][3]);
                pa[2] = Elem<__half>::pack(s[2 * kk + 1][0], s[2 * kk + 1][1]);
                pa[3] = Elem<__half>::pack(s[2 * kk + 1][2], s[2 * kk + 1][3]);
            } else {
                const float* src[4] = {&s[2 * kk][0], &s[2 * kk][2], &s[2 * kk + 1][0], &s[2 * kk + 1][2]};
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    const __nv_bfloat16 h0 = __float2bfloat16_rn(src[i][0]), h1 = __float2bfloat16_rn(src[i][1]);
                    pa[i] = Elem<__nv_bfloat16>::pack(__bfloat162float(h0), __bfloat162float(h1));
                    pl[i] = Elem<__nv_bfloat16>::pack(src[i][0] - __bfloat162float(h0),
                                                      src[i][1] - __bfloat162float(h1));
                }
            }
#pragma unroll
            for (int dp = 0; dp < D / 16; ++dp) {
                uint32_t vb[4];
                ldsm_x4_t(vb, vst + swz(kk * 16 + (mi & 1) * 8 + (lane & 7), dp * 2 + (mi >> 1), ROWB));
                mma16816(acc[2 * dp], pa, vb[0], vb[1], T());
                mma16816(acc[2 * dp + 1], pa, vb[2], vb[3], T());
                if (SPLIT) {
                    mma16816(acc[2 * dp], pl, vb[0], vb[1], T());
                    mma16816(acc[2 * dp + 1], pl, vb[2], vb[3], T());
                }
            }
        }
        __syncthreads();  // this stage is refilled by the next iteration's load
    }
    cp_async_wait<0>();

    // Normalise and store the rows below n_q (dense) or through the map (sparse).
#pragma unroll
    for (int r = 0; r < 2; ++r) {
        l[r] += __shfl_xor_sync(0xffffffffu, l[r], 1);
        l[r] += __shfl_xor_sync(0xffffffffu, l[r], 2);
    }
    const float inv[2] = {l[0] > 0.0f ? 1.0f / l[0] : 0.0f, l[1] > 0.0f ? 1.0f / l[1] : 0.0f};
#pragma unroll
    for (int r = 0; r < 2; ++r) {
        const uint32_t row = q0 + wr0 + g + 8 * r;
        if (row >= p.n_q)
            continue;
        int64_t dst = row;
        if (SPARSE && p.map != nullptr)
            dst = p.map[row];
        if (dst < 0)
            continue;
        const uint64_t orow = uint64_t(dst) * p.width + uint64_t(h) * D + 2 * tq;
#pragma unroll
        for (int nt = 0; nt < D / 8; ++nt)
            out_store2(p.o, orow + nt * 8, acc[nt][2 * r] * inv[r], acc[nt][2 * r + 1] * inv[r], p.o_type);
    }
}

template <int D, typename T, bool SPARSE, typename S>
cudaError_t launch_one(const AttnParams& p, cudaStream_t st)
{
    constexpr int smem = (BM + 4 * BN) * D * 2;
    auto kern = attn_mma_kernel<D, T, SPARSE, S>;
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e != cudaSuccess)
        return e;
    dim3 grid(p.q_pad / BM, p.heads);
    kern<<<grid, NT, smem, st>>>(p);
    return cudaGetLastError();
}

template <typename T, bool SPARSE, typename S>
cudaError_t by_dim(const AttnParams& p, int dim, cudaStream_t st)
{
    switch (dim) {
    case 64:
        return launch_one<64, T, SPARSE, S>(p, st);
    case 128:
        return launch_one<128, T, SPARSE, S>(p, st);
    case 256:
        return launch_one<256, T, SPARSE, S>(p, st);
    default:
        return cudaErrorInvalidValue;
    }
}

} // namespace

cudaError_t launch_attn_mma(const AttnParams& p, int dtype, int dim, bool sparse, bool sel_i32, cudaStream_t st)
{
    if (p.n_q == 0 || p.heads == 0)
        return cudaSuccess;
    if (!sparse)
        return dtype == kBF16 ? by_dim<__nv_bfloat16, false, uint16_t>(p, dim, st)
                              : by_dim<__half, false, uint16_t>(p, dim, st);
    if (dim != 128)
        return cudaErrorInvalidValue;
    if (sel_i32)
        return dtype == kBF16 ? launch_one<128, __nv_bfloat16, true, int32_t>(p, st)
                              : launch_one<128, __half, true, int32_t>(p, st);
    return dtype == kBF16 ? launch_one<128, __nv_bfloat16, true, uint16_t>(p, st)
                          : launch_one<128, __half, true, uint16_t>(p, st);
}

} // namespace mako
