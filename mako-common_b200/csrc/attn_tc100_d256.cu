// Flash attention for 256-wide heads on sm_100a tensor cores: the dense masked form of TransformerRuntime::attention
// (src/models/runtime.cpp:262-273) for the 256-wide heads of Qwen3.5's gated attention layers
// (src/models/qwen_text.cpp:397-422, flash_attn_sg<256, ...> in the reference, src/kernels/ops.metal:106-214).
//
// A 128-row Q tile of 256-wide heads is 64 KB of shared memory, so a CTA holds one tile and walks the keys in 64-row
// tiles (K and V 32 KB each, two-stage rings): 192 KB in all.  A persistent grid (one CTA per SM) takes the (tile,
// head) items longest first, so one item's epilogue overlaps the next item's Q load and first products.  Q.K^T is M 128 x N 64 x K 256 (16 instructions of
// K 16 at N 64, about two thirds of the full rate), P.V is M 128 x N 256 x K 64 (4 instructions, full rate).
//
// Warp roles (384 threads): warp 0 loads Q once and the K ring, warp 2 the V ring (TMA, 128-byte swizzle, boxes of
// 64 values), warp 1's elected thread issues UMMA in the fixed order QK(0), QK(1), then per key tile PV(j),
// QK(j + 2), with a commit after each group for its consumer and, after P.V, one releasing the V stage (a softmax
// thread releases the K stage when it sees S(j), which Q.K^T(j) finished reading).  Warps 4-11
// run the softmax: query row r (TMEM lane r) belongs to one thread of warps 4-7 (scores 0-31 of a key tile) and one
// of warps 8-11 (scores 32-63), which agree on the row maximum through shared memory.
// TMEM: S in two buffers (0-63, 64-127), P in two buffers (128-159, 160-191, fp16 pairs, the A operand of P.V) and O
// (256-511).  QK(j + 2) waits only until the softmax has read S(j); the softmax writes P(j) into the other buffer
// from P.V(j - 1), so it never waits for a product except to rescale O (rare, the reference's lazy rescale).
//
// Precision as the 128-wide kernel (attn_tc100.cu): Q.K^T in the input type, P.V in fp16 (bf16 V through the scaled
// fp16 copy), fp32 accumulation; every wait is bounded and a timeout sets p.err.
#include "common.cuh"
#include "kernels.h"
#include "tc100.cuh"

#include <cudaTypedefs.h>

namespace mako {
namespace {

using namespace tc;

constexpr int WD = 256, WBM = 128, WBN = 64, WNT = 384;
constexpr uint32_t QBOX = 128 * 64 * 2;              // Q: 128 rows x 64 values
constexpr uint32_t KBOX = 64 * 64 * 2;               // K / V: 64 rows x 64 values
constexpr uint32_t QTILE = 4 * QBOX, KTILE = 4 * KBOX;  // 64 KB, 32 KB
constexpr uint32_t W_Q = 0, W_K = QTILE, W_V = W_K + 2 * KTILE, W_BAR = W_V + 2 * KTILE;
constexpr uint32_t W_XMAX = W_BAR + 256;   // float [2 key tiles][2 column halves][128 rows]
constexpr uint32_t W_LSUM = W_XMAX + 2048;  // float [2 column halves][128 rows]
constexpr uint32_t W_TOTAL = W_LSUM + 1024 + 1024;
constexpr uint32_t COL_S = 0, COL_P = 128, COL_O = 256;
constexpr long long W_WAIT_LIMIT = 1ll << 31;

struct __align__(64) WParams {
    CUtensorMap tq, tk, tv;
    float* o;
    int* err;
    const float* vinv;
    uint32_t qk_fmt, o_type;
    uint32_t n_q, q_pad, n_k, k_pad, heads, kv_heads, q_pos0, block, width, n_tiles;
    float scale_log2;
};

__device__ __forceinline__ uint32_t pack_h2(float lo, float hi)
{
    __half2 v = __floats2half2_rn(lo, hi);
    return *reinterpret_cast<uint32_t*>(&v);
}

// Work items: (128-row tile, head), the tile with the most causal keys first, heads fastest (the K / V of every head
// of this shape fit in L2).  A persistent CTA takes one item per round of gridDim.x items, snaking (CTA c takes
// position c in even rounds and G - 1 - c in odd ones), so that every CTA gets a similar total; while the softmax
// warps store one item's output, the producers load the next item's Q and keys and the issuer starts its Q.K^T.
struct WItem {
    uint32_t h, q0, kvh, nb;
    bool live;  // false: past the last item, or a tile whose rows all lie past n_q
};
__device__ __forceinline__ WItem w_item(const WParams& p, uint32_t round)
{
    const uint32_t G = gridDim.x, c = (round & 1) ? G - 1 - blockIdx.x : blockIdx.x, i = round * G + c;
    WItem it{};
    if (i >= p.n_tiles * p.heads)
        return it;
    const uint32_t tile = p.n_tiles - 1 - i / p.heads;
    it.h = i % p.heads;
    it.q0 = tile * WBM;
    it.kvh = it.h / (p.heads / p.kv_heads);
    it.live = it.q0 < p.n_q;
    const uint32_t last = p.q_pos0 + min(it.q0 + WBM, p.n_q) - 1;
    const uint32_t n_keys = last >= p.block ? p.n_k : min(p.n_k, last + 1);
    it.nb = it.live ? (n_keys + WBN - 1) / WBN : 0;
    return it;
}
__device__ __forceinline__ uint32_t w_rounds(const WParams& p)
{
    return (p.n_tiles * p.heads + gridDim.x - 1) / gridDim.x;
}

__global__ void __launch_bounds__(WNT, 1) attn_tc256_kernel(const __grid_constant__ WParams p)
{
    extern __shared__ uint8_t smem_raw[];
    const uint32_t raw = smem_u32(smem_raw);
    const uint32_t base = (raw + 1023u) & ~1023u;
    uint8_t* const gbase = smem_raw + (base - raw);
    const uint32_t sQ = base + W_Q, sK = base + W_K, sV = base + W_V, sB = base + W_BAR;
    const uint32_t q_full = sB;
    auto k_full = [&](uint32_t s) { return sB + 8 + 8 * s; };
    auto k_empty = [&](uint32_t s) { return sB + 24 + 8 * s; };
    auto v_full = [&](uint32_t s) { return sB + 40 + 8 * s; };
    auto v_empty = [&](uint32_t s) { return sB + 56 + 8 * s; };
    auto s_full = [&](uint32_t b) { return sB + 72 + 8 * b; };
    auto s_free = [&](uint32_t b) { return sB + 88 + 8 * b; };
    auto p_full = [&](uint32_t b) { return sB + 104 + 8 * b; };
    const uint32_t pv_done = sB + 120, mma_done = sB + 128, tmem_slot = sB + 136;
    const uint32_t q_empty = sB + 144;  // an item's last Q.K^T has finished: Q may be overwritten
    volatile uint32_t* tmem_slot_ptr = reinterpret_cast<volatile uint32_t*>(smem_raw + (tmem_slot - raw));

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t rounds = w_rounds(p);

    if (threadIdx.x == 0) {
        mbar_init(q_full, 1);
        mbar_init(q_empty, 1);
        for (uint32_t s = 0; s < 2; ++s) {
            mbar_init(k_full(s), 1);
            mbar_init(k_empty(s), 1);
            mbar_init(v_full(s), 1);
            mbar_init(v_empty(s), 1);
            mbar_init(s_full(s), 1);
            mbar_init(s_free(s), 256);
            mbar_init(p_full(s), 256);
        }
        mbar_init(pv_done, 1);
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

    // Counters every role keeps alike: g counts the key tiles of the items so far (ring stages, S / P buffers and the
    // phases of their barriers; pv_done completes once per key tile), nq the live items (q_full / q_empty phases).
    if ((warp == 0 || warp == 2) && lane == 0) {
        // ---------------- TMA producers: warp 0 Q and the K ring, warp 2 the V ring ----------------
        const bool is_k = warp == 0;
        const CUtensorMap* map = is_k ? &p.tk : &p.tv;
        tma_prefetch_desc(map);
        if (is_k)
            tma_prefetch_desc(&p.tq);
        bool ok = true;
        uint32_t g = 0, nq = 0, issued = 0;
        for (uint32_t round = 0; ok && round < rounds; ++round) {
            const WItem it = w_item(p, round);
            if (!it.live)
                continue;
            if (is_k) {  // the item's Q, once its predecessor's last Q.K^T has read the buffer
                if (nq > 0 && !mbar_wait(q_empty, (nq - 1) & 1, W_WAIT_LIMIT)) {
                    ok = false;
                    break;
                }
                mbar_expect_tx(q_full, QTILE);
                for (int dh = 0; dh < 4; ++dh)
                    tma_load_3d(sQ + dh * QBOX, &p.tq, q_full, dh * 64, int(it.q0), int(it.h));
            }
            ++nq;
            for (uint32_t j = 0; j < it.nb; ++j) {
                const uint32_t gj = g + j, s = gj & 1;
                if (gj >= 2 && !mbar_wait(is_k ? k_empty(s) : v_empty(s), ((gj >> 1) & 1) ^ 1, W_WAIT_LIMIT)) {
                    ok = false;
                    break;
                }
                const uint32_t full = is_k ? k_full(s) : v_full(s), ring = is_k ? sK : sV;
                mbar_expect_tx(full, KTILE);
                for (int dh = 0; dh < 4; ++dh)
                    tma_load_3d(ring + s * KTILE + dh * KBOX, map, full, dh * 64, int(j * WBN), int(it.kvh));
                ++issued;
            }
            g += it.nb;
        }
        if (!ok)
            atomicExch(p.err, 31);
        // our copies in flight land before the CTA leaves (already so on the normal path)
        if (is_k && nq > 0)
            mbar_wait(q_full, (nq - 1) & 1, W_WAIT_LIMIT);
        for (uint32_t i = issued > 2 ? issued - 2 : 0; i < issued; ++i)
            mbar_wait(is_k ? k_full(i & 1) : v_full(i & 1), (i >> 1) & 1, W_WAIT_LIMIT);
    } else if (warp == 1) {
        // ---------------- UMMA issuer ----------------
        if (lane == 0) {
            const uint32_t idesc_qk = idesc_f16(p.qk_fmt, p.qk_fmt, 0, 0, WBM, WBN);
            const uint32_t idesc_pv = idesc_f16(0, 0, 0, 1, WBM, WD);
            auto qk = [&](uint32_t gj) {
                const uint32_t s = gj & 1;
                bool w = mbar_wait(k_full(s), (gj >> 1) & 1, W_WAIT_LIMIT);
                if (w && gj >= 2)  // S(gj - 2) read by the softmax
                    w = mbar_wait(s_free(s), ((gj - 2) >> 1) & 1, W_WAIT_LIMIT);
                if (!w)
                    return false;
                fence_after();
#pragma unroll
                for (uint32_t ks = 0; ks < WD / 16; ++ks)
                    umma_ss(tmem + COL_S + s * 64, sdesc(sQ + (ks >> 2) * QBOX + (ks & 3) * 32, 16, 1024),
                            sdesc(sK + s * KTILE + (ks >> 2) * KBOX + (ks & 3) * 32, 16, 1024), idesc_qk, ks > 0);
                umma_commit(s_full(s));
                return true;
            };
            bool ok = true;
            uint32_t g = 0, nq = 0;
            for (uint32_t round = 0; ok && round < rounds; ++round) {
                const WItem it = w_item(p, round);
                if (!it.live)
                    continue;
                ok = mbar_wait(q_full, nq & 1, W_WAIT_LIMIT);
                ++nq;
                if (!ok)
                    break;
                if (it.nb == 0) {
                    umma_commit(q_empty);
                    continue;
                }
                ok = qk(g) && (it.nb < 2 || qk(g + 1));
                if (ok && it.nb <= 2)
                    umma_commit(q_empty);
                for (uint32_t j = 0; ok && j < it.nb; ++j) {
                    const uint32_t gj = g + j, s = gj & 1;
                    ok = mbar_wait(p_full(s), (gj >> 1) & 1, W_WAIT_LIMIT) &&
                         mbar_wait(v_full(s), (gj >> 1) & 1, W_WAIT_LIMIT);
                    if (!ok)
                        break;
                    fence_after();
#pragma unroll
                    for (uint32_t kk = 0; kk < WBN / 16; ++kk)
                        umma_ts(tmem + COL_O, tmem + COL_P + s * 32 + kk * 8,
                                sdesc(sV + s * KTILE + kk * 2048, KBOX, 1024), idesc_pv, j > 0 || kk > 0);
                    umma_commit(pv_done);
                    umma_commit(v_empty(s));
                    if (j + 2 < it.nb) {
                        ok = qk(gj + 2);
                        if (ok && j + 3 == it.nb)
                            umma_commit(q_empty);
                    }
                }
                g += it.nb;
            }
            if (!ok)
                atomicExch(p.err, 32);
            umma_commit(mma_done);  // every MMA issued above has finished before TMEM is freed
            mbar_wait(mma_done, 0, W_WAIT_LIMIT);
        }
    } else if (warp >= 4) {
        // ---------------- softmax and epilogue: row `row`, key columns 32c .. 32c + 31 of each tile ----------------
        const uint32_t c = (warp - 4) >> 2, qd = warp & 3, row = qd * 32 + lane;
        const uint32_t tl = tmem + ((qd * 32) << 16);
        float* const xmax = reinterpret_cast<float*>(gbase + W_XMAX);
        float* const lsum = reinterpret_cast<float*>(gbase + W_LSUM);
        const float scale = p.scale_log2;
        const uint64_t scale2 = pack2(scale, scale);
        bool ok = true;
        uint32_t g = 0;
        // Every softmax thread walks all of its CTA's items, also after a failed wait (then without waiting or
        // computing), so that the two threads of a row keep meeting at the named barriers, which cannot time out.
        for (uint32_t round = 0; round < rounds; ++round) {
            const WItem it = w_item(p, round);
            if (!it.live)
                continue;
            const uint32_t h = it.h, q0 = it.q0, nb = it.nb;
            const float vscale = p.vinv ? p.vinv[it.kvh] : 1.0f;  // read now, used by the epilogue
            const uint32_t pos = p.q_pos0 + q0 + row;
            const uint32_t lim = pos >= p.block ? p.n_k : min(p.n_k, pos + 1);  // this row sees keys [0, lim)
            const uint32_t pos1 = p.q_pos0 + q0;
            const uint32_t lim1 = pos1 >= p.block ? p.n_k : min(p.n_k, pos1 + 1);  // the tile's first row
            float m = -INFINITY, l = 0.0f;
            for (uint32_t j = 0; j < nb; ++j) {
                const uint32_t gj = g + j, b = gj & 1;
                uint32_t r[32];
                float pmax = -INFINITY;
                if (ok)
                    ok = __all_sync(0xffffffffu, mbar_wait(s_full(b), (gj >> 1) & 1, W_WAIT_LIMIT));
                if (ok) {
                    fence_after();
                    tmem_ld32(tl + COL_S + b * 64 + 32 * c, r);
                    tmem_wait_ld();
                    reg_fence(r);
                    fence_before();
                    mbar_arrive(s_free(b));  // QK(j + 2) may overwrite S(j) now
                    if (threadIdx.x == 128)
                        mbar_arrive(k_empty(b));  // QK(j) has finished reading K(j)
                    const uint32_t j0 = j * WBN + 32 * c;
                    if (j * WBN + WBN > lim1) {  // a tile the mask cuts: keys at or past this row's limit drop out
#pragma unroll
                        for (int e = 0; e < 32; ++e)
                            if (j0 + e >= lim)
                                r[e] = 0xFF800000u;  // -inf
                    }
                    float mq[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
#pragma unroll
                    for (int e = 0; e < 32; e += 8)
#pragma unroll
                        for (int t = 0; t < 4; ++t)
                            mq[t] = max3f(mq[t], __uint_as_float(r[e + 2 * t]), __uint_as_float(r[e + 2 * t + 1]));
                    pmax = fmaxf(fmaxf(mq[0], mq[1]), fmaxf(mq[2], mq[3]));
                }
                // the row maximum over both column halves (partner: the same row in the other warpgroup)
                xmax[(b * 2 + c) * 128 + row] = pmax;
                named_bar(1 + qd, 64);
                if (!ok)
                    continue;
                const float mx = fmaxf(pmax, xmax[(b * 2 + (c ^ 1)) * 128 + row]) * scale;
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
                uint32_t pk[16];
                uint64_t sum2[2] = {pack2(0.0f, 0.0f), pack2(0.0f, 0.0f)};
#pragma unroll
                for (int e = 0; e < 16; ++e) {
                    float a, bb;
                    unpack2(ffma2(pack2(__uint_as_float(r[2 * e]), __uint_as_float(r[2 * e + 1])), scale2, mneg2), a,
                            bb);
                    a = ex2(a);
                    bb = ex2(bb);
                    sum2[e & 1] = fadd2(sum2[e & 1], pack2(a, bb));
                    pk[e] = pack_h2(a, bb);
                }
                {
                    float s0, s1, s2, s3;
                    unpack2(sum2[0], s0, s1);
                    unpack2(sum2[1], s2, s3);
                    l += (s0 + s1) + (s2 + s3);
                }
                // A rescale of O waits for P.V(j - 1), which adds to it (P.V(j) waits for this thread's P(j);
                // P.V(j - 2) finished before QK(j), committed after it).
                if (j > 0 && __any_sync(0xffffffffu, resc)) {
                    ok = __all_sync(0xffffffffu, mbar_wait(pv_done, (gj - 1) & 1, W_WAIT_LIMIT));
                    if (ok) {
                        fence_after();
                        const float gsc = resc ? f : 1.0f;
#pragma unroll
                        for (int k = 0; k < 4; ++k) {
                            uint32_t o[32];
                            tmem_ld32(tl + COL_O + 128 * c + 32 * k, o);
                            tmem_wait_ld();
                            reg_fence(o);
#pragma unroll
                            for (int e = 0; e < 32; ++e)
                                o[e] = __float_as_uint(__uint_as_float(o[e]) * gsc);
                            tmem_st32(tl + COL_O + 128 * c + 32 * k, o);
                        }
                    }
                }
                tmem_st16(tl + COL_P + b * 32 + 16 * c, pk);
                tmem_wait_st();
                fence_before();
                mbar_arrive(p_full(b));
            }
            // O is final once the item's last P.V has finished.  pv_done completes once per key tile and a parity
            // wait cannot tell a phase from the one two before it, so the wait goes phase by phase: P.V(nb - 3)
            // finished before S(nb - 1) was seen, P.V(nb - 2) and P.V(nb - 1) are waited for in turn.
            if (ok && nb > 0) {
                bool w = nb < 2 || mbar_wait(pv_done, (g + nb - 2) & 1, W_WAIT_LIMIT);
                w = w && mbar_wait(pv_done, (g + nb - 1) & 1, W_WAIT_LIMIT);
                ok = __all_sync(0xffffffffu, w);
                fence_after();
            }
            g += nb;
            lsum[c * 128 + row] = l;
            named_bar(1 + qd, 64);
            const float lt = lsum[row] + lsum[128 + row];
            const float inv = (lt > 0.0f ? 1.0f / lt : 0.0f) * vscale;
            const uint32_t grow = q0 + row;
            const uint64_t ooff = uint64_t(grow) * p.width + uint64_t(h) * WD + 128 * c;
#pragma unroll
            for (int k = 0; k < 4; ++k) {
                uint32_t o[32];
                if (ok && nb > 0) {
                    tmem_ld32(tl + COL_O + 128 * c + 32 * k, o);
                    tmem_wait_ld();
                    reg_fence(o);
                } else {
#pragma unroll
                    for (int e = 0; e < 32; ++e)
                        o[e] = 0u;
                }
                if (grow < p.n_q)
                    out_store32(p.o, ooff + 32 * k, o, inv, p.o_type);
            }
            // both threads of the row have read O (and the sum shares) before either publishes the next item's P
            fence_before();
            named_bar(1 + qd, 64);
            fence_after();
        }
        if (!ok && lane == 0)
            atomicExch(p.err, 33);
    }
    __syncwarp();
    fence_before();
    __syncthreads();
    if (warp == 1) {
        fence_after();
        tmem_dealloc(tmem, 512);
    }
}

} // namespace

cudaError_t launch_attn_tc256(const AttnParams& a, int dtype, const void* v16, const float* vinv, int* err,
                              cudaStream_t st)
{
    if (a.n_q == 0 || a.heads == 0)
        return cudaSuccess;
    WParams p;
    const bool bf = dtype == kBF16;
    if (!tile_map(&p.tq, a.q, bf, WD, a.q_pad, a.heads, WBM) ||
        !tile_map(&p.tk, a.k, bf, WD, a.k_pad, a.kv_heads, WBN) ||
        !tile_map(&p.tv, bf ? v16 : a.v, false, WD, a.k_pad, a.kv_heads, WBN))
        return cudaErrorInvalidValue;
    p.o = a.o;
    p.err = err;
    p.vinv = bf ? vinv : nullptr;
    p.qk_fmt = bf ? 1u : 0u;
    p.o_type = a.o_type;
    p.n_q = a.n_q;
    p.q_pad = a.q_pad;
    p.n_k = a.n_k;
    p.k_pad = a.k_pad;
    p.heads = a.heads;
    p.kv_heads = a.kv_heads;
    p.q_pos0 = a.q_pos0;
    p.block = a.block;
    p.width = a.width;
    p.n_tiles = (a.q_pad + WBM - 1) / WBM;
    p.scale_log2 = a.scale * kLog2e;
    cudaError_t e = cudaFuncSetAttribute(attn_tc256_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, W_TOTAL);
    if (e != cudaSuccess)
        return e;
    const uint32_t n_items = p.n_tiles * a.heads, sms = a.num_sms ? a.num_sms : 148;
    attn_tc256_kernel<<<n_items < sms ? n_items : sms, WNT, W_TOTAL, st>>>(p);
    return cudaGetLastError();
}

} // namespace mako
