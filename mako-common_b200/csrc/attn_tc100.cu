// Flash attention for 64- and 128-wide heads on sm_100a tensor cores (tcgen05 UMMA, TMEM accumulators, TMA-fed
// shared memory): the dense masked form of TransformerRuntime::attention (src/models/runtime.cpp:262-273; maths of
// flash_attn_coop, src/kernels/ops.metal:230-363).
//
// A CTA owns 256 query rows of one head as two 128-row tiles A and B that share every K / V tile (half the K / V
// reads of one tile per CTA).  Warp roles (384 threads):
//   warp 0        TMA producer: Q once, then 128-key K and V tiles into two-stage rings (128-byte swizzle).
//   warp 1        UMMA issuer (one thread) and TMEM owner: S_X = Q_X K^T (SS, M 128 N 128), O_X += P_X V (TS, P from
//                 TMEM, V MN-major from shared memory).
//   warps 4-7     softmax of tile A, warps 8-11 softmax of tile B: thread r owns query row r = TMEM lane r, so a
//                 row's 128 scores sit in one thread's registers (no shuffles).  Base-2 online softmax with the
//                 reference's lazy rescale (a row's maximum moves only when a score passes it by 8, so P <= 256 fits
//                 fp16; ops.metal:303-316); P goes back into S's TMEM columns as fp16 pairs for the P.V product.
// TMEM (512 columns): S_A 0-127, S_B 128-255, O_A 256-383, O_B 384-511.  The issue order per key tile is
// PV_A(j), QK_A(j+1), PV_B(j), QK_B(j+1) -- while one tile's softmax runs the tensor core works on the other's.
// QK_X(j+1) overwrites the P that PV_X(j) reads and is issued right behind it: the tensor pipe runs one thread's
// MMAs in issue order.
//
// P.V runs in fp16: for fp16 inputs V is used as it is; for bf16 inputs a pre-pass writes V * 2^k per kv head into
// an fp16 copy (k puts the head's largest |v| in [2^14, 2^15), exact for every value above 2^-28 of that maximum) and
// the epilogue multiplies by 2^-k.  P in fp16 costs ~2^-11 relative error where bf16 P would cost 2^-8.
//
// Every mbarrier wait is bounded (clock64); on a timeout the thread records an error code in p.err, waits (bounded)
// for its own copies / MMAs in flight, and the CTA frees its TMEM and returns.
#include "common.cuh"
#include "kernels.h"
#include "tc100.cuh"

#include <cudaTypedefs.h>

namespace mako {
namespace {

using namespace tc;

constexpr int TBM = 128, TBN = 128, TNS = 2, TNT = 384;
constexpr uint32_t BOX_BYTES = 128 * 64 * 2;  // one TMA box: 128 rows x 64 16-bit values
// Shared memory for TD-wide heads (64 or 128): Q of both tiles, the K and V rings, the barriers; in the
// head-sharded form also one output staging box (128 rows x 32 floats, 16 KB) per tile.
template <int TD>
struct TcSmem {
    static constexpr uint32_t TILE = (TD / 64) * BOX_BYTES;  // 128 rows x TD values
    static constexpr uint32_t Q = 0, K = 2 * TILE, V = K + TNS * TILE, BAR = V + TNS * TILE;
    static constexpr uint32_t TOTAL = BAR + 256 + 1024;  // + barriers + alignment slack
};
// the head-sharded form (128-wide heads): staging boxes 1024-byte aligned for the 128-byte swizzle
constexpr uint32_t TC_STG = TcSmem<128>::BAR + 1024, TC_TOTAL_GATHER = TC_STG + 2 * BOX_BYTES + 1024;
static_assert(TC_TOTAL_GATHER <= 227 * 1024, "the head-sharded form's shared memory");
constexpr long long WAIT_LIMIT = 1ll << 31;             // clock cycles (~1 s) before a wait gives up

struct __align__(64) TcParams {
    CUtensorMap tq, tk, tv;
    CUtensorMap to[8];  // head-sharded form: every destination o as [n_q][width] fp32, boxes of 128 rows x 32 floats
    float* od[8];   // output destinations (this rank's o, then the peers' mapped o for the head-sharded form)
    uint32_t n_od;  // destinations in od
    uint32_t head0;  // column of local head h: (head0 + h) * 128
    uint32_t o_type;  // element type of o (single destination): 0 fp32, 1 fp16, 2 bf16
    int* err;
    const float* vinv;  // per kv head: 1 / (the fp16 copy's scale), null for fp16 inputs
    uint32_t qk_fmt;    // Q / K element format: 0 fp16, 1 bf16
    uint32_t n_q, q_pad, n_k, k_pad, heads, kv_heads, q_pos0, block, width, n_tiles;
    uint32_t group_heads;  // heads per group of the work order (a multiple of heads / kv_heads)
    float scale_log2;
};

__device__ __forceinline__ uint32_t pack_half2(float lo, float hi)
{
    __half2 h = __floats2half2_rn(lo, hi);
    return *reinterpret_cast<uint32_t*>(&h);
}

// Work items: the heads in groups of group_heads whose keys and values fit in about half the L2 (all heads when they
// do), group after group; within a group, tile t = n_tiles - 1 down to 0 (rows [256 t, 256 t + 256)), each over the
// group's heads.  Whatever the mask, a later tile sees at least as many keys, so a group's items come longest first,
// while the CTAs in flight read the keys of one group only.  A CTA takes one item per round of gridDim.x items,
// snaking (CTA c takes position c in even rounds and G - 1 - c in odd ones) so that every CTA gets a similar total.
struct TcItem {
    uint32_t h, q0, kvh, nb;
    bool live;  // false: past the last item, or a tile whose rows all lie past n_q
};
__device__ __forceinline__ uint32_t item_index(uint32_t round)
{
    const uint32_t G = gridDim.x, c = (round & 1) ? G - 1 - blockIdx.x : blockIdx.x;
    return round * G + c;
}
__device__ __forceinline__ TcItem tc_item(const TcParams& p, uint32_t i)
{
    TcItem it;
    const uint32_t per_group = p.group_heads * p.n_tiles, grp = i / per_group, k = i % per_group;
    const uint32_t gh = min(p.group_heads, p.heads - grp * p.group_heads);  // heads in this group
    const uint32_t tile = p.n_tiles - 1 - k / gh;
    it.h = grp * p.group_heads + k % gh;
    it.q0 = tile * 2 * TBM;
    it.kvh = it.h / (p.heads / p.kv_heads);
    it.live = it.q0 < p.n_q;
    const uint32_t last = p.q_pos0 + min(it.q0 + 2 * TBM, p.n_q) - 1;
    const uint32_t n_keys = last >= p.block ? p.n_k : min(p.n_k, last + 1);
    it.nb = it.live ? (n_keys + TBN - 1) / TBN : 0;
    return it;
}

// TD: head width (64 or 128).  GATHER: the head-sharded form's epilogue (TMA stores into every rank's o through a
// staging box per tile, 128-wide heads); otherwise plain stores into p.od[0].  Either way a persistent grid: while
// the softmax warps store one item's output, the producer already loads the next item's Q and keys and the issuer
// starts its Q.K^T.
template <int TD, bool GATHER>
__global__ void __launch_bounds__(TNT, 1) attn_tc_kernel(const __grid_constant__ TcParams p)
{
    constexpr uint32_t TILE_BYTES = TcSmem<TD>::TILE;
    extern __shared__ uint8_t smem_raw[];
    const uint32_t raw = smem_u32(smem_raw);
    const uint32_t base = (raw + 1023u) & ~1023u;
    const uint32_t sQ = base + TcSmem<TD>::Q, sK = base + TcSmem<TD>::K, sV = base + TcSmem<TD>::V;
    const uint32_t sB = base + TcSmem<TD>::BAR;
    // barriers
    const uint32_t q_full = sB;
    auto k_full = [&](uint32_t s) { return sB + 8 + 8 * s; };
    auto k_empty = [&](uint32_t s) { return sB + 24 + 8 * s; };
    auto v_full = [&](uint32_t s) { return sB + 40 + 8 * s; };
    auto v_empty = [&](uint32_t s) { return sB + 56 + 8 * s; };
    auto s_full = [&](uint32_t x) { return sB + 72 + 8 * x; };
    auto p_full = [&](uint32_t x) { return sB + 88 + 8 * x; };
    auto pv_done = [&](uint32_t x) { return sB + 104 + 8 * x; };
    const uint32_t mma_done = sB + 120;
    const uint32_t tmem_slot = sB + 128;
    const uint32_t q_empty = sB + 136;  // an item's last Q.K^T has finished: Q may be overwritten
    volatile uint32_t* tmem_slot_ptr = reinterpret_cast<volatile uint32_t*>(smem_raw + (tmem_slot - raw));

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t n_items = p.n_tiles * p.heads;

    if (threadIdx.x == 0) {
        mbar_init(q_full, 1);
        mbar_init(q_empty, 1);
        for (uint32_t s = 0; s < TNS; ++s) {
            mbar_init(k_full(s), 1);
            mbar_init(k_empty(s), 1);
            mbar_init(v_full(s), 1);
            mbar_init(v_empty(s), 1);
        }
        for (uint32_t x = 0; x < 2; ++x) {
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

    // Counters every role keeps alike: g counts the key tiles of the items so far (K / V ring stages, and the phases
    // of s_full / p_full), nq the items with Q loaded, nk the items with at least one key tile (pv_done phases).
    if (warp < 4) {
        // the producer and issuer warpgroup gives registers to the softmax warpgroups (384 x 168 at launch =
        // 128 x 104 + 256 x 200)
        asm volatile("setmaxnreg.dec.sync.aligned.u32 104;\n" ::: "memory");
        if (warp == 0 && lane == 0) {
            // ---------------- TMA producer ----------------
            tma_prefetch_desc(&p.tq);
            tma_prefetch_desc(&p.tk);
            tma_prefetch_desc(&p.tv);
            bool ok = true;
            uint32_t g = 0, nq = 0, issued = 0;  // issued: K / V loads so far (2 per key tile)
            for (uint32_t round = 0; ok; ++round) {
                const uint32_t i = item_index(round);
                if (i >= n_items)
                    break;
                const TcItem it = tc_item(p, i);
                if (!it.live)
                    continue;
                if (nq > 0 && !mbar_wait(q_empty, (nq - 1) & 1, WAIT_LIMIT)) {
                    ok = false;
                    break;
                }
                mbar_expect_tx(q_full, 2 * TILE_BYTES);
                for (int x = 0; x < 2; ++x)
                    for (int half = 0; half < TD / 64; ++half)
                        tma_load_3d(sQ + x * TILE_BYTES + half * BOX_BYTES, &p.tq, q_full, half * 64,
                                    it.q0 + x * TBM, it.h);
                ++nq;
                for (uint32_t j = 0; j < it.nb; ++j) {
                    const uint32_t gj = g + j, s = gj % TNS, ph = (gj / TNS) & 1;
                    if (gj >= TNS && !mbar_wait(k_empty(s), ph ^ 1, WAIT_LIMIT)) {
                        ok = false;
                        break;
                    }
                    mbar_expect_tx(k_full(s), TILE_BYTES);
                    for (int half = 0; half < TD / 64; ++half)
                        tma_load_3d(sK + s * TILE_BYTES + half * BOX_BYTES, &p.tk, k_full(s), half * 64, j * TBN,
                                    it.kvh);
                    ++issued;
                    if (gj >= TNS && !mbar_wait(v_empty(s), ph ^ 1, WAIT_LIMIT)) {
                        ok = false;
                        break;
                    }
                    mbar_expect_tx(v_full(s), TILE_BYTES);
                    for (int half = 0; half < TD / 64; ++half)
                        tma_load_3d(sV + s * TILE_BYTES + half * BOX_BYTES, &p.tv, v_full(s), half * 64, j * TBN,
                                    it.kvh);
                    ++issued;
                }
                g += it.nb;
            }
            if (!ok)
                atomicExch(p.err, 1);
            // Our copies in flight land before the CTA leaves (already so on the normal path).
            if (nq > 0)
                mbar_wait(q_full, (nq - 1) & 1, WAIT_LIMIT);
            for (uint32_t k = issued > 2 * TNS ? issued - 2 * TNS : 0; k < issued; ++k) {
                const uint32_t gj = k / 2, s = gj % TNS, ph = (gj / TNS) & 1;
                mbar_wait((k & 1) ? v_full(s) : k_full(s), ph, WAIT_LIMIT);
            }
        } else if (warp == 1 && lane == 0) {
            // ---------------- UMMA issuer ----------------
            const uint32_t idesc_qk = idesc_f16(p.qk_fmt, p.qk_fmt, 0, 0, TBM, TBN);
            const uint32_t idesc_pv = idesc_f16(0, 0, 0, 1, TBM, TD);
            auto qk = [&](uint32_t x, uint32_t stage) {
#pragma unroll
                for (uint32_t ks = 0; ks < TD / 16; ++ks) {
                    const uint32_t off = (ks >> 2) * BOX_BYTES + (ks & 3) * 32;
                    umma_ss(tmem + x * 128, sdesc(sQ + x * TILE_BYTES + off, 16, 1024),
                            sdesc(sK + stage * TILE_BYTES + off, 16, 1024), idesc_qk, ks > 0);
                }
            };
            auto pv = [&](uint32_t x, uint32_t stage, bool acc) {
#pragma unroll
                for (uint32_t kk = 0; kk < TBN / 16; ++kk)
                    umma_ts(tmem + 256 + x * 128, tmem + x * 128 + kk * 8,
                            sdesc(sV + stage * TILE_BYTES + kk * 2048, BOX_BYTES, 1024), idesc_pv, acc || kk > 0);
            };
            bool ok = true;
            uint32_t g = 0, nq = 0;
            for (uint32_t round = 0; ok; ++round) {
                const uint32_t i = item_index(round);
                if (i >= n_items)
                    break;
                const TcItem it = tc_item(p, i);
                if (!it.live)
                    continue;
                if (!(ok = mbar_wait(q_full, nq & 1, WAIT_LIMIT)))
                    break;
                ++nq;
                if (it.nb == 0) {
                    umma_commit(q_empty);
                    continue;
                }
                if (!(ok = mbar_wait(k_full(g % TNS), (g / TNS) & 1, WAIT_LIMIT)))
                    break;
                fence_after();
                qk(0, g % TNS);
                umma_commit(s_full(0));
                qk(1, g % TNS);
                umma_commit(s_full(1));
                umma_commit(k_empty(g % TNS));
                if (it.nb == 1)
                    umma_commit(q_empty);
                // Fixed order per key tile j: PV_A(j), QK_A(j+1), PV_B(j), QK_B(j+1).  QK_X(j+1) is issued right
                // behind PV_X(j) without waiting for it: the tensor pipe executes one thread's MMAs in issue order, so
                // P_X(j) is read before Q.K^T overwrites its columns.  Each commit tracks every MMA issued before it,
                // so when the softmax sees S_X(j+1) the product PV_X(j) has finished too (its O may be rescaled).
                // An item's first Q.K^T follows the previous item's last P.V the same way.
                for (uint32_t j = 0; j < it.nb && ok; ++j) {
                    const uint32_t gj = g + j, st = gj % TNS, g1 = gj + 1, st1 = g1 % TNS;
                    ok = mbar_wait(v_full(st), (gj / TNS) & 1, WAIT_LIMIT);
#pragma unroll
                    for (uint32_t x = 0; x < 2 && ok; ++x) {
                        if (!(ok = mbar_wait(p_full(x), gj & 1, WAIT_LIMIT)))
                            break;
                        fence_after();
                        pv(x, st, j > 0);
                        if (x == 1)
                            umma_commit(v_empty(st));
                        if (j + 1 < it.nb) {
                            if (x == 0 && !(ok = mbar_wait(k_full(st1), (g1 / TNS) & 1, WAIT_LIMIT)))
                                break;
                            qk(x, st1);
                            umma_commit(s_full(x));
                            if (x == 1) {
                                umma_commit(k_empty(st1));
                                if (j + 2 == it.nb)
                                    umma_commit(q_empty);
                            }
                        } else {
                            umma_commit(pv_done(x));  // the tile's last product: its O is final
                        }
                    }
                }
                g += it.nb;
            }
            if (!ok)
                atomicExch(p.err, 2);
            umma_commit(mma_done);  // every MMA issued above has finished before TMEM is freed
            mbar_wait(mma_done, 0, WAIT_LIMIT);
        }
    } else {
        asm volatile("setmaxnreg.inc.sync.aligned.u32 200;\n" ::: "memory");
        // ---------------- softmax (and epilogue) of tile X ----------------
        const uint32_t x = (warp - 4) >> 2, ql = (warp & 3) * 32, row = ql + lane;
        const uint32_t tl = tmem + (ql << 16);
        const uint32_t colS = x * 128, colO = 256 + x * 128;
        const float scale = p.scale_log2;
        bool ok = true;
        uint32_t g = 0, nk = 0;
        for (uint32_t round = 0; ok; ++round) {
            const uint32_t i = item_index(round);
            if (i >= n_items)
                break;
            const TcItem it = tc_item(p, i);
            if (!it.live)
                continue;
            const uint32_t h = it.h, q0 = it.q0, nb = it.nb;
            const uint32_t pos = p.q_pos0 + q0 + x * TBM + row;
            const uint32_t lim = pos >= p.block ? p.n_k : min(p.n_k, pos + 1);  // this row sees keys [0, lim)
            const uint32_t pos1 = p.q_pos0 + q0 + x * TBM;
            const uint32_t lim1 = pos1 >= p.block ? p.n_k : min(p.n_k, pos1 + 1);  // the tile's first row
            float m = -INFINITY, l = 0.0f;
            for (uint32_t j = 0; j < nb; ++j) {
                ok = __all_sync(0xffffffffu, mbar_wait(s_full(x), (g + j) & 1, WAIT_LIMIT));
                if (!ok)
                    break;
                fence_after();
                uint32_t r[4][32];
                tmem_ld128(tl + colS, r);  // one instruction for the row's 128 scores (0.7% faster than four)
                tmem_wait_ld();
#pragma unroll
                for (int c = 0; c < 4; ++c)
                    reg_fence(r[c]);
                const uint32_t j0 = j * TBN;
                if (j0 + TBN > lim1) {  // a tile the mask cuts: keys at or past this row's limit drop out
#pragma unroll
                    for (int c = 0; c < TBN; ++c)
                        if (j0 + c >= lim)
                            r[c >> 5][c & 31] = 0xFF800000u;  // -inf
                }
                // Row maximum of the raw scores (scale > 0 keeps the order), three at a time, four chains.
                float mq[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
#pragma unroll
                for (int c = 0; c < TBN; c += 8)
#pragma unroll
                    for (int t = 0; t < 4; ++t)
                        mq[t] = max3f(mq[t], __uint_as_float(r[(c + 2 * t) >> 5][(c + 2 * t) & 31]),
                                      __uint_as_float(r[(c + 2 * t + 1) >> 5][(c + 2 * t + 1) & 31]));
                const float mx = fmaxf(fmaxf(mq[0], mq[1]), fmaxf(mq[2], mq[3])) * scale;
                float f = 1.0f;
                bool resc = false;
                if (mx > m + 8.0f) {
                    f = m == -INFINITY ? 0.0f : ex2(m - mx);
                    m = mx;
                    l *= f;
                    resc = true;
                }
                // P = 2^(s * scale - m), two lanes per FMA; a row with no visible key so far has every s = -inf.
                const float mneg = m == -INFINITY ? 0.0f : -m;
                const uint64_t scale2 = pack2(scale, scale), mneg2 = pack2(mneg, mneg);
                uint32_t pk[2][32];
                uint64_t sum2[2] = {pack2(0.0f, 0.0f), pack2(0.0f, 0.0f)};
#pragma unroll
                for (int c = 0; c < TBN / 2; ++c) {
                    const uint64_t s2 = pack2(__uint_as_float(r[(2 * c) >> 5][(2 * c) & 31]),
                                              __uint_as_float(r[(2 * c + 1) >> 5][(2 * c + 1) & 31]));
                    float a, b;
                    unpack2(ffma2(s2, scale2, mneg2), a, b);
                    a = ex2(a);
                    b = ex2(b);
                    sum2[c & 1] = fadd2(sum2[c & 1], pack2(a, b));
                    pk[c >> 5][c & 31] = pack_half2(a, b);
                }
                {
                    float s0, s1, s2, s3;
                    unpack2(sum2[0], s0, s1);
                    unpack2(sum2[1], s2, s3);
                    l += (s0 + s1) + (s2 + s3);
                }
                tmem_st64(tl + colS, pk);  // the row's P in one instruction
                // Rescale this tile's O before P.V adds to it (PV_X(j-1) finished before S_X(j) was seen: the commit
                // that signalled S_X(j) tracks it).
                if (__any_sync(0xffffffffu, resc && j > 0)) {
                    const float gsc = resc ? f : 1.0f;
#pragma unroll
                    for (int c = 0; c < TD / 32; ++c) {
                        uint32_t o[32];
                        tmem_ld32(tl + colO + c * 32, o);
                        tmem_wait_ld();
                        reg_fence(o);
#pragma unroll
                        for (int e = 0; e < 32; ++e)
                            o[e] = __float_as_uint(__uint_as_float(o[e]) * gsc);
                        tmem_st32(tl + colO + c * 32, o);
                    }
                }
                tmem_wait_st();
                fence_before();
                mbar_arrive(p_full(x));
            }
            if (ok && nb > 0) {
                ok = __all_sync(0xffffffffu, mbar_wait(pv_done(x), nk & 1, WAIT_LIMIT));
                fence_after();
            }
            nk += nb > 0;
            g += nb;
            const float inv = (l > 0.0f ? 1.0f / l : 0.0f) * (p.vinv ? p.vinv[it.kvh] : 1.0f);
            const uint32_t grow = q0 + x * TBM + row;
            if (GATHER) {
                // Head-sharded form: the tile's output goes through its staging box, 32 columns at a time as a
                // 128-byte swizzled box of 128 rows x 32 floats, and TMA stores each box into every rank's o.  The
                // stores run asynchronously: the box is rewritten once they have read it, and the next item's
                // products run meanwhile.
                const uint32_t stage = base + TC_STG + x * BOX_BYTES;
#pragma unroll
                for (int cc = 0; cc < TD / 32; ++cc) {
                    uint32_t o[32];
                    if (ok && nb > 0) {
                        tmem_ld32(tl + colO + cc * 32, o);
                        tmem_wait_ld();
                        reg_fence(o);
                    } else {
#pragma unroll
                        for (int e = 0; e < 32; ++e)
                            o[e] = 0u;
                    }
                    if (row == 0)
                        bulk_wait_read0();  // the box's previous stores have read it
                    named_bar(1 + x, 128);
                    const uint32_t rbase = stage + row * 128;
#pragma unroll
                    for (int k = 0; k < 8; ++k)
                        asm volatile("st.shared.v4.f32 [%0], {%1, %2, %3, %4};\n" ::"r"(rbase + ((k ^ (row & 7)) * 16)),
                                     "f"(__uint_as_float(o[4 * k]) * inv), "f"(__uint_as_float(o[4 * k + 1]) * inv),
                                     "f"(__uint_as_float(o[4 * k + 2]) * inv), "f"(__uint_as_float(o[4 * k + 3]) * inv)
                                     : "memory");
                    fence_proxy_async_smem();
                    named_bar(1 + x, 128);
                    if (row == 0) {
                        for (uint32_t dI = 0; dI < p.n_od; ++dI)
                            tma_store_2d(&p.to[dI], stage, int((p.head0 + h) * TD + cc * 32), int(q0 + x * TBM));
                        bulk_commit();
                    }
                }
            } else {
                // the row's whole output read in one instruction, then stored 32 values at a time
                const uint64_t ooff = uint64_t(grow) * p.width + uint64_t(h) * TD;
                uint32_t o[TD / 32][32];
                if (ok && nb > 0) {
                    if constexpr (TD == 128)
                        tmem_ld128(tl + colO, o);
                    else
                        tmem_ld64(tl + colO, o);
                    tmem_wait_ld();
#pragma unroll
                    for (int c = 0; c < TD / 32; ++c)
                        reg_fence(o[c]);
                } else {
#pragma unroll
                    for (int c = 0; c < TD / 32; ++c)
#pragma unroll
                        for (int e = 0; e < 32; ++e)
                            o[c][e] = 0u;
                }
#pragma unroll
                for (int c = 0; c < TD / 32; ++c)
                    if (grow < p.n_q)
                        out_store32(p.od[0], ooff + c * 32, o[c], inv, p.o_type);
            }
        }
        if (!ok && lane == 0)
            atomicExch(p.err, 3);
        if (GATHER && row == 0)
            bulk_wait0();  // the tile's last boxes have been stored
    }
    __syncwarp();
    fence_before();
    __syncthreads();
    if (warp == 1) {
        fence_after();
        tmem_dealloc(tmem, 512);
    }
}

// ---- bf16 V -> fp16 copy ------------------------------------------------------------------------------------------
//
// One read of V and one write of the copy in the common case: vconv_kernel converts every value as it is (no scale)
// and records each kv head's max |v| over the rows that can be attended (rows < n_rows with valid[row] != 0, as float
// bits); vfix_kernel then looks at that maximum.  A head whose maximum lies in [2^-3, 2^16) (or is 0) keeps the
// unscaled copy: nothing overflows fp16, and a value below fp16's normal range (2^-14) is off by at most 2^-25, under
// 2^-22 of the head's maximum.  Any other head (tiny, huge, inf or NaN) is converted again from V with the power of two
// that puts its maximum in [2^14, 2^15) -- exact for every value above 2^-28 of the maximum -- and vinv = 2^-k undoes
// it in the epilogue.  Rows that cannot be attended are written as zeros.

// The maxima that keep the unscaled copy: 0, or [2^-3, 2^16) as float bits.
__device__ __forceinline__ bool v_unscaled_ok(uint32_t bits)
{
    return bits == 0 || (bits >= (124u << 23) && bits < (143u << 23));
}

// 8 bf16 values (one 16-byte chunk) -> 8 fp16 values scaled by s, and the chunk's max |v| as float bits.
__device__ __forceinline__ uint4 v_chunk(const uint4 w, float s, uint32_t& best)
{
    const uint32_t in[4] = {w.x, w.y, w.z, w.w};
    uint32_t o[4];
#pragma unroll
    for (int k = 0; k < 4; ++k) {
        best = max(best, (in[k] & 0x7FFFu) << 16);
        best = max(best, (in[k] >> 16 & 0x7FFFu) << 16);
        const float a = __uint_as_float(in[k] << 16) * s, b = __uint_as_float(in[k] & 0xFFFF0000u) * s;
        o[k] = pack_half2(a, b);
    }
    return make_uint4(o[0], o[1], o[2], o[3]);
}

constexpr int VC_UNROLL = 4;  // 16-byte chunks a thread has in flight

// Grid (bx, kv_heads), 256 threads: the copy with s (1 here; the scaled redo of vfix_kernel uses the same loop) and,
// when vmax is given, the head's max |v| by atomicMax.  cshift = log2(dim / 8): chunk i lies in row i >> cshift.
__device__ __forceinline__ void v_copy(const __nv_bfloat16* v, __half* v16, uint32_t* vmax, float s, uint32_t kvh,
                                       uint32_t cshift, uint32_t k_pad, uint32_t n_rows, const uint8_t* valid)
{
    const uint64_t per_head = uint64_t(k_pad) << cshift;
    const uint4* src = reinterpret_cast<const uint4*>(v) + uint64_t(kvh) * per_head;
    uint4* dst = reinterpret_cast<uint4*>(v16) + uint64_t(kvh) * per_head;
    const uint64_t live = uint64_t(n_rows) << cshift;  // chunks of rows that may be read
    const uint64_t step = uint64_t(gridDim.x) * blockDim.x * VC_UNROLL;
    uint32_t best = 0;
    for (uint64_t i0 = uint64_t(blockIdx.x) * blockDim.x * VC_UNROLL + threadIdx.x; i0 < per_head; i0 += step) {
        uint4 w[VC_UNROLL];
        bool use[VC_UNROLL];
#pragma unroll
        for (int u = 0; u < VC_UNROLL; ++u) {
            const uint64_t i = i0 + uint64_t(u) * blockDim.x;
            use[u] = i < live && (!valid || valid[i >> cshift]);
            w[u] = use[u] ? __ldcs(src + i) : make_uint4(0, 0, 0, 0);
        }
#pragma unroll
        for (int u = 0; u < VC_UNROLL; ++u) {
            const uint64_t i = i0 + uint64_t(u) * blockDim.x;
            if (i < per_head)
                dst[i] = use[u] ? v_chunk(w[u], s, best) : make_uint4(0, 0, 0, 0);
        }
    }
    if (vmax) {
#pragma unroll
        for (int o = 16; o > 0; o >>= 1)
            best = max(best, __shfl_xor_sync(0xffffffffu, best, o));
        if ((threadIdx.x & 31) == 0 && best)
            atomicMax(vmax + kvh, best);
    }
}

__global__ void __launch_bounds__(256) vconv_kernel(const __nv_bfloat16* v, __half* v16, uint32_t* vmax,
                                                    uint32_t cshift, uint32_t k_pad, uint32_t n_rows,
                                                    const uint8_t* valid)
{
    v_copy(v, v16, vmax, 1.0f, blockIdx.y, cshift, k_pad, n_rows, valid);
    asm volatile("griddepcontrol.launch_dependents;\n" ::: "memory");  // vfix may be scheduled now
}

// The power of two that puts `bits` (a float's bits, |v|max) in [2^14, 2^15), and its inverse; 1 for 0 / inf / nan.
__device__ __forceinline__ void v_scale(uint32_t bits, float& s, float& inv)
{
    const int ex = int(bits >> 23);
    if (bits == 0 || ex >= 255) {
        s = inv = 1.0f;
        return;
    }
    const int e = max(ex - 127, -100);
    s = __int_as_float((127 + 14 - e) << 23);
    inv = __int_as_float((127 + e - 14) << 23);
}

// Grid as vconv_kernel: vinv for every head, and the scaled copy again for the heads whose maximum needs it.
__global__ void __launch_bounds__(256) vfix_kernel(const __nv_bfloat16* v, __half* v16, const uint32_t* vmax,
                                                   float* vinv, uint32_t cshift, uint32_t k_pad, uint32_t n_rows,
                                                   const uint8_t* valid)
{
    asm volatile("griddepcontrol.wait;\n" ::: "memory");  // vconv_kernel's copy and maxima are visible from here on
    const uint32_t kvh = blockIdx.y, bits = vmax[kvh];
    if (v_unscaled_ok(bits)) {
        if (blockIdx.x == 0 && threadIdx.x == 0)
            vinv[kvh] = 1.0f;
        return;
    }
    float s, inv;
    v_scale(bits, s, inv);
    if (blockIdx.x == 0 && threadIdx.x == 0)
        vinv[kvh] = inv;
    v_copy(v, v16, nullptr, s, kvh, cshift, k_pad, n_rows, valid);
}

// ---- host ----------------------------------------------------------------------------------------------------------

// o [n_q][width] fp32 as a TMA store target: boxes of 128 rows x 32 floats (128 bytes, 128-byte swizzle).
bool out_map(CUtensorMap* map, float* o, uint32_t n_q, uint32_t width)
{
    auto enc = tensor_map_encoder();
    if (!enc)
        return false;
    cuuint64_t dims[2] = {width, n_q};
    cuuint64_t strides[1] = {uint64_t(width) * 4};
    cuuint32_t box[2] = {32, 128};
    cuuint32_t estr[2] = {1, 1};
    return enc(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, o, dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
               CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_NONE,
               CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

} // namespace

cudaError_t launch_v_to_f16(const void* v, void* v16, uint32_t* vmax, float* vinv, uint32_t dim, uint32_t kv_heads,
                            uint32_t k_pad, uint32_t n_rows, const uint8_t* valid, int num_sms, cudaStream_t st)
{
    if (dim != 64 && dim != 128 && dim != 256)
        return cudaErrorInvalidValue;
    cudaError_t e = cudaMemsetAsync(vmax, 0, kv_heads * sizeof(uint32_t), st);
    if (e != cudaSuccess)
        return e;
    const uint32_t cshift = dim == 64 ? 3 : dim == 128 ? 4 : 5;
    const uint64_t chunks = uint64_t(k_pad) << cshift;
    uint32_t bx = uint32_t((chunks + 256 * VC_UNROLL - 1) / (256 * VC_UNROLL));
    const uint32_t cap = uint32_t((num_sms * 8 + kv_heads - 1) / kv_heads);
    bx = bx < 1 ? 1 : (bx > cap ? cap : bx);
    const auto* vb = static_cast<const __nv_bfloat16*>(v);
    auto* vh = static_cast<__half*>(v16);
    vconv_kernel<<<dim3(bx, kv_heads), 256, 0, st>>>(vb, vh, vmax, cshift, k_pad, n_rows, valid);
    if ((e = cudaGetLastError()) != cudaSuccess)
        return e;
    // vfix launched as a programmatic dependent of vconv: its blocks are scheduled as vconv's last blocks run and
    // wait (griddepcontrol.wait) for vconv's writes.
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(bx, kv_heads);
    cfg.blockDim = dim3(256);
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, vfix_kernel, vb, vh, static_cast<const uint32_t*>(vmax), vinv, cshift, k_pad,
                              n_rows, valid);
}

cudaError_t launch_attn_tc(const AttnParams& a, int dtype, int dim, const void* v16, const float* vinv, int* err,
                           cudaStream_t st)
{
    if (a.n_q == 0 || a.heads == 0)
        return cudaSuccess;
    if (dim != 64 && dim != 128)
        return cudaErrorInvalidValue;
    TcParams p;
    const bool bf = dtype == kBF16;
    if (!tile_map(&p.tq, a.q, bf, dim, a.q_pad, a.heads, TBM) ||
        !tile_map(&p.tk, a.k, bf, dim, a.k_pad, a.kv_heads, TBN) ||
        !tile_map(&p.tv, bf ? v16 : a.v, false, dim, a.k_pad, a.kv_heads, TBN))
        return cudaErrorInvalidValue;
    if (a.n_od == 0) {
        p.od[0] = a.o;
        p.n_od = 1;
        p.head0 = 0;
    } else {
        if (a.n_od > 8)
            return cudaErrorInvalidValue;
        for (uint32_t i = 0; i < a.n_od; ++i) {
            p.od[i] = a.od[i];
            if (a.n_od > 1 && !out_map(&p.to[i], a.od[i], a.n_q, a.width))
                return cudaErrorInvalidValue;
        }
        p.n_od = a.n_od;
        p.head0 = a.head0;
    }
    p.err = err;
    p.vinv = bf ? vinv : nullptr;
    p.qk_fmt = bf ? 1u : 0u;
    p.o_type = a.o_type;
    if (p.n_od > 1 && p.o_type != 0)
        return cudaErrorInvalidValue;  // the head-sharded epilogue stores fp32 boxes
    p.n_q = a.n_q;
    p.q_pad = a.q_pad;
    p.n_k = a.n_k;
    p.k_pad = a.k_pad;
    p.heads = a.heads;
    p.kv_heads = a.kv_heads;
    p.q_pos0 = a.q_pos0;
    p.block = a.block;
    p.width = a.width;
    p.n_tiles = (a.q_pad + 2 * TBM - 1) / (2 * TBM);
    {
        // kv heads whose keys and values take at most 64 MB (about half the 126 MB L2), at least one
        const uint64_t kv_bytes = uint64_t(a.n_k) * dim * 2 * 2;
        uint64_t kv_per_group = kv_bytes ? (uint64_t(64) << 20) / kv_bytes : a.kv_heads;
        kv_per_group = kv_per_group < 1 ? 1 : (kv_per_group > a.kv_heads ? a.kv_heads : kv_per_group);
        p.group_heads = uint32_t(kv_per_group) * (a.heads / a.kv_heads);
    }
    p.scale_log2 = a.scale * kLog2e;
    const bool gather = p.n_od > 1;
    if (gather && dim != 128)
        return cudaErrorInvalidValue;  // the head-sharded epilogue stages boxes of 128-wide rows
    auto kern = dim == 64 ? attn_tc_kernel<64, false> : gather ? attn_tc_kernel<128, true> : attn_tc_kernel<128, false>;
    const uint32_t smem = dim == 64 ? TcSmem<64>::TOTAL : gather ? TC_TOTAL_GATHER : TcSmem<128>::TOTAL;
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e != cudaSuccess)
        return e;
    // One CTA per SM, each working through its share of the items.
    const uint32_t n_items = p.n_tiles * a.heads;
    const uint32_t sms = a.num_sms ? a.num_sms : 148;
    const uint32_t grid = n_items < sms ? n_items : sms;
    kern<<<grid, TNT, smem, st>>>(p);
    return cudaGetLastError();
}

} // namespace mako
