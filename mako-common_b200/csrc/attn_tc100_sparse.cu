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
// A persistent grid (one CTA of 384 threads per SM) works through (tile, head) items head by head.  Warp 0 loads each
// item's Q once and the K ring, warp 2 the V ring (TMA, 64-row boxes for K and V so each half can come from anywhere;
// K in a 2-stage ring, V in a 3-stage ring), warp 1 issues UMMA, and warps 4-11 run the softmax and the epilogue:
// each query row (TMEM lane) belongs to one thread of warps 4-7 (parity 0) and one of warps 8-11 (parity 1), which
// take alternate passes.  TMEM (512 columns): S of parity x in columns 128 x .. 128 x + 127 (its P, fp16 pairs,
// written over the first 64), one O accumulator (256-383) and the item's Q (384-447, the A operand of Q.K^T, copied
// there by the softmax threads from the TMA tile).  The issue order is QK(0), QK(1), then per pass PV(i), QK(i + 2).
// Precision, bounded waits and the error flag as the dense kernel (attn_tc100.cu).
#include "common.cuh"
#include "kernels.h"
#include "tc100.cuh"

#include <cudaTypedefs.h>

#include <type_traits>

namespace mako {
namespace {

using namespace tc;

constexpr int SD = 128, SNT = 384, NSK = 2, NSV = 3;
constexpr uint32_t DBOX = 128 * 64 * 2;  // one d-half of a 128-row tile: 16 KB
constexpr uint32_t HBOX = 64 * 64 * 2;   // a 64-row x 64-value TMA box: 8 KB
constexpr uint32_t STILE = 2 * DBOX;     // 128 rows x 128 values
constexpr uint32_t S_Q = 0, S_K = STILE, S_V = S_K + NSK * STILE, S_BAR = S_V + NSV * STILE;
constexpr uint32_t S_STAT = S_BAR + 256;   // float2 [2 parities][128 rows]: each thread's (maximum, sum share)
constexpr uint32_t S_MAX = S_STAT + 2048;  // float [128 rows]: the running maximum handed between the parities
constexpr uint32_t S_STAGE = (S_MAX + 512 + 1023) / 1024 * 1024;  // 2 KB per softmax warp: 32 rows x 16 floats
constexpr uint32_t S_TOTAL = S_STAGE + 8 * 2048 + 1024;
// TMEM columns: S (and the P that replaces it) of parity x at 128 x, O at COL_O, Q (bf16 or fp16 pairs) at COL_Q,
// and at COL_SPARE + 32 x the epilogue's parked output chunk of parity x
constexpr uint32_t COL_O = 256, COL_Q = 384, COL_SPARE = 448;
constexpr long long S_WAIT_LIMIT = 1ll << 31;

struct __align__(64) SpParams {
    CUtensorMap tk, tv;  // k and v (or the fp16 copy of v), 64-row boxes
    CUtensorMap tq;      // q, 128-row boxes
    CUtensorMap to;      // o [n_q][width] fp32, boxes of 32 rows x 16 floats (64-byte swizzle), when use_tma_out
    const void* q;
    float* o;
    int* err;
    const float* vinv;
    const void* sel;
    const void* nsel;
    const uint8_t* valid;
    const int32_t* map;
    uint32_t sel_i32, qk_fmt, o_type, use_tma_out;
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
    return p.sel_i32 ? uint32_t(__ldg(static_cast<const int32_t*>(base) + i))
                     : uint32_t(__ldg(static_cast<const uint16_t*>(base) + i));
}

// A tile's list lengths as read from nsel (two cubes; 0 past the cubes), loaded without being used, so that a caller
// can issue the loads early and build the TileInfo later (tile_from).
struct TileRaw {
    int64_t n[2];
};
__device__ __forceinline__ TileRaw tile_raw(const SpParams& p, uint32_t u, uint32_t h)
{
    TileRaw r{{0, 0}};
    if (u < p.tiles_cube)
        for (uint32_t hh = 0; hh < 2; ++hh) {
            const uint32_t c = 2 * u + hh;
            if (c < p.n_cubes)
                r.n[hh] = p.sel_i32 ? int64_t(static_cast<const int32_t*>(p.nsel)[uint64_t(h) * p.n_cubes + c])
                                    : int64_t(static_cast<const uint16_t*>(p.nsel)[uint64_t(h) * p.n_cubes + c]);
        }
    return r;
}
__device__ __forceinline__ TileInfo tile_from(const SpParams& p, uint32_t u, const TileRaw& r)
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
            const int64_t raw = c < p.n_cubes ? r.n[hh] : 0;
            t.ns[hh] = raw <= 0 ? 0u : (raw < int64_t(p.max_sel) ? uint32_t(raw) : p.max_sel);
        }
        t.ncp = max(t.ns[0], t.ns[1]);
        t.np = t.ncp + (p.dense1 > p.dense0 ? (p.dense1 - p.dense0 + 127) / 128 : 0);
    } else {
        t.row0 = p.n_cubes * 64 + (u - p.tiles_cube) * 128;
        t.np = (p.n_k + 127) / 128;
    }
    return t;
}
__device__ __forceinline__ TileInfo tile_info(const SpParams& p, uint32_t u, uint32_t h)
{
    return tile_from(p, u, tile_raw(p, u, h));
}

// The list entry a cube pass reads (pass pi, half hh), or 0xFFFFFFFF when the list has no entry there; read well
// before use so its latency hides behind a pass.
__device__ __forceinline__ uint32_t raw_entry(const SpParams& p, const TileInfo& t, uint32_t h, uint32_t pi,
                                              uint32_t hh)
{
    if (!(t.cube && pi < t.ns[hh]))
        return 0xFFFFFFFFu;
    return list_entry(p, p.sel, (uint64_t(h) * p.n_cubes + t.cube_id[hh]) * p.max_sel + pi);
}
// Key rows of pass `pi`, half `hh` (tile rows 64 hh .. 64 hh + 63 of K / V) start at j0; keys j < hi are in range.
// Cube passes: the half belongs to one query cube, whose list entry for the pass is `raw` (none, or >= n_cubes: the
// half is empty, hi = j0 = 0, and rows 0 .. 63 are still loaded so that the masked half of K / V holds finite
// values).  Other passes: 128 consecutive keys of the dense rows or of all keys.
__device__ __forceinline__ void keys_of(const SpParams& p, const TileInfo& t, uint32_t pi, uint32_t hh, uint32_t raw,
                                        uint32_t& j0, uint32_t& hi)
{
    if (t.cube && pi < t.ncp) {
        const bool ok = raw < p.n_cubes;
        j0 = ok ? raw * 64 : 0;
        hi = ok ? j0 + 64 : 0;
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

// Masks (to -inf bits) the columns c of r whose key j0 + c is out of range or invalid.  NC columns from j0, which
// is a multiple of 32 (cube starts, dense0 and 128-key steps), so valid[] is read 16 bytes at a time.
template <int NC>
__device__ __forceinline__ void mask_keys(uint32_t (&r)[NC], const uint8_t* valid, uint32_t j0, uint32_t hi)
{
    if (hi >= j0 + NC && !valid)
        return;
#pragma unroll
    for (int c0 = 0; c0 < NC; c0 += 16) {
        uint4 w = make_uint4(0x01010101u, 0x01010101u, 0x01010101u, 0x01010101u);
        if (valid && j0 + c0 < hi)
            w = __ldg(reinterpret_cast<const uint4*>(valid + j0 + c0));
        const uint32_t words[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
        for (int c = 0; c < 16; ++c) {
            const bool ok = j0 + c0 + c < hi && ((words[c >> 2] >> (8 * (c & 3))) & 0xFFu) != 0;
            if (!ok)
                r[c0 + c] = 0xFF800000u;
        }
    }
}

// Work item i of tiles_total * heads: head h = i / tiles_total, row tile u = tiles_total - 1 - i % tiles_total (the
// tiles after the cubes, which see every key, first).  Consecutive items share a head, so the CTAs in flight read the
// keys of a few heads and those stay in L2.  A persistent CTA takes one item per round of gridDim.x items, snaking as
// the dense kernel does; while the softmax warps store one item's output, the producers load the next item's Q and
// first key cubes and the issuer starts its Q.K^T.
__device__ __forceinline__ uint32_t sp_item(uint32_t round)
{
    const uint32_t G = gridDim.x, c = (round & 1) ? G - 1 - blockIdx.x : blockIdx.x;
    return round * G + c;
}

// Passes alternate between two softmax warpgroups ("parities"): parity x takes the passes whose running number (over
// the CTA's items) has x as its low bit, each parity with its own S buffer (a pass's P replaces its S in place and
// P.V reads it from TMEM).  Both parities accumulate into one O, so a row's running maximum is one sequence over the
// item's passes, as in the reference: the thread that owns pass i takes the maximum pass i - 1 left (a named-barrier
// hand-over between the two threads of the row), raises it when the pass's own maximum passes it by 8, hands it on,
// and rescales O once the other parity's P.V(i - 1) has finished.  Each thread keeps its own share of the row sum,
// relative to the maximum it last saw; the epilogue adds the two shares.  Q.K^T of pass i + 2 into the same S buffer
// is issued right behind P.V(i): the tensor pipe executes one thread's MMAs in issue order.  Q sits in TMEM as the A
// operand of Q.K^T, so Q.K^T reads only K from shared memory.
__global__ void __launch_bounds__(SNT, 1) attn_tc_sparse_kernel(const __grid_constant__ SpParams p)
{
    extern __shared__ uint8_t smem_raw[];
    const uint32_t raw = smem_u32(smem_raw);
    const uint32_t base = (raw + 1023u) & ~1023u;
    uint8_t* const gbase = smem_raw + (base - raw);
    const uint32_t sB = base + S_BAR;
    auto k_full = [&](uint32_t s) { return sB + 8 * s; };
    auto k_empty = [&](uint32_t s) { return sB + 24 + 8 * s; };
    auto v_full = [&](uint32_t s) { return sB + 48 + 8 * s; };
    auto v_empty = [&](uint32_t s) { return sB + 72 + 8 * s; };
    auto s_full = [&](uint32_t x) { return sB + 96 + 8 * x; };
    auto p_full = [&](uint32_t x) { return sB + 112 + 8 * x; };
    auto o_done = [&](uint32_t x) { return sB + 128 + 8 * x; };  // the item's last P.V of parity x has finished
    const uint32_t q_full = sB + 152, mma_done = sB + 160;
    const uint32_t tmem_slot = sB + 168;
    const uint32_t q_empty = sB + 176;  // an item's last Q.K^T has finished: TMEM's Q may be overwritten
    const uint32_t q_tmem = sB + 184;   // the item's Q is in TMEM, and shared memory's Q buffer is free again
    volatile uint32_t* tmem_slot_ptr = reinterpret_cast<volatile uint32_t*>(smem_raw + (tmem_slot - raw));

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t n_items = p.tiles_total * p.heads;
    auto item = [&](uint32_t i, uint32_t& h, uint32_t& kvh) {
        h = i / p.tiles_total;
        kvh = h / (p.heads / p.kv_heads);
        return tile_info(p, p.tiles_total - 1 - i % p.tiles_total, h);
    };

    if (threadIdx.x == 0) {
        for (uint32_t s = 0; s < 3; ++s) {
            mbar_init(k_full(s), 1);
            mbar_init(k_empty(s), 1);
            mbar_init(v_full(s), 1);
            mbar_init(v_empty(s), 1);
        }
        for (uint32_t x = 0; x < 2; ++x) {
            mbar_init(s_full(x), 1);
            mbar_init(p_full(x), 4);  // one arrival per warp of the parity's warpgroup
            mbar_init(o_done(x), 1);
        }
        mbar_init(q_full, 1);
        mbar_init(q_empty, 1);
        mbar_init(q_tmem, 8);  // one arrival per softmax warp
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

    // Counters every role keeps alike: g counts the passes of the items so far (ring stages, parities and the phases
    // of their barriers), nq the items with passes (Q loads and copies, q_full / q_tmem / q_empty phases), nd[x] the
    // items with a pass of parity x (o_done(x) phases).
    if (warp < 4) {
        // the producer / issuer warpgroup gives registers to the softmax warpgroups (384 x 168 at launch =
        // 128 x 104 + 256 x 200)
        asm volatile("setmaxnreg.dec.sync.aligned.u32 104;\n" ::: "memory");
        if ((warp == 0 || warp == 2) && lane == 0) {
            // ---------------- TMA producers: warp 0 Q and the K ring, warp 2 the V ring ----------------
            const bool is_k = warp == 0;
            const CUtensorMap* map = is_k ? &p.tk : &p.tv;
            const uint32_t ring = base + (is_k ? S_K : S_V), nst = is_k ? NSK : NSV;
            tma_prefetch_desc(map);
            if (is_k)
                tma_prefetch_desc(&p.tq);
            bool ok = true;
            uint32_t g = 0, nq = 0, issued = 0;
            for (uint32_t round = 0; ok; ++round) {
                const uint32_t i = sp_item(round);
                if (i >= n_items)
                    break;
                uint32_t h, kvh;
                const TileInfo t = item(i, h, kvh);
                if (t.np == 0)
                    continue;
                if (is_k) {  // the item's Q, once the softmax warps have copied the previous one into TMEM
                    if (nq > 0 && !mbar_wait(q_tmem, (nq - 1) & 1, S_WAIT_LIMIT)) {
                        ok = false;
                        break;
                    }
                    mbar_expect_tx(q_full, STILE);
                    for (int dh = 0; dh < 2; ++dh)
                        tma_load_3d(base + S_Q + dh * DBOX, &p.tq, q_full, dh * 64, int(t.row0), int(h));
                }
                ++nq;
                uint32_t rawn[2] = {raw_entry(p, t, h, 0, 0), raw_entry(p, t, h, 0, 1)};
                for (uint32_t pi = 0; pi < t.np; ++pi) {
                    uint32_t j0[2], hi;
                    keys_of(p, t, pi, 0, rawn[0], j0[0], hi);
                    keys_of(p, t, pi, 1, rawn[1], j0[1], hi);
                    if (pi + 1 < t.np) {  // the next pass's list entries are read while this pass waits for its stage
                        rawn[0] = raw_entry(p, t, h, pi + 1, 0);
                        rawn[1] = raw_entry(p, t, h, pi + 1, 1);
                    }
                    const uint32_t gi = g + pi, s = gi % nst, ph = (gi / nst) & 1;
                    if (gi >= nst && !mbar_wait(is_k ? k_empty(s) : v_empty(s), ph ^ 1, S_WAIT_LIMIT)) {
                        ok = false;
                        break;
                    }
                    const uint32_t full = is_k ? k_full(s) : v_full(s);
                    mbar_expect_tx(full, STILE);
                    for (uint32_t hh = 0; hh < 2; ++hh)
                        for (int dh = 0; dh < 2; ++dh)
                            tma_load_3d(ring + s * STILE + dh * DBOX + hh * HBOX, map, full, dh * 64, int(j0[hh]),
                                        kvh);
                    ++issued;
                }
                g += t.np;
            }
            if (!ok)
                atomicExch(p.err, 11);
            // Our copies in flight land before the CTA leaves (already so on the normal path).
            if (is_k && nq > 0)
                mbar_wait(q_full, (nq - 1) & 1, S_WAIT_LIMIT);
            for (uint32_t k = issued > nst ? issued - nst : 0; k < issued; ++k)
                mbar_wait(is_k ? k_full(k % nst) : v_full(k % nst), (k / nst) & 1, S_WAIT_LIMIT);
        } else if (warp == 1 && lane == 0) {
            // ---------------- UMMA issuer ----------------
            // Per item QK(0), QK(1), then per pass PV(i), QK(i + 2), one commit per Q.K^T; the K and V stages are
            // released by a softmax thread that observes those completions anyway.
            const uint32_t idesc_qk = idesc_f16(p.qk_fmt, p.qk_fmt, 0, 0, 128, 128);
            const uint32_t idesc_pv = idesc_f16(0, 0, 0, 1, 128, SD);
            // Q.K^T(gj) into parity gj's S; `seen`: K(gj) is known to have landed (a softmax thread waited for it)
            auto qk = [&](uint32_t gj, bool seen) {
                const uint32_t s = gj % NSK, x = gj & 1;
                if (!seen && !mbar_wait(k_full(s), (gj / NSK) & 1, S_WAIT_LIMIT))
                    return false;
                fence_after();
#pragma unroll
                for (uint32_t ks = 0; ks < SD / 16; ++ks)
                    umma_ts(tmem + x * 128, tmem + COL_Q + ks * 8,
                            sdesc(base + S_K + s * STILE + (ks >> 2) * DBOX + (ks & 3) * 32, 16, 1024), idesc_qk,
                            ks > 0);
                umma_commit(s_full(x));
                return true;
            };
            bool ok = true;
            uint32_t g = 0, nq = 0;
            for (uint32_t round = 0; ok; ++round) {
                const uint32_t i = sp_item(round);
                if (i >= n_items)
                    break;
                uint32_t h, kvh;
                const TileInfo t = item(i, h, kvh);
                if (t.np == 0)
                    continue;
                ok = mbar_wait(q_tmem, nq & 1, S_WAIT_LIMIT);
                ++nq;
                fence_after();
                ok = ok && qk(g, false) && (t.np < 2 || qk(g + 1, false));
                if (ok && t.np <= 2)
                    umma_commit(q_empty);
                for (uint32_t pi = 0; ok && pi < t.np; ++pi) {
                    const uint32_t gi = g + pi, x = gi & 1, s = gi % NSV;
                    ok = mbar_wait(p_full(x), (gi >> 1) & 1, S_WAIT_LIMIT);  // P(i), V(i) and K(i + 2)
                    if (!ok)
                        break;
                    fence_after();
#pragma unroll
                    for (uint32_t kk = 0; kk < 8; ++kk)
                        umma_ts(tmem + COL_O, tmem + 128 * x + kk * 8,
                                sdesc(base + S_V + s * STILE + kk * 2048, DBOX, 1024), idesc_pv, pi > 0 || kk > 0);
                    if (pi + 2 < t.np) {
                        ok = qk(gi + 2, true);  // K(i + 2) was waited for before P(i) was published
                        if (ok && pi + 3 == t.np)
                            umma_commit(q_empty);
                    } else {
                        umma_commit(o_done(x));  // parity x's last product of the item
                    }
                }
                g += t.np;
            }
            if (!ok)
                atomicExch(p.err, 12);
            umma_commit(mma_done);  // every MMA issued above has finished before TMEM is freed
            mbar_wait(mma_done, 0, S_WAIT_LIMIT);
        }
    } else {
        asm volatile("setmaxnreg.inc.sync.aligned.u32 200;\n" ::: "memory");
        // ---------------- softmax of parity x and the epilogue: tile row `row` ----------------
        const uint32_t x = (warp - 4) >> 2, qd = warp & 3, row = qd * 32 + lane, hr = row >> 6;
        const uint32_t tl = tmem + ((qd * 32) << 16);
        const uint32_t colS = 128 * x;
        float* const mrow = reinterpret_cast<float*>(gbase + S_MAX);
        float2* const stat = reinterpret_cast<float2*>(gbase + S_STAT);
        // named barriers of the row quadrant qd: 1 + 2 qd + y hands the running maximum to parity y's thread,
        // 9 + qd pairs the two threads in the epilogue
        const uint32_t bar_get = 1 + 2 * qd + x, bar_put = 1 + 2 * qd + (x ^ 1), bar_epi = 9 + qd;
        const float scale = p.scale_log2;
        const uint64_t scale2 = pack2(scale, scale);
        bool ok = true;
        uint32_t g = 0, nq = 0, nd0 = 0, nd1 = 0;
        auto nd = [&](uint32_t y) { return y ? nd1 : nd0; };
        // Every softmax thread walks all of its CTA's items, also after a failed wait (then without waiting or
        // computing, but still meeting its partner at every named barrier, which cannot time out).  An item
        // without passes (no key at all) stores zeros.
        // The next item's list lengths and its first list entry are loaded one item ahead (before the current
        // item's epilogue), so an item's start does not wait on global memory.
        auto unit = [&](uint32_t i) { return p.tiles_total - 1 - i % p.tiles_total; };
        auto entry_of = [&](const TileInfo& tt, uint32_t hh_, uint32_t pi) {
            return tt.cube && pi < tt.ncp ? raw_entry(p, tt, hh_, pi, hr) : 0u;
        };
        // Q of the next item with passes into TMEM: this thread's row, d-half x (64 values, two a column, the
        // layout of an A operand), read from the 128-byte-swizzled tile TMA left in shared memory.
        auto copy_q = [&]() {
            if (ok && nq > 0)  // the previous item's last Q.K^T has read TMEM's Q
                ok = __all_sync(0xffffffffu, mbar_wait(q_empty, (nq - 1) & 1, S_WAIT_LIMIT));
            if (ok)
                ok = __all_sync(0xffffffffu, mbar_wait(q_full, nq & 1, S_WAIT_LIMIT));
            if (ok) {
                fence_after();
                uint32_t r[32];
                const uint32_t src = base + S_Q + x * DBOX + row * 128;
#pragma unroll
                for (int c = 0; c < 8; ++c)
                    asm volatile("ld.shared.v4.u32 {%0, %1, %2, %3}, [%4];\n"
                                 : "=r"(r[4 * c]), "=r"(r[4 * c + 1]), "=r"(r[4 * c + 2]), "=r"(r[4 * c + 3])
                                 : "r"(src + ((c ^ (row & 7)) * 16))
                                 : "memory");
                tmem_st32(tl + COL_Q + 32 * x, r);
                tmem_wait_st();
            }
            fence_before();
            __syncwarp();
            if (lane == 0)
                mbar_arrive(q_tmem);
            ++nq;
        };
        uint32_t ii = sp_item(0);
        TileInfo t = ii < n_items ? tile_info(p, unit(ii), ii / p.tiles_total) : TileInfo{};
        uint32_t raw_next = ii < n_items ? entry_of(t, ii / p.tiles_total, (g & 1) == x ? 0u : 1u) : 0u;
        bool q_in = false;  // the current item's Q was copied at the end of the previous item
        // The epilogue reads this thread's 64 output columns out of O, stores the first 32 right away and parks the
        // other 32 in spare TMEM columns (COL_SPARE + 32 x), so that O is free for the next item's first P.V sooner;
        // the parked chunk is stored after this thread's next pass (pend: a chunk is parked).  The store metadata
        // below belongs to the item whose output is being stored.
        int pend = 0;
        float p_inv = 0.0f;
        uint64_t p_orow = 0;
        bool p_tma = false, p_store = false;
        uint32_t p_col = 0, p_row = 0;
        const uint32_t stage = base + S_STAGE + (warp - 4) * 2048;
        auto store_chunk = [&](int k, const uint32_t (&o)[32]) {
            if (p_tma) {
                // the warp's 32 rows x 16 columns at a time through its staging buffer (row = lane, 16-byte
                // chunks in the 64-byte swizzle's order), stored by one TMA box
#pragma unroll
                for (int hf = 0; hf < 2; ++hf) {
                    if (lane == 0)
                        bulk_wait_read0();  // the previous box has been read out of the buffer
                    __syncwarp();
#pragma unroll
                    for (int c = 0; c < 4; ++c)
                        asm volatile("st.shared.v4.f32 [%0], {%1, %2, %3, %4};\n" ::"r"(
                                         stage + lane * 64 + ((c ^ ((lane >> 1) & 3)) * 16)),
                                     "f"(__uint_as_float(o[16 * hf + 4 * c]) * p_inv),
                                     "f"(__uint_as_float(o[16 * hf + 4 * c + 1]) * p_inv),
                                     "f"(__uint_as_float(o[16 * hf + 4 * c + 2]) * p_inv),
                                     "f"(__uint_as_float(o[16 * hf + 4 * c + 3]) * p_inv)
                                     : "memory");
                    fence_proxy_async_smem();
                    __syncwarp();
                    if (lane == 0) {
                        tma_store_2d(&p.to, stage, int(p_col + 32 * k + 16 * hf), int(p_row));
                        bulk_commit();
                    }
                }
            } else if (p_store) {
                out_store32(p.o, p_orow + 32 * k, o, p_inv, p.o_type);
            }
        };
        auto store_one = [&]() {
            if (pend > 0) {
                uint32_t pb[32];
                tmem_ld32(tl + COL_SPARE + 32 * x, pb);
                tmem_wait_ld();
                reg_fence(pb);
                store_chunk(1, pb);
            }
            pend = 0;
        };
        for (uint32_t round = 0; ii < n_items; ++round) {
            const uint32_t h = ii / p.tiles_total, kvh = h / (p.heads / p.kv_heads);
            const uint32_t ii_n = sp_item(round + 1);
            const TileRaw rn = ii_n < n_items ? tile_raw(p, unit(ii_n), ii_n / p.tiles_total) : TileRaw{{0, 0}};
            if (t.np > 0 && !q_in)
                copy_q();
            float mref = -INFINITY, l = 0.0f;  // this thread's share of the row sum, relative to maximum mref
            // the epilogue's global reads (v's scale, the row map) issued now, consumed after the passes
            const float vscale = p.vinv ? p.vinv[kvh] : 1.0f;
            const uint32_t grow = t.row0 + row;
            bool store = t.active && grow < p.n_q && (!t.cube || t.cube_id[hr] < p.n_cubes);
            int64_t dst = grow;
            if (store && p.map) {
                dst = p.map[grow];
                store = dst >= 0;
            }

            // One pass of this parity: S (NK columns of this row from column c0) to P in place.  NK 64: a cube pass,
            // the row's own cube half (the other half's P is zero); NK 128: every column.
            auto pass = [&](auto nk_tag, uint32_t pi, uint32_t gi, uint32_t c0, uint32_t key0, uint32_t hi) {
                constexpr int NK = decltype(nk_tag)::value;
                uint32_t r[NK / 32][32];
                if constexpr (NK == 64)
                    tmem_ld64(tl + colS + c0, r);  // the row's scores in one instruction
                else
                    tmem_ld128(tl + colS + c0, r);
                tmem_wait_ld();
#pragma unroll
                for (int k = 0; k < NK / 32; ++k) {
                    reg_fence(r[k]);
                    mask_keys<32>(r[k], p.valid, key0 + 32 * k, hi);
                }
                float mq[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
#pragma unroll
                for (int c = 0; c < NK; c += 8)
#pragma unroll
                    for (int e = 0; e < 4; ++e)
                        mq[e] = max3f(mq[e], __uint_as_float(r[(c + 2 * e) >> 5][(c + 2 * e) & 31]),
                                      __uint_as_float(r[(c + 2 * e + 1) >> 5][(c + 2 * e + 1) & 31]));
                const float mx = fmaxf(fmaxf(mq[0], mq[1]), fmaxf(mq[2], mq[3])) * scale;
                // the running maximum after pass i - 1 (written by the other parity's thread of this row)
                float mprev = -INFINITY;
                if (pi > 0) {
                    named_bar(bar_get, 64);
                    mprev = mrow[row];
                }
                const float m = mx > mprev + 8.0f ? mx : mprev;
                if (pi + 1 < t.np) {
                    mrow[row] = m;
                    named_arrive(bar_put, 64);
                }
                // O holds the earlier passes at maximum mprev; this thread's sum share at mref
                const bool resc = m != mprev && mprev != -INFINITY;
                if (m != mref) {
                    l = mref == -INFINITY ? 0.0f : l * ex2(mref - m);
                    mref = m;
                }
                const float mneg = m == -INFINITY ? 0.0f : -m;
                const uint64_t mneg2 = pack2(mneg, mneg);
                uint32_t pk[NK / 64][32];
                uint64_t sum2[2] = {pack2(0.0f, 0.0f), pack2(0.0f, 0.0f)};
#pragma unroll
                for (int c = 0; c < NK / 2; ++c) {
                    float a, b;
                    unpack2(ffma2(pack2(__uint_as_float(r[(2 * c) >> 5][(2 * c) & 31]),
                                        __uint_as_float(r[(2 * c + 1) >> 5][(2 * c + 1) & 31])),
                                  scale2, mneg2),
                            a, b);
                    a = ex2(a);
                    b = ex2(b);
                    sum2[c & 1] = fadd2(sum2[c & 1], pack2(a, b));
                    pk[c >> 5][c & 31] = pack_half2s(a, b);
                }
                {
                    float s0, s1, s2, s3;
                    unpack2(sum2[0], s0, s1);
                    unpack2(sum2[1], s2, s3);
                    l += (s0 + s1) + (s2 + s3);
                }
                // P over S's first 64 columns (two keys a column): a cube pass fills its cube's 32 and zeros the
                // other 32; every S value this thread needs is in registers by now
                if (NK == 64) {
                    tmem_st32(tl + colS + 32 * hr, pk[0]);
                    tmem_st16_zero(tl + colS + 32 * (hr ^ 1));
                    tmem_st16_zero(tl + colS + 32 * (hr ^ 1) + 16);
                } else {
#pragma unroll
                    for (int k = 0; k < NK / 64; ++k)
                        tmem_st32(tl + colS + 32 * k, pk[k]);
                }
                // Rescale O before P.V(i) adds to it, once the other parity's P.V(i - 1) has finished: the commit
                // of Q.K^T(i + 1), issued after it, or the commit of that parity's last product of the item.
                if (__any_sync(0xffffffffu, resc)) {
                    const bool w = pi + 1 < t.np ? mbar_wait(s_full(x ^ 1), ((gi + 1) >> 1) & 1, S_WAIT_LIMIT)
                                                 : mbar_wait(o_done(x ^ 1), nd(x ^ 1) & 1, S_WAIT_LIMIT);
                    ok = __all_sync(0xffffffffu, w);
                    fence_after();
                    const float gsc = resc ? ex2(mprev - m) : 1.0f;
#pragma unroll
                    for (int k = 0; ok && k < 4; ++k) {
                        uint32_t o[32];
                        tmem_ld32(tl + COL_O + 32 * k, o);
                        tmem_wait_ld();
                        reg_fence(o);
#pragma unroll
                        for (int e = 0; e < 32; ++e)
                            o[e] = __float_as_uint(__uint_as_float(o[e]) * gsc);
                        tmem_st32(tl + COL_O + 32 * k, o);
                    }
                }
                tmem_wait_st();
                fence_before();
                // P(i) is published once V(i) and K(i + 2) have landed too, so that the issuer waits on one barrier
                // between P.V(i) and Q.K^T(i + 2) (both arrive well ahead; the waits cost the softmax time it has)
                const bool vw = lane != 0 || (mbar_wait(v_full(gi % NSV), (gi / NSV) & 1, S_WAIT_LIMIT) &&
                                              (pi + 2 >= t.np ||
                                               mbar_wait(k_full((gi + 2) % NSK), ((gi + 2) / NSK) & 1, S_WAIT_LIMIT)));
                ok = __all_sync(0xffffffffu, vw) && ok;
                if (lane == 0)
                    mbar_arrive_n(p_full(x), 1);
            };

            // This thread's list entry (its cube's) for each of this parity's cube passes, read one pass of the
            // parity (two passes) ahead so that the load's latency hides behind a pass.
            auto entry = [&](uint32_t pi) { return entry_of(t, h, pi); };
            const uint32_t first = ((g & 1) == x) ? 0u : 1u;  // this parity's first pass of the item
            for (uint32_t pi = first; pi < t.np; pi += 2) {
                const uint32_t gi = g + pi;
                const uint32_t raw = raw_next;
                if (pi + 2 < t.np)
                    raw_next = entry(pi + 2);
                const bool half = t.cube && pi < t.ncp;  // this row sees only its cube's 64 keys
                uint32_t j0, hi;
                keys_of(p, t, pi, half ? hr : 0, half ? raw : 0u, j0, hi);
                if (ok)
                    ok = __all_sync(0xffffffffu, mbar_wait(s_full(x), (gi >> 1) & 1, S_WAIT_LIMIT));
                if (ok && (threadIdx.x & 127) == 0) {
                    // S(i) seen: Q.K^T(i) has finished reading K(i), and P.V(i - 2), committed before it, V(i - 2)
                    mbar_arrive(k_empty(gi % NSK));
                    if (gi >= 2)
                        mbar_arrive(v_empty((gi - 2) % NSV));
                }
                if (ok) {
                    fence_after();
                    if (half)
                        pass(std::integral_constant<int, 64>{}, pi, gi, 64 * hr, j0, hi);
                    else
                        pass(std::integral_constant<int, 128>{}, pi, gi, 0, j0, hi);
                } else {  // no computing, but the hand-over of the maximum still pairs up
                    if (pi > 0)
                        named_bar(bar_get, 64);
                    if (pi + 1 < t.np)
                        named_arrive(bar_put, 64);
                }
                store_one();  // the previous item's output, a chunk after each pass
            }
            while (pend > 0)
                store_one();
            // the next item, and its first entry for this parity, before this item's epilogue
            const uint32_t g0 = g;
            g += t.np;
            const TileInfo tn = ii_n < n_items ? tile_from(p, unit(ii_n), rn) : TileInfo{};
            raw_next = ii_n < n_items ? entry_of(tn, ii_n / p.tiles_total, (g & 1) == x ? 0u : 1u) : 0u;
            // the next item's Q into TMEM now, so that its first products overlap this item's epilogue
            q_in = tn.np > 0;
            if (q_in)
                copy_q();
            if (ok && t.np > 0) {  // O is final once the item's last P.V has landed
                const uint32_t xl = (g0 + t.np - 1) & 1;
                ok = __all_sync(0xffffffffu, mbar_wait(o_done(xl), nd(xl) & 1, S_WAIT_LIMIT));
                fence_after();
            }
            if (t.np > 0) {  // the parities with a pass in this item
                nd0 += (g0 & 1) == 0 || t.np > 1;
                nd1 += (g0 & 1) == 1 || t.np > 1;
            }
            // The row's sum: this thread's share and the other parity's thread's, each relative to the maximum
            // it last saw (the larger of the two is the row's final maximum); this thread stores output columns
            // [64 x, 64 x + 64).
            stat[x * 128 + row] = make_float2(mref, l);
            named_bar(bar_epi, 64);
            const float2 s0 = stat[row], s1 = stat[128 + row];
            const float M = fmaxf(s0.x, s1.x);
            const float L = M == -INFINITY ? 0.0f
                                           : (s0.x == -INFINITY ? 0.0f : s0.y * ex2(s0.x - M)) +
                                                 (s1.x == -INFINITY ? 0.0f : s1.y * ex2(s1.x - M));
            const bool has = ok && t.np > 0 && M != -INFINITY;
            p_inv = (L > 0.0f ? 1.0f / L : 0.0f) * vscale;
            p_orow = uint64_t(dst) * p.width + uint64_t(h) * SD + 64 * x;
            // identity rows and fp32 o: the warp stores its rows by TMA (rows past n_q are clipped by the tensor
            // map); a cube tile's half past the last cube belongs to another tile and is not written
            p_tma = p.use_tma_out && t.active && (!t.cube || t.cube_id[hr] < p.n_cubes);
            p_store = store;
            p_col = h * SD + 64 * x;
            p_row = t.row0 + 32 * qd;
            // warp-collective loads; an item without passes leaves an older item's values, replaced by zeros.
            // The first chunk is stored now, the second after this thread's next pass.
            {
                uint32_t pa[32], pb[32];
                tmem_ld32(tl + COL_O + 64 * x, pa);
                tmem_ld32(tl + COL_O + 64 * x + 32, pb);
                tmem_wait_ld();
                reg_fence(pa);
                reg_fence(pb);
#pragma unroll
                for (int e = 0; e < 32; ++e)
                    pb[e] = has ? pb[e] : 0u;
                tmem_st32(tl + COL_SPARE + 32 * x, pb);  // kept in TMEM until after this thread's next pass
                tmem_wait_st();
                // O is free for the next item once both threads of every row are here
                fence_before();
                named_bar(bar_epi, 64);
                fence_after();
#pragma unroll
                for (int e = 0; e < 32; ++e)
                    pa[e] = has ? pa[e] : 0u;
                store_chunk(0, pa);
            }
            pend = 1;
            ii = ii_n;
            t = tn;
        }
        while (pend > 0)
            store_one();
        if (!ok && lane == 0)
            atomicExch(p.err, 13);
        if (lane == 0)
            bulk_wait0();  // this warp's output boxes have landed
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

cudaError_t launch_attn_tc_sparse(const AttnParams& a, int dtype, bool sel_i32, const void* v16, const float* vinv,
                                  int* err, cudaStream_t st)
{
    if (a.n_q == 0 || a.heads == 0)
        return cudaSuccess;
    SpParams p;
    const bool bf = dtype == kBF16;
    if (!tile_map(&p.tk, a.k, bf, SD, a.k_pad, a.kv_heads, 64) ||
        !tile_map(&p.tv, bf ? v16 : a.v, false, SD, a.k_pad, a.kv_heads, 64) ||
        !tile_map(&p.tq, a.q, bf, SD, a.q_pad, a.heads, 128))
        return cudaErrorInvalidValue;
    p.q = a.q;
    p.o = a.o;
    p.use_tma_out = 0;
    if (a.o_type == 0 && !a.map) {  // identity rows, fp32: the epilogue stores by TMA
        auto enc = tensor_map_encoder();
        if (!enc)
            return cudaErrorInvalidValue;
        cuuint64_t dims[2] = {a.width, a.n_q};
        cuuint64_t strides[1] = {uint64_t(a.width) * 4};
        cuuint32_t box[2] = {16, 32};
        cuuint32_t estr[2] = {1, 1};
        if (enc(&p.to, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, a.o, dims, strides, box, estr,
                CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_64B, CU_TENSOR_MAP_L2_PROMOTION_NONE,
                CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
            return cudaErrorInvalidValue;
        p.use_tma_out = 1;
    }
    p.err = err;
    p.vinv = bf ? vinv : nullptr;
    p.sel = a.sel;
    p.nsel = a.nsel;
    p.valid = a.valid;
    p.map = a.map;
    p.sel_i32 = sel_i32 ? 1u : 0u;
    p.qk_fmt = bf ? 1u : 0u;
    p.o_type = a.o_type;
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
    if (p.tiles_total == 0)
        return cudaSuccess;
    const uint32_t n_items = p.tiles_total * a.heads, sms = a.num_sms ? a.num_sms : 148;
    attn_tc_sparse_kernel<<<n_items < sms ? n_items : sms, SNT, S_TOTAL, st>>>(p);
    return cudaGetLastError();
}

} // namespace mako
