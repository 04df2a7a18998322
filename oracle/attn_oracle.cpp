// CPU oracle for the attention hot path -- TEST INFRASTRUCTURE ONLY.
//
// This file is the checker, never the product: only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline
// leg (and its `--impl reference` arm) may load the library built from it.  The CUDA path in mako-common_b200/
// never calls it.
//
// It restates, in double precision, the scalar C++ attention that mako-common's own test uses as its reference
// (tests/sparse_attn_test.cpp:98-182), generalised to the mask rules of the Metal kernels it checks:
//   * dense / causal / "block" mask predicate .......... src/kernels/ops.metal:161,289 (AttnArgs :54-64)
//   * per-row key set, dot in double, scale in float ... tests/sparse_attn_test.cpp:133,143-173
//   * rows with no visible key give zeros .............. src/kernels/ops.metal:194,355 (l == 0 -> inv 0)
//   * block-sparse pass list, valid mask, output map ... src/kernels/ops.metal:1079-1110,1174-1184
//   * cube pooling / scores / top-k incl. `local` ....... src/kernels/ops.metal:927-1027,
//                                                         tests/sparse_attn_test.cpp:103-128,184-208
// Inputs arrive as the raw 16-bit patterns the device reads (fp16 or bf16) and are widened exactly.
//
// Parity pin: the reference cannot be built here (Metal only), so the pins are the reference test's own
// procedure re-run on its own fixture (oracle_sparse_test_fixture below re-creates tests/sparse_attn_test.cpp:46-77
// with libstdc++'s std::normal_distribution) plus an independent numpy restatement in tests/.
#include <algorithm>
#include <cmath>
#include <cstdint>
#include <cstring>
#include <random>
#include <vector>

#ifdef _OPENMP
#include <omp.h>
#endif

namespace {

// Every fp16 bit pattern's value (exact), so widening is a table read rather than a software conversion.
struct F16Table {
    float v[65536];
    F16Table()
    {
        for (uint32_t i = 0; i < 65536; ++i) {
            const uint16_t b = uint16_t(i);
            _Float16 h;
            std::memcpy(&h, &b, 2);
            v[i] = float(h);
        }
    }
};
const F16Table kF16;

// 0: IEEE fp16, 1: bfloat16.
inline double widen(uint16_t bits, int dtype)
{
    if (dtype == 1) {
        const uint32_t u = uint32_t(bits) << 16;
        float f;
        std::memcpy(&f, &u, 4);
        return f;
    }
    return kF16.v[bits];
}

inline float widen_f(uint16_t bits, int dtype) { return float(widen(bits, dtype)); }

// Key j is visible to the query at position pos (src/kernels/ops.metal:161,289).
inline bool visible(uint32_t j, uint32_t pos, uint32_t n_k, uint32_t block)
{
    return j < n_k && (j <= pos || (pos >= block && j >= block));
}

// softmax(scale * q.k) . v over `keys` for one query row, in double; zeros when there is no key
// (tests/sparse_attn_test.cpp:156-173; src/kernels/ops.metal:355 for the empty case).
void attend_row(const uint16_t* qrow, const uint16_t* khead, const uint16_t* vhead, const std::vector<uint32_t>& keys,
                uint32_t dim, float scale, int dtype, float* out)
{
    if (keys.empty()) {
        for (uint32_t d = 0; d < dim; ++d)
            out[d] = 0.0f;
        return;
    }
    std::vector<double> qd(dim), w(keys.size()), ref(dim, 0.0);
    for (uint32_t d = 0; d < dim; ++d)
        qd[d] = widen(qrow[d], dtype);
    double mx = -1e300;
    for (size_t i = 0; i < keys.size(); ++i) {
        const uint16_t* kr = khead + uint64_t(keys[i]) * dim;
        double s = 0;
        for (uint32_t d = 0; d < dim; ++d)
            s += qd[d] * widen(kr[d], dtype);
        w[i] = s * scale;
        mx = std::max(mx, w[i]);
    }
    double sum = 0;
    for (double& x : w) {
        x = std::exp(x - mx);
        sum += x;
    }
    for (size_t i = 0; i < keys.size(); ++i) {
        const uint16_t* vr = vhead + uint64_t(keys[i]) * dim;
        const double p = w[i] / sum;
        for (uint32_t d = 0; d < dim; ++d)
            ref[d] += p * widen(vr[d], dtype);
    }
    for (uint32_t d = 0; d < dim; ++d)
        out[d] = float(ref[d]);
}

int set_threads(int threads)
{
#ifdef _OPENMP
    if (threads > 0)
        omp_set_num_threads(threads);
    return omp_get_max_threads();
#else
    (void)threads;
    return 1;
#endif
}

} // namespace

extern "C" {

// Threads the OpenMP loops use (threads <= 0: the library default).
int oracle_threads(int threads) { return set_threads(threads); }

// Dense masked attention (TransformerRuntime::attention, src/models/runtime.cpp:262-273): q [heads][q_pad][dim],
// k/v [kv_heads][k_pad][dim] (16-bit patterns), o [n_q][width] floats at column h*dim; head h reads kv head
// h / (heads / kv_heads).  rows: the query rows to compute (null: all n_q), n_rows of them.
void oracle_attention(int dtype, const uint16_t* q, const uint16_t* k, const uint16_t* v, float* o, uint32_t n_q,
                      uint32_t q_pad, uint32_t n_k, uint32_t k_pad, uint32_t heads, uint32_t kv_heads, uint32_t q_pos0,
                      uint32_t block, uint32_t dim, uint32_t width, const uint32_t* rows, uint32_t n_rows, int threads)
{
    set_threads(threads);
    const float scale = 1.0f / std::sqrt(float(dim));
    const uint32_t nr = rows ? n_rows : n_q;
    const int64_t total = int64_t(nr) * heads;
#pragma omp parallel for schedule(dynamic, 4)
    for (int64_t t = 0; t < total; ++t) {
        const uint32_t h = uint32_t(t / nr), i = rows ? rows[t % nr] : uint32_t(t % nr);
        if (i >= n_q)
            continue;
        const uint32_t kvh = h / (heads / kv_heads), pos = q_pos0 + i;
        std::vector<uint32_t> keys;
        keys.reserve(n_k);
        for (uint32_t j = 0; j < n_k; ++j)
            if (visible(j, pos, n_k, block))
                keys.push_back(j);
        attend_row(q + (uint64_t(h) * q_pad + i) * dim, k + uint64_t(kvh) * k_pad * dim,
                   v + uint64_t(kvh) * k_pad * dim, keys, dim, scale, dtype, o + uint64_t(i) * width + uint64_t(h) * dim);
    }
}

// One query per sequence over its whole cache: attention() with n_q = 1, q_pos0 = len - 1, causal.  q [batch][heads]
// [dim], k/v [batch][kv_heads][k_stride][dim], o [batch][heads * dim]; kv_len per sequence (host).
void oracle_decode(int dtype, const uint16_t* q, const uint16_t* k, const uint16_t* v, float* o, uint32_t batch,
                   const int32_t* kv_len, uint32_t heads, uint32_t kv_heads, uint32_t dim, uint32_t k_stride,
                   int threads)
{
    set_threads(threads);
    const float scale = 1.0f / std::sqrt(float(dim));
    const int64_t total = int64_t(batch) * heads;
#pragma omp parallel for schedule(dynamic, 1)
    for (int64_t t = 0; t < total; ++t) {
        const uint32_t b = uint32_t(t / heads), h = uint32_t(t % heads), kvh = h / (heads / kv_heads);
        const uint32_t len = kv_len[b] > 0 ? uint32_t(kv_len[b]) : 0;
        std::vector<uint32_t> keys(len);
        for (uint32_t j = 0; j < len; ++j)
            keys[j] = j;
        const uint64_t kbase = (uint64_t(b) * kv_heads + kvh) * k_stride * dim;
        attend_row(q + (uint64_t(b) * heads + h) * dim, k + kbase, v + kbase, keys, dim, scale, dtype,
                   o + uint64_t(b) * heads * dim + uint64_t(h) * dim);
    }
}

// Block-sparse attention over 128-wide heads (flash_attn_sparse_128, src/kernels/ops.metal:1039-1185): a query row
// in tile qt = r / 64 < n_cubes sees the valid rows of each selected cube (an entry listed twice counts twice) and the
// valid rows of [dense0, dense1); a later row sees every valid key below n_k.  Row r's output goes to o row map[r],
// dropped when map[r] < 0.  sel [heads][n_cubes][max_sel], nsel [heads][n_cubes] (clamped to max_sel); cube entries
// >= n_cubes are skipped (the CUDA kernel does the same instead of reading out of range).
void oracle_attention_sparse(int dtype, const uint16_t* q, const uint16_t* k, const uint16_t* v, float* o,
                             uint32_t n_q, uint32_t q_pad, uint32_t n_k, uint32_t k_pad, uint32_t heads,
                             uint32_t kv_heads, uint32_t width, uint32_t n_cubes, uint32_t max_sel, uint32_t dense0,
                             uint32_t dense1, const uint16_t* sel, const uint16_t* nsel, const uint8_t* valid,
                             const int32_t* map, const uint32_t* rows, uint32_t n_rows, int threads)
{
    set_threads(threads);
    constexpr uint32_t D = 128;
    const float scale = 1.0f / std::sqrt(float(D));
    const uint32_t nr = rows ? n_rows : n_q;
    const int64_t total = int64_t(nr) * heads;
#pragma omp parallel for schedule(dynamic, 4)
    for (int64_t t = 0; t < total; ++t) {
        const uint32_t h = uint32_t(t / nr), r = rows ? rows[t % nr] : uint32_t(t % nr);
        if (r >= n_q || map[r] < 0)
            continue;
        const uint32_t kvh = h / (heads / kv_heads), qt = r / 64;
        std::vector<uint32_t> keys;
        if (qt < n_cubes) {
            const uint32_t ns = std::min<uint32_t>(nsel[uint64_t(h) * n_cubes + qt], max_sel);
            const uint16_t* s = sel + (uint64_t(h) * n_cubes + qt) * max_sel;
            for (uint32_t i = 0; i < ns; ++i) {
                if (s[i] >= n_cubes)
                    continue;
                for (uint32_t j = uint32_t(s[i]) * 64; j < uint32_t(s[i]) * 64 + 64; ++j)
                    if (valid[j])
                        keys.push_back(j);
            }
            for (uint32_t j = dense0; j < dense1; ++j)
                if (valid[j])
                    keys.push_back(j);
        } else {
            for (uint32_t j = 0; j < n_k; ++j)
                if (valid[j])
                    keys.push_back(j);
        }
        attend_row(q + (uint64_t(h) * q_pad + r) * D, k + uint64_t(kvh) * k_pad * D, v + uint64_t(kvh) * k_pad * D,
                   keys, D, scale, dtype, o + uint64_t(map[r]) * width + uint64_t(h) * D);
    }
}

// cube_select (src/models/runtime.cpp:286-303): pooled means per 64-row cube, their dot products, the top k per
// (head, query cube).  mode 0: in double (tests/sparse_attn_test.cpp:104-118); mode 1: the fp32 order the CUDA kernels
// use -- a sequential sum over the cube's 64 rows then one division by cnt (ops.metal:935-938), and per score
// s += ((q0 k0 + q1 k1) + q2 k2) + q3 k3 over d in fours (ops.metal:952-953), unfused (built with
// -ffp-contract=off).  Both select the same way as cube_topk (ops.metal:970-1025): the local cubes first (qc, then
// qc - stride and qc + stride when inside), their scores then out of the running; then repeatedly the largest score,
// ties to the smaller index, index 0 when none is above -inf.  sel [heads][n_cubes][k], nsel [heads][n_cubes] with
// k = min(topk, n_cubes).  qp/kp ([heads][n_cubes][128]) and sc ([heads][n_cubes][n_cubes]) receive the fp32 values in
// mode 1 when non-null.
void oracle_cube_select(int dtype, const uint16_t* q, const uint16_t* k, uint32_t heads, uint32_t q_pad,
                        uint32_t k_pad, uint32_t n_cubes, const uint32_t* cnt, uint32_t topk, uint32_t local,
                        uint32_t stride, int mode, uint16_t* sel, uint16_t* nsel, float* qp_out, float* kp_out,
                        float* sc_out)
{
    constexpr uint32_t D = 128;
    const uint32_t kk = std::min(topk, n_cubes);
    for (uint32_t h = 0; h < heads; ++h) {
        std::vector<double> qp(uint64_t(n_cubes) * D), kp(qp.size()), sc(uint64_t(n_cubes) * n_cubes);
        for (int which = 0; which < 2; ++which) {
            const uint16_t* x = which ? k : q;
            const uint32_t pad = which ? k_pad : q_pad;
            std::vector<double>& out = which ? kp : qp;
            float* fout = which ? kp_out : qp_out;
            for (uint32_t c = 0; c < n_cubes; ++c)
                for (uint32_t d = 0; d < D; ++d) {
                    const uint16_t* p = x + (uint64_t(h) * pad + uint64_t(c) * 64) * D + d;
                    double val;
                    if (mode == 0) {
                        double s = 0;
                        for (uint32_t r = 0; r < 64; ++r)
                            s += widen(p[uint64_t(r) * D], dtype);
                        val = cnt[c] ? s / cnt[c] : 0.0;
                    } else {
                        float s = 0.0f;
                        for (uint32_t r = 0; r < 64; ++r)
                            s += widen_f(p[uint64_t(r) * D], dtype);
                        const float f = cnt[c] ? s / float(cnt[c]) : 0.0f;
                        if (fout)
                            fout[(uint64_t(h) * n_cubes + c) * D + d] = f;
                        val = f;
                    }
                    out[uint64_t(c) * D + d] = val;
                }
        }
#pragma omp parallel for schedule(static)
        for (uint32_t qc = 0; qc < n_cubes; ++qc)
            for (uint32_t kc = 0; kc < n_cubes; ++kc) {
                const double* a = &qp[uint64_t(qc) * D];
                const double* b = &kp[uint64_t(kc) * D];
                double val;
                if (mode == 0) {
                    double s = 0;
                    for (uint32_t d = 0; d < D; ++d)
                        s += a[d] * b[d];
                    val = s;
                } else {
                    float s = 0.0f;
                    for (uint32_t d = 0; d < D; d += 4) {
                        float t = float(a[d]) * float(b[d]);
                        t = t + float(a[d + 1]) * float(b[d + 1]);
                        t = t + float(a[d + 2]) * float(b[d + 2]);
                        t = t + float(a[d + 3]) * float(b[d + 3]);
                        s = s + t;
                    }
                    if (sc_out)
                        sc_out[(uint64_t(h) * n_cubes + qc) * n_cubes + kc] = s;
                    val = s;
                }
                sc[uint64_t(qc) * n_cubes + kc] = val;
            }
#pragma omp parallel for schedule(dynamic, 16)
        for (uint32_t qc = 0; qc < n_cubes; ++qc) {
            std::vector<double> s(sc.begin() + uint64_t(qc) * n_cubes, sc.begin() + uint64_t(qc + 1) * n_cubes);
            uint16_t* out = sel + (uint64_t(h) * n_cubes + qc) * kk;
            uint32_t it = 0;
            if (local) {
                const uint32_t picks[3] = {qc, qc >= stride ? qc - stride : n_cubes,
                                           qc + stride < n_cubes ? qc + stride : n_cubes};
                for (uint32_t j = 0; j < local && it < kk; ++j)
                    if (picks[j] < n_cubes) {
                        out[it++] = uint16_t(picks[j]);
                        s[picks[j]] = -INFINITY;
                    }
            }
            for (; it < kk; ++it) {
                double best = -INFINITY;
                uint32_t bi = 0;
                for (uint32_t i = 0; i < n_cubes; ++i)
                    if (s[i] > best) {
                        best = s[i];
                        bi = i;
                    }
                out[it] = uint16_t(bi);
                s[bi] = -INFINITY;
            }
            nsel[uint64_t(h) * n_cubes + qc] = uint16_t(kk);
        }
    }
}

// The fixture of tests/sparse_attn_test.cpp:46-86 re-created: D 128, 2 heads, 6 cubes with cnt {64,64,64,64,64,20},
// 60 dense rows (n 444, q_pad 448, k_pad 512), std::mt19937(7) with std::normal_distribution<float> drawn in the
// test's order (q, then k, then v; per head, per row below k_pad, per d; a draw only for valid rows), rounded to
// fp16.  q [2][448][128], k/v [2][512][128], valid [512], map [448] (identity on valid rows, -1 elsewhere),
// cnt [6].  The values follow libstdc++'s normal_distribution; libc++ (the reference's macOS build) draws others.
void oracle_sparse_test_fixture(uint16_t* q, uint16_t* k, uint16_t* v, uint8_t* valid, int32_t* map, uint32_t* cnt)
{
    constexpr uint32_t D = 128, heads = 2, cubes = 6, dense = 60;
    const uint32_t cnts[cubes] = {64, 64, 64, 64, 64, 20};
    const uint32_t n = cubes * 64 + dense, q_pad = (n + 63) / 64 * 64, k_pad = (n + 127) / 128 * 128;
    const uint32_t dense0 = cubes * 64, dense1 = n;
    std::memcpy(cnt, cnts, sizeof(cnts));
    std::fill_n(valid, k_pad, uint8_t(0));
    std::fill_n(map, q_pad, -1);
    for (uint32_t c = 0; c < cubes; ++c)
        for (uint32_t r = 0; r < cnts[c]; ++r)
            valid[c * 64 + r] = 1;
    for (uint32_t r = dense0; r < dense1; ++r)
        valid[r] = 1;
    for (uint32_t r = 0; r < n; ++r)
        if (valid[r])
            map[r] = int32_t(r);
    std::mt19937 rng(7);
    std::normal_distribution<float> nd;
    uint16_t* bufs[3] = {q, k, v};
    const uint32_t pads[3] = {q_pad, k_pad, k_pad};
    for (int b = 0; b < 3; ++b)
        for (uint32_t hh = 0; hh < heads; ++hh)
            for (uint32_t r = 0; r < k_pad; ++r)
                for (uint32_t d = 0; d < D; ++d) {
                    const _Float16 x = _Float16(valid[r] ? nd(rng) : 0.0f);
                    if (r < pads[b])
                        std::memcpy(&bufs[b][(uint64_t(hh) * pads[b] + r) * D + d], &x, 2);
                }
}

// Head-tile producers (TransformerRuntime::heads / heads_norm / heads_partial, src/models/runtime.cpp:215-260):
// restates heads_half (src/kernels/ops.metal:21-43), heads_norm_half (:371-408) and heads_partial (:577-613) in
// double.  y row row0 + r of head h takes x row map[r] (or r; a zero row where map[r] < 0) at col0 + h * stride:
// RMS-normed over the head times w when eps > 0 (x / sqrt(sum(x^2) / dim + eps) * w[d]), then rotated when rope is
// 1 (halves: i with i + rot / 2 over the first rot values, pair i % (rot / 2)) or 2 (adjacent pairs 2i, 2i + 1 over
// the whole head, pair i) by the (cos, sin) pairs cs + t * cs_row: u' = u c - v s, v' = v c + u s.  y receives the
// values before 16-bit rounding, [heads][n_pad][dim]; other rows are left as they are.
void oracle_heads(const float* x, uint64_t ld, uint32_t col0, uint32_t stride, uint32_t dim, uint32_t rot,
                  uint32_t rope, uint32_t rows, uint32_t heads, uint32_t n_pad, uint32_t row0, const float* cs,
                  uint32_t cs_row, const float* w, float eps, const int32_t* map, float* y)
{
    std::vector<double> v(dim), o(dim);
    for (uint32_t h = 0; h < heads; ++h)
        for (uint32_t r = 0; r < rows; ++r) {
            float* yr = y + (uint64_t(h) * n_pad + row0 + r) * dim;
            const int64_t t = map ? int64_t(map[r]) : int64_t(r);
            if (t < 0) {
                std::fill(yr, yr + dim, 0.0f);
                continue;
            }
            const float* xr = x + uint64_t(t) * ld + col0 + uint64_t(h) * stride;
            for (uint32_t i = 0; i < dim; ++i)
                v[i] = xr[i];
            if (eps > 0.0f) {
                double ss = 0.0;
                for (uint32_t i = 0; i < dim; ++i)
                    ss += v[i] * v[i];
                const double inv = 1.0 / std::sqrt(ss / dim + double(eps));
                for (uint32_t i = 0; i < dim; ++i)
                    v[i] *= inv * double(w[i]);
            }
            o = v;
            const float* c = cs ? cs + uint64_t(t) * cs_row * 2 : nullptr;
            if (rope == 2) {
                for (uint32_t i = 0; i + 1 < dim; i += 2) {
                    const double cc = c[i], sn = c[i + 1];  // pair i / 2 at floats 2 (i / 2), 2 (i / 2) + 1
                    o[i] = v[i] * cc - v[i + 1] * sn;
                    o[i + 1] = v[i + 1] * cc + v[i] * sn;
                }
            } else if (rope == 1 && rot) {
                const uint32_t half = rot / 2;
                for (uint32_t i = 0; i < half; ++i) {
                    const double cc = c[2 * i], sn = c[2 * i + 1];
                    o[i] = v[i] * cc - v[i + half] * sn;
                    o[i + half] = v[i + half] * cc + v[i] * sn;
                }
            }
            for (uint32_t i = 0; i < dim; ++i)
                yr[i] = float(o[i]);
        }
}

// The output projection (Runtime::proj on a 16-bit matrix, src/gpu/runtime.cpp:164-190): y[t][j] = sum_i x[t][i]
// w[j][i] in double over the 16-bit x [T][k] and w [n][k] (x is what the reference's to_bf16 / to_half makes of the
// fp32 attention output), y [T][ldy] floats.  rows: the t to compute (null: all), n_rows of them.
void oracle_proj(int dtype, const uint16_t* w, const uint16_t* x, float* y, uint32_t T, uint32_t k, uint32_t n,
                 uint32_t ldy, const uint32_t* rows, uint32_t n_rows, int threads)
{
    set_threads(threads);
    const uint32_t nr = rows ? n_rows : T;
    std::vector<double> wd(uint64_t(n) * k);
    for (uint64_t i = 0; i < wd.size(); ++i)
        wd[i] = widen(w[i], dtype);
#pragma omp parallel for schedule(dynamic, 1)
    for (int64_t r = 0; r < int64_t(nr); ++r) {
        const uint32_t t = rows ? rows[r] : uint32_t(r);
        if (t >= T)
            continue;
        std::vector<double> xd(k);
        for (uint32_t i = 0; i < k; ++i)
            xd[i] = widen(x[uint64_t(t) * k + i], dtype);
        for (uint32_t j = 0; j < n; ++j) {
            const double* wr = &wd[uint64_t(j) * k];
            double s = 0;
            for (uint32_t i = 0; i < k; ++i)
                s += xd[i] * wr[i];
            y[uint64_t(t) * ldy + j] = float(s);
        }
    }
}

} // extern "C"
