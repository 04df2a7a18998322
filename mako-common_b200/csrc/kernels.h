// Internal launch interface between the C ABI (mako_attn.cu) and the kernels.  Plain structs, device pointers.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

namespace mako {

enum Dtype : int { kF16 = 0, kBF16 = 1 };

// This thread's message for mako_attn_last_error(): set_error formats it and returns `code`.
int set_error(int code, const char* fmt, ...);
void clear_error();

// One attention launch: the fields of the reference's AttnArgs (src/kernels/ops.metal:54-64) plus, for the
// block-sparse form, those of SparseAttnArgs (ops.metal:1029-1034) and its index buffers.
struct AttnParams {
    const void* q;  // [heads][q_pad][dim]
    const void* k;  // [kv_heads][k_pad][dim]
    const void* v;  // [kv_heads][k_pad][dim]
    float* o;       // [rows][width], head h at column h * dim
    uint32_t n_q, q_pad, n_k, k_pad, heads, kv_heads, q_pos0, block, width;
    float scale;  // softmax scale (1 / sqrt(dim))
    // block-sparse pass list
    uint32_t n_cubes, max_sel, dense0, dense1;
    const void* sel;       // [heads][n_cubes][max_sel] uint16 (cube_select) or int32 (kept-block lists)
    const void* nsel;      // [heads][n_cubes], same integer type as sel
    const uint8_t* valid;  // [k_pad] key validity, null: every key valid
    const int32_t* map;    // [q_pad] output row per query row (< 0 dropped), null: identity
    // Output destinations of the head-sharded form (tcgen05 dense kernel only): the same rows are stored into
    // od[0 .. n_od) (this rank's o and the peers' mapped o), local head h at column (head0 + h) * dim.  n_od == 0:
    // the single destination `o` at column h * dim.
    float* od[8];
    uint32_t n_od, head0;
    uint32_t o_type;  // element type of o: 0 fp32, 1 fp16, 2 bf16 (single-destination forms)
    uint32_t num_sms;  // SMs of the device (the persistent kernels' grid); 0: 148
};

// Portable flash attention on mma.sync tensor cores, any head width of 64 / 128 / 256.
cudaError_t launch_attn_mma(const AttnParams& p, int dtype, int dim, bool sparse, bool sel_i32, cudaStream_t s);

// Flash attention for 64- or 128-wide heads (dim) on sm_100a (tcgen05 / TMEM / TMA); the head-sharded form (n_od > 1)
// for 128-wide heads.  bf16 inputs need v16 / vinv from launch_v_to_f16; err receives a nonzero code if a pipeline
// wait timed out.
cudaError_t launch_attn_tc(const AttnParams& p, int dtype, int dim, const void* v16, const float* vinv, int* err,
                           cudaStream_t s);
// Flash attention for 256-wide heads on sm_100a: one 128-row tile per CTA, 64-key K / V tiles.  bf16 inputs need
// v16 / vinv from launch_v_to_f16 (dim 256).
cudaError_t launch_attn_tc256(const AttnParams& p, int dtype, const void* v16, const float* vinv, int* err,
                              cudaStream_t s);
// Block-sparse attention for 128-wide heads on sm_100a: two query cubes per 128-row UMMA tile, their key-cube lists
// walked in lockstep.  bf16 inputs need v16 / vinv (launch_v_to_f16 over all k_pad rows with the valid mask).
cudaError_t launch_attn_tc_sparse(const AttnParams& p, int dtype, bool sel_i32, const void* v16, const float* vinv,
                                  int* err, cudaStream_t s);
// v16 = fp16(v * 2^k) per kv head and vinv = 2^-k, for [kv_heads][k_pad][dim] tiles: k = 0 when the head's max |v|
// over rows < n_rows with valid[row] lies in [2^-3, 2^16) (one read of v, one write of v16), else k puts it in
// [2^14, 2^15) (that head converted again); other rows 0.  vmax: [kv_heads] scratch.
cudaError_t launch_v_to_f16(const void* v, void* v16, uint32_t* vmax, float* vinv, uint32_t dim, uint32_t kv_heads,
                            uint32_t k_pad, uint32_t n_rows, const uint8_t* valid, int num_sms, cudaStream_t s);

// Split-KV decode: one query row per (sequence, head) over keys [0, len).
struct DecodeParams {
    const void* q;  // query row of (b, h) at q + b * q_bstride + h * q_hstride
    const void* k;  // key row j of (b, kvh) at k + b * k_bstride + kvh * k_hstride + j * dim
    const void* v;  // as k
    float* o;       // output of (b, h) at o + b * o_bstride + h * dim
    float* o_part;  // scratch [batch][heads][n_splits][dim]
    float2* ml_part;  // scratch [batch][heads][n_splits]: (max in log2 units, sum)
    const int32_t* kv_len;  // device [batch] lengths, or null: `len` for every sequence
    uint32_t len;           // kv_len null: every sequence's length; else the cap (max_kv_len): no key past it is read
    uint64_t q_bstride, q_hstride, k_bstride, k_hstride, o_bstride;  // in elements
    uint32_t batch, heads, kv_heads, chunk, n_splits;
    float scale;
    uint32_t keep_partials;  // 1: always write partials (the KV-sharded combine reads them), never o
    uint32_t o_type;         // element type of o: 0 fp32, 1 fp16, 2 bf16
};
// Keys a split takes and how many splits, for the longest sequence max_len (chunk_opt: 0 automatic, else the
// requested multiple of 64).
void decode_plan(uint32_t max_len, uint32_t batch, uint32_t kv_heads, uint32_t heads, int num_sms, uint32_t chunk_opt,
                 uint32_t* chunk, uint32_t* n_splits);
cudaError_t launch_decode(const DecodeParams& p, int dtype, int dim, cudaStream_t s);

// Head-tile producers: y [heads][n_pad][dim] 16-bit, row row0 + r from x row map[r] (or r): head h's values at
// x + row * ld + col0 + h * stride, RMS-normed times w when eps > 0, rotated when rope is 1 (halves i, i + rot / 2 over
// the first rot values) or 2 (adjacent pairs over the whole head) by the (cos, sin) pairs cs + row * cs_row.
struct HeadsParams {
    const float* x;
    const float* cs;   // float2 pairs
    const float* w;    // [dim], when eps > 0
    const int32_t* map;  // [rows] or null; < 0: a zero row
    void* y;
    uint64_t ld;
    uint32_t col0, stride, dim, rot, rope, rows, heads, n_pad, row0, cs_row, vec4;
    float eps;
};
cudaError_t launch_heads(const HeadsParams& p, int dtype, cudaStream_t s);

// ---- multi-GPU exchange (one process per GPU, peers' memory mapped through CUDA IPC) ------------------------------

constexpr uint32_t kMaxRanks = 8;
constexpr uint32_t kXchgStride = 260;  // floats per exchanged decode row: o[dim <= 256], max, sum, 2 pad
// Layout of a rank's exchange area (bytes from its base):
//   0     barrier flags u32 [2 parities][2 kinds (enter, done)][kMaxRanks]
//   256   decode row flags u32 [2][kMaxRanks][rows_cap]
//   xoff  decode rows f32 [2][kMaxRanks][rows_cap][kXchgStride], xoff = 256 + 2 * kMaxRanks * rows_cap * 4 rounded
//         up to 256
__host__ __device__ inline uint64_t xchg_rows_offset(uint32_t rows_cap) { return (256 + uint64_t(2) * kMaxRanks * rows_cap * 4 + 255) / 256 * 256; }
__host__ __device__ inline uint64_t xchg_bytes(uint32_t rows_cap)
{
    return xchg_rows_offset(rows_cap) + uint64_t(2) * kMaxRanks * rows_cap * kXchgStride * 4;
}

struct XchgParams {
    unsigned char* area[kMaxRanks];  // every rank's exchange area as this process addresses it (area[rank]: own)
    uint32_t n_ranks, rank, epoch, rows_cap;
    int* err;
};
// Every rank signals the others and waits (bounded) until all have signalled `epoch` for barrier `kind`
// (0 enter, 1 done); stream-ordered: work before it on every rank happens before work after it on any rank.
cudaError_t launch_group_barrier(const XchgParams& x, uint32_t kind, cudaStream_t s);
// KV-sharded decode, second half: merges this rank's splits per (sequence, head), pushes the row to every rank's
// area, waits for all ranks' rows and merges them by log-sum-exp into o.
cudaError_t launch_decode_xchg(const DecodeParams& p, const XchgParams& x, int dim, cudaStream_t s);
// The two kernels of launch_decode one at a time: the splits (partials, or o for one-split sequences unless
// p.keep_partials), then the log-sum-exp combine (a programmatic dependent of the split kernel).
cudaError_t launch_decode_split(const DecodeParams& p, int dtype, int dim, cudaStream_t s);
cudaError_t launch_decode_combine(const DecodeParams& p, int dim, cudaStream_t s);

// cube_select: pooled means, their scores, the top k per (head, query cube).
struct CubeParams {
    const void* q;
    const void* k;
    const uint32_t* cnt;
    float* qp;  // scratch [heads][n_cubes][128]
    float* kp;  // scratch [heads][n_cubes][128]
    float* sc;  // scratch [heads][n_cubes][n_cubes]
    uint16_t* sel;   // [heads][n_cubes][min(topk, n_cubes)]
    uint16_t* nsel;  // [heads][n_cubes]
    uint32_t heads, q_pad, k_pad, n_cubes, topk, local, stride;
};
cudaError_t launch_cube_select(const CubeParams& p, int dtype, cudaStream_t s);

// The output projection after the attention: y[t][j] = sum_i x[t][i] w[j][i], x [T][k] and w [n][k] 16-bit (one type),
// y [T][ldy] fp32; k a multiple of 64.
struct ProjParams {
    const void* x;
    const void* w;
    float* y;
    uint32_t T, k, n, ldy, num_sms;
};
cudaError_t launch_proj_gemm(const ProjParams& p, int dtype, int* err, cudaStream_t s);

} // namespace mako
