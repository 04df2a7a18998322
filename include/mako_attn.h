/* mako_attn.h -- C ABI of the B200 (sm_100a) attention path for mako-common.
 *
 * This library replaces the attention slice of mako-common's Metal dispatch glue (src/gpu/runtime.{hpp,cpp},
 * src/mtl/) and kernels (src/kernels/ops.metal attention kernels).  Each entry point below names the reference
 * interface it replaces.  Conventions for every call:
 *   - pointers are CUDA device pointers (16-byte aligned) unless a comment says host;
 *   - `stream` is a cudaStream_t (NULL: the legacy default stream); calls only enqueue work, never synchronise;
 *   - tensors are owned by the caller; the context owns its scratch (like gpu::Runtime::scratch,
 *     src/gpu/runtime.cpp:117-125), so one context serves one thread / one stream at a time;
 *   - the return value is MAKO_OK or a negative code; mako_attn_last_error() gives this thread's message for the
 *     last failure.  Argument errors are reported before anything is enqueued (the reference throws
 *     std::runtime_error at the same points: src/models/runtime.cpp:266-267,290-291,311-312).
 * Element types: MAKO_F16 (IEEE half, the reference's `half` tiles) or MAKO_BF16.  Outputs are fp32 as in the
 * reference (o [n_q][width] floats, head h at column h * dim), or the call's 16-bit type under
 * MAKO_OPT_OUTPUT_16BIT.
 */
#ifndef MAKO_ATTN_H
#define MAKO_ATTN_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define MAKO_ATTN_VERSION 1

enum { MAKO_F16 = 0, MAKO_BF16 = 1 };

enum {
    MAKO_OK = 0,
    MAKO_EINVAL = -22,  /* an argument the call cannot take */
    MAKO_ENOMEM = -12,  /* scratch allocation failed */
    MAKO_ECUDA = -5,    /* a CUDA call failed (launch error, bad device) */
    MAKO_ENOTSUP = -95  /* a combination this build does not provide */
};

/* Options for mako_attn_set_option. */
enum {
    /* Dense and block-sparse attention kernels: 0 (default) and 2 the tcgen05 kernels, every head width
     * (MAKO_ENOTSUP on a device other than sm_100); 1 the mma.sync kernels, kept as the baseline that tests and
     * benchmarks compare against, never chosen automatically. */
    MAKO_OPT_PREFILL_KERNEL = 1,
    /* 1 (default): mako_attention with n_q == 1 runs the split-KV decode kernel; 0: the prefill kernel. */
    MAKO_OPT_DECODE_ROUTE = 2,
    /* Keys per split of the decode kernel: 0 (default) chooses from the longest sequence and the SM count; else a
     * multiple of 64 (raised when a sequence would need more than 1024 splits). */
    MAKO_OPT_DECODE_CHUNK = 3,
    /* 1: every call also records a CUDA event pair around its main kernel (the attention or split kernel, not the
     * bf16 V pre-pass, the decode combine or the group barriers) for mako_attn_kernel_times; 0 (default): none. */
    MAKO_OPT_KERNEL_TIMING = 4,
    /* 1: mako_attention, mako_attention_decode, mako_attention_sparse and mako_attention_block_sparse write o in the
     * call's 16-bit type (the values the reference's to_half / to_bf16 pass makes of its fp32 o before the output
     * projection, src/gpu/runtime.cpp:164-190), 2 bytes per value, `o` pointing at that storage; o row widths of the
     * prefill paths a multiple of 8.  0 (default): fp32 o.  The sharded forms keep fp32 (MAKO_ENOTSUP when set). */
    MAKO_OPT_OUTPUT_16BIT = 5,
    /* The persistent kernels' grid (tcgen05 dense and block-sparse attention, the output projection): 0 (default) one
     * CTA per SM; n > 0 at most n CTAs, each then working through more items -- for tests of the paths that carry
     * one item's state into the next on small problems. */
    MAKO_OPT_GRID_CTAS = 6
};

typedef struct mako_attn_ctx mako_attn_ctx;

/* This thread's message for its last failed call ("" if none). */
const char* mako_attn_last_error(void);
int mako_attn_version(void);

/* A context on CUDA device `device`: its scratch buffers and options.  Replaces gpu::Runtime's scratch and
 * pipeline cache (src/gpu/runtime.cpp:117-135); destroy frees the scratch (synchronising the device). */
int mako_attn_create(int device, mako_attn_ctx** out);
int mako_attn_destroy(mako_attn_ctx* ctx);
int mako_attn_set_option(mako_attn_ctx* ctx, int option, int64_t value);
/* Kernel launches this context has enqueued since it was created (a counter for profiling harnesses; the
 * reference's equivalent is its per-kernel telemetry, src/gpu/runtime.cpp:343-370). */
int mako_attn_launches(mako_attn_ctx* ctx, uint64_t* out);
/* Device time in milliseconds of each main kernel recorded since the last call (MAKO_OPT_KERNEL_TIMING), oldest
 * first: up to `cap` values into ms, their count into *n; waits for the recorded kernels to finish and forgets them.
 * A measurement hook for benchmarks; the reference's counterpart is its per-kernel GPU timestamps
 * (src/gpu/runtime.cpp:343-370). */
int mako_attn_kernel_times(mako_attn_ctx* ctx, float* ms, uint32_t cap, uint32_t* n);
/* Reads and clears the context's device error flag (synchronising the device): nonzero when a pipelined kernel gave
 * up on a wait (its bounded spin ran out) and left its outputs incomplete.  No reference counterpart: the reference
 * learns of a failed command buffer in gpu::Runtime::finish (src/gpu/runtime.cpp:466-471). */
int mako_attn_device_error(mako_attn_ctx* ctx, int* out);

/* Flash attention over 16-bit head tiles: q [heads][q_pad][dim], k and v [kv_heads][k_pad][dim] into
 * o [n_q][width] floats, head h at column h * dim and reading kv head h / (heads / kv_heads).  Key j is visible to
 * query i (position pos = q_pos0 + i) when j < n_k and (j <= pos or (pos >= block and j >= block)):
 * block = 0 bidirectional, block = UINT32_MAX causal.  dim 64, 128 or 256; width 0 means heads * dim.  Rows that
 * see no key are 0.  Padded key / value rows [n_k, k_pad) must hold finite values (the reference zeroes them).
 * Replaces TransformerRuntime::attention (src/models/runtime.hpp:90-95, src/models/runtime.cpp:262-273); the
 * reference computes width as heads * dim.  q_pad must be a multiple of 64 and at least n_q (the reference's grid,
 * q_pad / 64 tiles of 64 rows), k_pad at least n_k.  n_q == 1 runs the split-KV decode kernel. */
int mako_attention(mako_attn_ctx* ctx, void* stream, int dtype, const void* q, const void* k, const void* v, float* o,
                   uint32_t n_q, uint32_t q_pad, uint32_t n_k, uint32_t k_pad, uint32_t heads, uint32_t kv_heads,
                   uint32_t q_pos0, uint32_t block, uint32_t dim, uint32_t width);

/* Batched single-token decode over a KV cache of varying lengths: q [batch][heads][dim],
 * k and v [batch][kv_heads][k_stride][dim], kv_len [batch] int32 on the device (each at most max_kv_len and at most
 * k_stride), o [batch][heads * dim] floats.  Sequence b's query attends keys [0, kv_len[b]); a length <= 0 gives 0,
 * and a length above max_kv_len is read as max_kv_len (no key past it is read, every o row is still written).
 * No reference counterpart kernel: the reference's decode step is mako_attention's form with n_q = 1,
 * q_pos0 = len - 1, block = UINT32_MAX (src/models/runtime.cpp:262-273), looped over sequences by the caller. */
int mako_attention_decode(mako_attn_ctx* ctx, void* stream, int dtype, const void* q, const void* k, const void* v,
                          float* o, uint32_t batch, const int32_t* kv_len, uint32_t max_kv_len, uint32_t heads,
                          uint32_t kv_heads, uint32_t dim, uint32_t k_stride);

/* mako_attention_decode without any device allocation and without a context, for callers that cannot call
 * cudaMalloc: a process whose device memory is wholly committed elsewhere (a fixed pool it reserved up front, or
 * memory it borrowed under a lending protocol and must not grow beyond), or a loop that cannot afford
 * cudaMalloc / cudaFree synchronising the device.  No counterpart in the reference.
 * Same arguments and results as mako_attention_decode, on the current device.  The split partials live in one
 * file-scope device array of 4 MiB that every GPU loading this library holds until the process exits; the call
 * picks larger splits when needed so that they fit, and returns MAKO_EINVAL when even one split per sequence would
 * not (batch * heads * (4 * dim + 8) bytes above 4 MiB).  The first call on each device looks up the array's device
 * address (cudaGetSymbolAddress) and remembers it; make that first call before any stream capture, and do not call
 * it on a device again after cudaDeviceReset there (the remembered address belonged to the destroyed context).
 * Every call uses the same array, so calls that overlap on the GPU (other streams, other threads) race: serialise
 * them. */
int mako_attention_decode_noalloc(void* stream, int dtype, const void* q, const void* k, const void* v, float* o,
                                  uint32_t batch, const int32_t* kv_len, uint32_t max_kv_len, uint32_t heads,
                                  uint32_t kv_heads, uint32_t dim, uint32_t k_stride);

/* Cube selection for block-sparse attention over 128-wide heads: per head and query cube (64 rows), the `topk`
 * key cubes whose mean-pooled k scores highest against the cube's mean-pooled q (cnt[c]: valid rows of cube c,
 * device uint32 [n_cubes]; invalid rows must be zero).  local 0: by score; 1: the query cube itself first; 3: also
 * the cubes `stride` before and after.  *sel receives [heads][n_cubes][min(topk, n_cubes)] uint16 and *nsel
 * [heads][n_cubes] uint16, both device scratch owned by ctx and valid until its next mako_cube_select.
 * Replaces TransformerRuntime::cube_select (src/models/runtime.hpp:96-108, src/models/runtime.cpp:286-303):
 * n_cubes <= 4096, topk > 0, local in {0, 1, 3}; also n_cubes * 64 <= q_pad and <= k_pad. */
int mako_cube_select(mako_attn_ctx* ctx, void* stream, int dtype, const void* q, const void* k, uint32_t heads,
                     uint32_t q_pad, uint32_t k_pad, uint32_t n_cubes, const uint32_t* cnt, uint32_t topk,
                     uint16_t** sel, uint16_t** nsel, uint32_t local, uint32_t stride);

/* Block-sparse attention over 128-wide heads: query tile t < n_cubes (rows 64 t .. 64 t + 63) attends the valid
 * rows of its selected cubes (sel [heads][n_cubes][min(topk, n_cubes)], nsel [heads][n_cubes], as
 * mako_cube_select returns them; an entry listed twice counts twice, entries >= n_cubes are skipped) and the valid
 * rows of [dense0, dense1); a later tile attends every valid key below n_k.  valid [k_pad] uint8; query row r's
 * output goes to o row map[r] (map [q_pad] int32, < 0: dropped).  Replaces TransformerRuntime::attention_sparse
 * (src/models/runtime.hpp:109-111, src/models/runtime.cpp:305-317): q_pad a multiple of 64, k_pad of 128, dense0
 * of 32; also dense0 <= dense1 <= k_pad, n_cubes * 64 <= q_pad and <= k_pad, width >= heads * 128, valid 16-byte
 * aligned like the tensors (the kernel reads it 16 keys at a time). */
int mako_attention_sparse(mako_attn_ctx* ctx, void* stream, int dtype, const void* q, const void* k, const void* v,
                          float* o, uint32_t n_q, uint32_t q_pad, uint32_t n_k, uint32_t k_pad, uint32_t heads,
                          uint32_t kv_heads, uint32_t width, uint32_t n_cubes, uint32_t topk, uint32_t dense0,
                          uint32_t dense1, const uint16_t* sel, const uint16_t* nsel, const uint8_t* valid,
                          const int32_t* map);

/* The cube layout of MiniMax-H3's sparse attention (src/models/h3.cpp:510-546; host code, host arrays): the video
 * tokens of `frames` frames of ph x pw patches in 4 x 4 x 4 cubes of (frame, patch row, patch column), the grid padded
 * to multiples of 4 with rows that are no token, then `dense` other rows.  Tile row r of the layout is model row
 * map[r] (video token (f, y, x) is model row video_row0 + f * rows_per_frame + y * pw + x, dense row i is model row i;
 * -1 for padding), valid[r] = 1 for tokens, cnt[c] = the tokens of cube c.  info receives the cube count, the rows,
 * q_pad (a multiple of 64) and k_pad (of 128) -- the sizes of map and valid --, the dense range, topk =
 * max(1, ceil(keep * n_cubes)) and the frame-slab stride for cube_select's `local` option.  With null arrays only info
 * is filled.  Rejects more than 4096 cubes with the reference's message. */
typedef struct {
    uint32_t n_cubes, rows, q_pad, k_pad, dense0, dense1, topk, stride;
} mako_cube_layout_info;
int mako_cube_layout(uint32_t frames, uint32_t ph, uint32_t pw, uint32_t rows_per_frame, uint32_t video_row0,
                     uint32_t dense, float keep, int32_t* map, uint8_t* valid, uint32_t* cnt,
                     mako_cube_layout_info* info);

/* Block-sparse attention from kept-block lists: n rows (a multiple of 64) of 64-row blocks, query block t of head
 * h attends the key blocks lists[h][t][0 .. counts[h][t]) (int32 device arrays, [heads][n / 64][max_list] and
 * [heads][n / 64]); every key valid, output row r to o row r (width heads * 128).  The same kernel as
 * mako_attention_sparse with no dense rows, an all-valid mask and the identity map -- the form H3's cube layout
 * takes when every row is a full cube (src/models/h3.cpp:510-546). */
int mako_attention_block_sparse(mako_attn_ctx* ctx, void* stream, int dtype, const void* q, const void* k,
                                const void* v, float* o, uint32_t n, uint32_t heads, uint32_t kv_heads,
                                const int32_t* lists, const int32_t* counts, uint32_t max_list);

/* ---- Head-tile producers: the 16-bit tiles the attention calls read, from fp32 projection rows ----------------
 * y is [heads][n_pad][dim] of `dtype` (the reference writes half; MAKO_BF16 is offered for bf16 attention), 16-byte
 * aligned like the attention tensors.  cs holds
 * the rotation angles as (cos, sin) float pairs; x, cs and w are device fp32 arrays.  Calls are stream-ordered. */

/* TransformerRuntime::heads (src/models/runtime.hpp:75-77, runtime.cpp:215-226; kernel heads_half, ops.metal:21-43):
 * y[h][t][d] = x[t][col0 + h * 128 + d] for t < T, rotated when rope is 1 (halves, d with d + 64) or 2 (adjacent
 * pairs) by cs[t][pair]; the rows [T, n_pad) are zeroed.  128-wide heads. */
int mako_heads(mako_attn_ctx* ctx, void* stream, int dtype, const float* x, uint32_t ld, uint32_t col0,
               uint32_t heads, uint32_t T, uint32_t n_pad, const float* cs, uint32_t rope, void* y);
/* TransformerRuntime::heads_norm (runtime.hpp:78-81, runtime.cpp:228-241; kernel heads_norm_half,
 * ops.metal:371-408): mako_heads with each head RMS-normed first (x / sqrt(mean(x^2) + eps) * w[d]), written at rows
 * row0 .. row0 + T - 1; the other rows are left as they are. */
int mako_heads_norm(mako_attn_ctx* ctx, void* stream, int dtype, const float* x, uint32_t ld, uint32_t col0,
                    uint32_t heads, uint32_t T, uint32_t n_pad, const float* cs, uint32_t rope, const float* w,
                    float eps, uint32_t row0, void* y);
/* TransformerRuntime::heads_partial (runtime.hpp:82-87, runtime.cpp:243-260; kernel heads_partial,
 * ops.metal:577-613): heads of `dim` (a multiple of 32, at most 256) at col0 + h * stride of each row, RMS-normed
 * times w when w is given (eps), their first `rot` values rotated as halves (i with i + rot / 2) by cs[t][i]
 * (rot / 2 pairs a row); with a map, y row r comes from x row map[r] and its angles (a zero row where map[r] < 0).
 * Rejects what the reference rejects (dim > 256, dim % 32, odd rot) and, added, rot > dim. */
int mako_heads_partial(mako_attn_ctx* ctx, void* stream, int dtype, const float* x, uint32_t ld, uint32_t col0,
                       uint32_t stride, uint32_t dim, uint32_t rot, uint32_t heads, uint32_t T, uint32_t n_pad,
                       const float* cs, const float* w, float eps, void* y, const int32_t* map);
/* Kernel heads_clear (ops.metal:45-52), dispatched by the models after heads_partial (src/models/h3.cpp:352-356):
 * zero the rows [from, n_pad) of every head of y [heads][n_pad][dim], so padded keys and values read as zeros. */
int mako_heads_clear(mako_attn_ctx* ctx, void* stream, int dtype, void* y, uint32_t dim, uint32_t n_pad, uint32_t from,
                     uint32_t heads);

/* ---- The consumer of the attention's output --------------------------------------------------------------------- */

/* The output projection: y[t][j] = sum_i x[t][i] * w[j][i] for x [T][k] (the attention's o in its 16-bit form,
 * MAKO_OPT_OUTPUT_16BIT) and the matrix w [n][k] (one output row per j), both of `dtype`, accumulated in fp32 into
 * y [T][ldy] floats (ldy 0: n).  Replaces Runtime::proj (src/gpu/runtime.cpp:164-190) for BF16 / F16 matrices, which
 * the reference calls right after the attention (src/models/h3.cpp:366, src/models/qwen_text.cpp:312) and which
 * rounds the fp32 o to 16 bits first (the attention's 16-bit output does that rounding in its epilogue, the same
 * round-to-nearest-even).  Same rejection as the reference: k a multiple of 64; also 16-byte aligned tensors and ldy a
 * multiple of 4.  sm_100 only (MAKO_ENOTSUP otherwise). */
int mako_proj(mako_attn_ctx* ctx, void* stream, int dtype, const void* w, const void* x, float* y, uint32_t T,
              uint32_t k, uint32_t n, uint32_t ldy);

/* ---- Multi-GPU: one process per GPU of one box, the peers' memory mapped through CUDA IPC ------------------------
 * No reference counterpart: mako-common drives one Apple GPU.  BASELINE's sharded forms -- heads across GPUs with the
 * outputs gathered, and one long sequence's KV cache across GPUs with a log-sum-exp combine -- are built from these.
 * Every rank of a group makes the same collective calls (mako_attention_gather, mako_attention_decode_kv_sharded) in
 * the same order; each call's device waits on the other ranks are bounded (about a second) and a timeout sets the
 * context's device error flag (mako_attn_device_error) instead of hanging. */

#define MAKO_MAX_RANKS 8

/* An opaque 64-byte CUDA IPC memory handle (cudaIpcMemHandle_t), passed between processes by the caller. */
typedef struct {
    unsigned char bytes[64];
} mako_ipc_handle;

/* cudaMalloc on ctx's device of memory the other processes of this box can map, and its handle. */
int mako_peer_alloc(mako_attn_ctx* ctx, size_t bytes, void** ptr, mako_ipc_handle* handle);
int mako_peer_free(mako_attn_ctx* ctx, void* ptr);
/* Maps another process's mako_peer_alloc buffer (cudaIpcOpenMemHandle with lazy peer access); *ptr addresses it from
 * ctx's device.  mako_peer_close unmaps it. */
int mako_peer_open(mako_attn_ctx* ctx, const mako_ipc_handle* handle, void** ptr);
int mako_peer_close(mako_attn_ctx* ctx, void* ptr);

typedef struct mako_attn_group mako_attn_group;
/* This rank's member of a group of n_ranks (<= MAKO_MAX_RANKS) processes: an exchange area for barrier flags and
 * decode rows (max_rows = the most (sequence, head) rows one decode call will exchange), zeroed, and its handle for the
 * caller to hand to every other rank.  The group uses ctx (its device, scratch and error flag) until destroyed. */
int mako_group_create(mako_attn_ctx* ctx, uint32_t rank, uint32_t n_ranks, uint32_t max_rows, mako_attn_group** out,
                      mako_ipc_handle* handle);
/* Maps the other ranks' areas: handles[r] is rank r's handle from mako_group_create (this rank's own entry is not
 * read).  Call once, on every rank, before the first collective call. */
int mako_group_connect(mako_attn_group* g, const mako_ipc_handle* handles);
/* As mako_group_connect for ranks that share one process (one thread per GPU, peer access enabled by the caller):
 * areas[r] is rank r's area as ctx's device addresses it (mako_group_area gives each rank's own). */
int mako_group_connect_ptrs(mako_attn_group* g, void* const* areas);
/* This rank's exchange area (device pointer) and its size in bytes. */
int mako_group_area(mako_attn_group* g, void** area, size_t* bytes);
int mako_group_destroy(mako_attn_group* g);

/* Head-sharded attention with the output all-gather fused into the kernel: this rank holds heads
 * [head0, head0 + heads) of a larger problem (q [heads][q_pad][128], k and v [kv_heads][k_pad][128], its shard,
 * heads % kv_heads == 0) and stores each output row's slice (columns (head0 + h) * 128) into every rank's o:
 * o_ranks is a host array of n_ranks device pointers as this process addresses them (its own o and the others' o
 * mapped with mako_peer_open), each o [n_q][width] floats.  When this call's work on `stream` completes, this rank's
 * o holds every rank's heads.  The call begins with a barrier (no rank writes into an o that its owner may still be
 * reading from the previous call) and ends with one (every rank's stores have landed).  Masking as mako_attention
 * (q_pos0, block); 128-wide heads on sm_100 only (MAKO_ENOTSUP otherwise).  Replaces, for one rank, what the
 * reference's TransformerRuntime::attention (src/models/runtime.cpp:262-273) computes for all heads. */
int mako_attention_gather(mako_attn_group* g, void* stream, int dtype, const void* q, const void* k, const void* v,
                          float* const* o_ranks, uint32_t n_q, uint32_t q_pad, uint32_t n_k, uint32_t k_pad,
                          uint32_t heads, uint32_t kv_heads, uint32_t head0, uint32_t q_pos0, uint32_t block,
                          uint32_t width);

/* KV-sharded decode: every rank holds the same queries q [batch][heads][dim] and its own share of each sequence's
 * keys, k and v [batch][kv_heads][k_stride][dim] with kv_len [batch] (device int32, this rank's key count per
 * sequence, at most max_kv_len); o [batch][heads * dim] receives on every rank the attention over all ranks' keys.
 * Each rank merges its splits into one (o, max, sum) row per (sequence, head), stores it into every rank's exchange
 * area over NVLink and merges all ranks' rows by log-sum-exp (one kernel after the split kernel).  batch * heads must
 * be at most the group's max_rows.  Same element types and dims as mako_attention_decode. */
int mako_attention_decode_kv_sharded(mako_attn_group* g, void* stream, int dtype, const void* q, const void* k,
                                     const void* v, float* o, uint32_t batch, const int32_t* kv_len,
                                     uint32_t max_kv_len, uint32_t heads, uint32_t kv_heads, uint32_t dim,
                                     uint32_t k_stride);

#ifdef __cplusplus
} /* extern "C" */
#endif

#endif /* MAKO_ATTN_H */
