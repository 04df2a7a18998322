// mako_attn.hpp -- C++ shim over the C ABI (mako_attn.h) with the method names, argument order and error behaviour
// of mako-common's TransformerRuntime attention members (src/models/runtime.hpp:90-111): device pointers and a
// cudaStream_t take the place of MTL::Buffer* and the command encoder, and a failed call throws std::runtime_error
// with the library's message, as the reference throws before encoding (src/models/runtime.cpp:266-267,290-291,
// 311-312).  Calls are stream-ordered and do not synchronise; one Attention object per thread / stream.
#pragma once

#include "mako_attn.h"

#include <cstdint>
#include <stdexcept>
#include <string>
#include <vector>

namespace mako::attn {

enum class Dtype : int { f16 = MAKO_F16, bf16 = MAKO_BF16 };

class Attention {
public:
    static constexpr uint32_t kHeadDim = 128;  // src/models/runtime.hpp:33

    explicit Attention(int device = 0, Dtype dtype = Dtype::f16) : dtype_(int(dtype))
    {
        check(mako_attn_create(device, &ctx_));
    }
    ~Attention() { mako_attn_destroy(ctx_); }
    Attention(const Attention&) = delete;
    Attention& operator=(const Attention&) = delete;

    void set_dtype(Dtype d) { dtype_ = int(d); }
    void set_stream(void* stream) { stream_ = stream; }
    // o in the tiles' 16-bit type (what the reference's to_half / to_bf16 makes of o before the output projection)
    // instead of fp32: `o` then points at that storage.
    void set_output_16bit(bool on) { check(mako_attn_set_option(ctx_, MAKO_OPT_OUTPUT_16BIT, on ? 1 : 0)); }

    // TransformerRuntime::attention (src/models/runtime.hpp:90-95).
    void attention(const void* q, const void* k, const void* v, float* o, uint32_t n_q, uint32_t q_pad, uint32_t n_k,
                   uint32_t k_pad, uint32_t heads, uint32_t kv_heads, uint32_t q_pos0, uint32_t block,
                   uint32_t dim = kHeadDim)
    {
        check(mako_attention(ctx_, stream_, dtype_, q, k, v, o, n_q, q_pad, n_k, k_pad, heads, kv_heads, q_pos0, block,
                             dim, 0));
    }
    // TransformerRuntime::cube_select (src/models/runtime.hpp:104-106): sel / nsel become this object's scratch.
    void cube_select(const void* q, const void* k, uint32_t heads, uint32_t q_pad, uint32_t k_pad, uint32_t n_cubes,
                     const uint32_t* cnt, uint32_t topk, uint16_t*& sel, uint16_t*& nsel, uint32_t local = 0,
                     uint32_t stride = 0)
    {
        check(mako_cube_select(ctx_, stream_, dtype_, q, k, heads, q_pad, k_pad, n_cubes, cnt, topk, &sel, &nsel, local,
                               stride));
    }
    // TransformerRuntime::attention_sparse (src/models/runtime.hpp:107-110).
    void attention_sparse(const void* q, const void* k, const void* v, float* o, uint32_t n_q, uint32_t q_pad,
                          uint32_t n_k, uint32_t k_pad, uint32_t heads, uint32_t kv_heads, uint32_t width,
                          uint32_t n_cubes, uint32_t topk, uint32_t dense0, uint32_t dense1, const uint16_t* sel,
                          const uint16_t* nsel, const uint8_t* valid, const int32_t* map)
    {
        check(mako_attention_sparse(ctx_, stream_, dtype_, q, k, v, o, n_q, q_pad, n_k, k_pad, heads, kv_heads, width,
                                    n_cubes, topk, dense0, dense1, sel, nsel, valid, map));
    }
    // Batched decode over a KV cache (no reference member: its decode step is attention() with n_q = 1).
    void attention_decode(const void* q, const void* k, const void* v, float* o, uint32_t batch, const int32_t* kv_len,
                          uint32_t max_kv_len, uint32_t heads, uint32_t kv_heads, uint32_t dim, uint32_t k_stride)
    {
        check(mako_attention_decode(ctx_, stream_, dtype_, q, k, v, o, batch, kv_len, max_kv_len, heads, kv_heads, dim,
                                    k_stride));
    }
    // Runtime::proj for a BF16 / F16 matrix (src/gpu/runtime.cpp:164-190) on the attention's 16-bit output:
    // y[t][j] = sum_i x[t][i] w[j][i], x [T][k] and w [n][k] of this object's dtype, y [T][ldy] floats (0: n).
    void proj(const void* w, const void* x, float* y, uint32_t T, uint32_t k, uint32_t n, uint32_t ldy = 0)
    {
        check(mako_proj(ctx_, stream_, dtype_, w, x, y, T, k, n, ldy));
    }
    // TransformerRuntime::heads_partial (src/models/runtime.hpp:82-87): y 16-bit tiles of this object's dtype.
    void heads_partial(const float* x, uint32_t ld, uint32_t col0, uint32_t stride, uint32_t dim, uint32_t rot,
                       uint32_t heads, uint32_t T, uint32_t n_pad, const float* cs, const float* w, float eps, void* y,
                       const int32_t* map = nullptr)
    {
        check(mako_heads_partial(ctx_, stream_, dtype_, x, ld, col0, stride, dim, rot, heads, T, n_pad, cs, w, eps, y,
                                 map));
    }
    // TransformerRuntime::heads (runtime.hpp:75-77) and heads_norm (:78-81).
    void heads(const float* x, uint32_t ld, uint32_t col0, uint32_t heads, uint32_t T, uint32_t n_pad, const float* cs,
               uint32_t rope, void* y)
    {
        check(mako_heads(ctx_, stream_, dtype_, x, ld, col0, heads, T, n_pad, cs, rope, y));
    }
    void heads_norm(const float* x, uint32_t ld, uint32_t col0, uint32_t heads, uint32_t T, uint32_t n_pad,
                    const float* cs, uint32_t rope, const float* w, float eps, uint32_t row0, void* y)
    {
        check(mako_heads_norm(ctx_, stream_, dtype_, x, ld, col0, heads, T, n_pad, cs, rope, w, eps, row0, y));
    }
    // The heads_clear dispatch (ops.metal:45-52): zero rows [from, n_pad) of every head.
    void heads_clear(void* y, uint32_t dim, uint32_t n_pad, uint32_t from, uint32_t heads)
    {
        check(mako_heads_clear(ctx_, stream_, dtype_, y, dim, n_pad, from, heads));
    }
    // The check gpu::Runtime::finish makes after a command buffer (src/gpu/runtime.cpp:466-471): throws if a
    // pipelined kernel gave up on a wait.  Synchronises the device.
    void finish()
    {
        int err = 0;
        check(mako_attn_device_error(ctx_, &err));
        if (err)
            throw std::runtime_error("attention: a kernel gave up on a pipeline wait (code " + std::to_string(err) + ")");
    }
    mako_attn_ctx* handle() const { return ctx_; }
    void* stream() const { return stream_; }
    int dtype() const { return dtype_; }

    static void check(int rc)
    {
        if (rc != MAKO_OK)
            throw std::runtime_error(mako_attn_last_error());
    }

private:
    mako_attn_ctx* ctx_ = nullptr;
    void* stream_ = nullptr;
    int dtype_ = MAKO_F16;
};

// One process's member of a group of ranks on one box (no reference counterpart: mako-common drives one GPU).
// `exchange` passes this rank's handle to every rank and returns all ranks' handles in rank order -- MPI_Allgather,
// a torch.distributed all_gather_object, a file: whatever the host already uses to launch its ranks.
class Group {
public:
    template <typename Exchange>
    Group(Attention& attn, uint32_t rank, uint32_t n_ranks, uint32_t max_rows, Exchange&& exchange) : attn_(attn)
    {
        mako_ipc_handle mine;
        Attention::check(mako_group_create(attn.handle(), rank, n_ranks, max_rows, &g_, &mine));
        const std::vector<mako_ipc_handle> all = exchange(mine);
        if (all.size() != n_ranks) {
            mako_group_destroy(g_);
            throw std::runtime_error("group: the exchange returned the wrong number of handles");
        }
        const int rc = mako_group_connect(g_, all.data());
        if (rc != MAKO_OK) {
            const std::string msg = mako_attn_last_error();
            mako_group_destroy(g_);
            throw std::runtime_error(msg);
        }
    }
    ~Group() { mako_group_destroy(g_); }
    Group(const Group&) = delete;
    Group& operator=(const Group&) = delete;

    // attention() for this rank's heads [head0, head0 + heads), each output row's slice stored into every rank's o
    // (o_ranks: n_ranks pointers as this process addresses them, the others' mapped with mako_peer_open).
    void attention_gather(const void* q, const void* k, const void* v, float* const* o_ranks, uint32_t n_q,
                          uint32_t q_pad, uint32_t n_k, uint32_t k_pad, uint32_t heads, uint32_t kv_heads,
                          uint32_t head0, uint32_t q_pos0, uint32_t block, uint32_t width)
    {
        Attention::check(mako_attention_gather(g_, attn_.stream(), attn_.dtype(), q, k, v, o_ranks, n_q, q_pad, n_k,
                                               k_pad, heads, kv_heads, head0, q_pos0, block, width));
    }
    // attention_decode() over this rank's share of each sequence's keys, merged with the other ranks' shares.
    void attention_decode_kv_sharded(const void* q, const void* k, const void* v, float* o, uint32_t batch,
                                     const int32_t* kv_len, uint32_t max_kv_len, uint32_t heads, uint32_t kv_heads,
                                     uint32_t dim, uint32_t k_stride)
    {
        Attention::check(mako_attention_decode_kv_sharded(g_, attn_.stream(), attn_.dtype(), q, k, v, o, batch, kv_len,
                                                          max_kv_len, heads, kv_heads, dim, k_stride));
    }

private:
    Attention& attn_;
    mako_attn_group* g_ = nullptr;
};

// The cube layout of a video sequence for the sparse path (src/models/h3.cpp:510-546): host arrays to copy to the
// device (map [q_pad], valid [k_pad], cnt [n_cubes]) and the sizes the sparse calls take.  Throws as the reference
// does past 4096 cubes.
struct CubeLayout {
    mako_cube_layout_info info{};
    std::vector<int32_t> map;
    std::vector<uint8_t> valid;
    std::vector<uint32_t> cnt;
};

inline CubeLayout cube_layout(uint32_t frames, uint32_t ph, uint32_t pw, uint32_t rows_per_frame,
                              uint32_t video_row0, uint32_t dense, float keep)
{
    CubeLayout c;
    Attention::check(mako_cube_layout(frames, ph, pw, rows_per_frame, video_row0, dense, keep, nullptr, nullptr,
                                      nullptr, &c.info));
    c.map.resize(c.info.q_pad);
    c.valid.resize(c.info.k_pad);
    c.cnt.resize(c.info.n_cubes);
    Attention::check(mako_cube_layout(frames, ph, pw, rows_per_frame, video_row0, dense, keep, c.map.data(),
                                      c.valid.data(), c.cnt.data(), &c.info));
    return c;
}

} // namespace mako::attn
