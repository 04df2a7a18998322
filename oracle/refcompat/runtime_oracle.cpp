// TransformerRuntime's sparse-attention members (src/models/runtime.cpp:286-317) over the CPU oracle, so that the
// reference's own test (tests/sparse_attn_test.cpp) checks the oracle with its own loops and tolerances.  Test
// infrastructure only: it links ../attn_oracle.cpp and nothing of the CUDA library.
//
// MAKO_ORACLE_SELECT_MODE picks the oracle's cube_select arithmetic: 1 (default) the fp32 order the CUDA kernels
// reproduce bit for bit, 0 double precision.
#include "models/runtime.hpp"

#include <algorithm>
#include <cstdlib>
#include <format>
#include <stdexcept>

extern "C" {
void oracle_cube_select(int dtype, const uint16_t* q, const uint16_t* k, uint32_t heads, uint32_t q_pad,
                        uint32_t k_pad, uint32_t n_cubes, const uint32_t* cnt, uint32_t topk, uint32_t local,
                        uint32_t stride, int mode, uint16_t* sel, uint16_t* nsel, float* qp_out, float* kp_out,
                        float* sc_out);
void oracle_attention_sparse(int dtype, const uint16_t* q, const uint16_t* k, const uint16_t* v, float* o,
                             uint32_t n_q, uint32_t q_pad, uint32_t n_k, uint32_t k_pad, uint32_t heads,
                             uint32_t kv_heads, uint32_t width, uint32_t n_cubes, uint32_t max_sel, uint32_t dense0,
                             uint32_t dense1, const uint16_t* sel, const uint16_t* nsel, const uint8_t* valid,
                             const int32_t* map, const uint32_t* rows, uint32_t n_rows, int threads);
}

namespace mako::models {

struct Backend {
    int select_mode = 1;
};

TransformerRuntime::TransformerRuntime(mtl::Context& ctx, gpu::Telemetry) : ctx_(ctx), be_(std::make_unique<Backend>())
{
    if (const char* m = std::getenv("MAKO_ORACLE_SELECT_MODE"))
        be_->select_mode = std::atoi(m);
}

TransformerRuntime::~TransformerRuntime() = default;

MTL::Buffer* TransformerRuntime::scratch(const std::string& name, uint64_t bytes)
{
    auto it = scratch_.find(name);
    if (it == scratch_.end() || it->second->length() < bytes)
        it = scratch_.insert_or_assign(name, std::make_unique<MTL::Buffer>(std::max<uint64_t>(bytes, 16))).first;
    return it->second.get();
}

MTL::ComputeCommandEncoder* TransformerRuntime::encoder(MTL::CommandBuffer*, uint32_t, int) { return &enc_; }

void TransformerRuntime::finish(MTL::CommandBuffer*) {}

void TransformerRuntime::cube_select(MTL::ComputeCommandEncoder*&, MTL::Buffer* q, MTL::Buffer* k, uint32_t heads,
                                     uint32_t q_pad, uint32_t k_pad, uint32_t n_cubes, MTL::Buffer* cnt, uint32_t topk,
                                     MTL::Buffer*& sel, MTL::Buffer*& nsel, uint32_t local, uint32_t stride)
{
    if (n_cubes > 4096 || !topk || (local != 0 && local != 1 && local != 3))
        throw std::runtime_error(std::format("cube_select: {} cubes, top {}, local {}", n_cubes, topk, local));
    const uint32_t kk = std::min(topk, n_cubes);
    sel = scratch("c_sel", uint64_t(heads) * n_cubes * kk * 2);
    nsel = scratch("c_nsel", uint64_t(heads) * n_cubes * 2);
    oracle_cube_select(0, static_cast<const uint16_t*>(q->contents()), static_cast<const uint16_t*>(k->contents()),
                       heads, q_pad, k_pad, n_cubes, static_cast<const uint32_t*>(cnt->contents()), topk, local, stride,
                       be_->select_mode, static_cast<uint16_t*>(sel->contents()),
                       static_cast<uint16_t*>(nsel->contents()), nullptr, nullptr, nullptr);
}

void TransformerRuntime::attention_sparse(MTL::ComputeCommandEncoder*&, MTL::Buffer* q, MTL::Buffer* k, MTL::Buffer* v,
                                          MTL::Buffer* o, uint32_t n_q, uint32_t q_pad, uint32_t n_k, uint32_t k_pad,
                                          uint32_t heads, uint32_t kv_heads, uint32_t width, uint32_t n_cubes,
                                          uint32_t topk, uint32_t dense0, uint32_t dense1, MTL::Buffer* sel,
                                          MTL::Buffer* nsel, MTL::Buffer* valid, MTL::Buffer* map)
{
    if (q_pad % 64 || k_pad % 128 || dense0 % 32)
        throw std::runtime_error(
            "attention_sparse: q_pad a multiple of 64, k_pad of 128, the dense rows from a multiple of 32");
    oracle_attention_sparse(0, static_cast<const uint16_t*>(q->contents()), static_cast<const uint16_t*>(k->contents()),
                            static_cast<const uint16_t*>(v->contents()), static_cast<float*>(o->contents()), n_q, q_pad,
                            n_k, k_pad, heads, kv_heads, width, n_cubes, std::min(topk, n_cubes), dense0, dense1,
                            static_cast<const uint16_t*>(sel->contents()), static_cast<const uint16_t*>(nsel->contents()),
                            static_cast<const uint8_t*>(valid->contents()), static_cast<const int32_t*>(map->contents()),
                            nullptr, 0, 0);
}

} // namespace mako::models
