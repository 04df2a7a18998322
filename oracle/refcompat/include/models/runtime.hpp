// Stand-in for mako-common's src/models/runtime.hpp, cut down to what tests/sparse_attn_test.cpp uses of
// TransformerRuntime (the members its Harness exposes, sparse_attn_test.cpp:19-30) with the reference's signatures
// (runtime.hpp:105-111; gpu::Runtime's scratch / encoder / finish / ctx_ / cur_cb_, src/gpu/runtime.hpp:77,118,124,
// 174,192).  Two backends define the members: refcompat/runtime_cuda.cpp forwards to this repository's library
// (include/mako_attn.hpp) and refcompat/runtime_oracle.cpp to the CPU oracle.  Test infrastructure only.
#pragma once

#include "mtl/context.hpp"

#include <cstdint>
#include <map>
#include <memory>
#include <string>

namespace mako::gpu {
// src/gpu/runtime.hpp:25
enum class Telemetry { off, summary, steps, layers, kernels };
} // namespace mako::gpu

namespace mako::models {

struct Backend; // the backend's state (library context and stream, or nothing)

class TransformerRuntime {
public:
    virtual ~TransformerRuntime();
    virtual const char* name() const { return "model"; }

protected:
    TransformerRuntime(mtl::Context& ctx, gpu::Telemetry telemetry);

    static constexpr uint32_t kHeadDim = 128;

    // gpu::Runtime::scratch (src/gpu/runtime.cpp:117-125): a named buffer, replaced by a larger one when too small.
    MTL::Buffer* scratch(const std::string& name, uint64_t bytes);
    // gpu::Runtime::encoder: opens a command buffer's work (the CUDA backend uploads every buffer's host copy here).
    MTL::ComputeCommandEncoder* encoder(MTL::CommandBuffer* cb, uint32_t layer, int section);
    // gpu::Runtime::finish: waits for the work, throws if it failed (the CUDA backend downloads every buffer here).
    void finish(MTL::CommandBuffer* cb);

    void cube_select(MTL::ComputeCommandEncoder*& enc, MTL::Buffer* q, MTL::Buffer* k, uint32_t heads, uint32_t q_pad,
                     uint32_t k_pad, uint32_t n_cubes, MTL::Buffer* cnt, uint32_t topk, MTL::Buffer*& sel,
                     MTL::Buffer*& nsel, uint32_t local = 0, uint32_t stride = 0);
    void attention_sparse(MTL::ComputeCommandEncoder*& enc, MTL::Buffer* q, MTL::Buffer* k, MTL::Buffer* v,
                          MTL::Buffer* o, uint32_t n_q, uint32_t q_pad, uint32_t n_k, uint32_t k_pad, uint32_t heads,
                          uint32_t kv_heads, uint32_t width, uint32_t n_cubes, uint32_t topk, uint32_t dense0,
                          uint32_t dense1, MTL::Buffer* sel, MTL::Buffer* nsel, MTL::Buffer* valid, MTL::Buffer* map);

    mtl::Context& ctx_;
    MTL::CommandBuffer* cur_cb_ = nullptr;

private:
    MTL::ComputeCommandEncoder enc_;
    std::map<std::string, std::unique_ptr<MTL::Buffer>> scratch_;
    std::unique_ptr<Backend> be_;
};

} // namespace mako::models
