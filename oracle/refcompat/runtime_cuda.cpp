// TransformerRuntime's sparse-attention members (src/models/runtime.cpp:286-317) over this repository's CUDA library,
// through the C++ shim include/mako_attn.hpp, so that the reference's own test (tests/sparse_attn_test.cpp) checks
// the B200 kernels with its own loops and tolerances.  Test infrastructure: the test binary it builds runs on a GPU.
//
// Buffers follow Metal's shared storage as the test uses it: each scratch buffer has a host copy (contents()) and a
// device copy; encoder() uploads every host copy, finish() waits for the stream, downloads every device copy and
// throws if the library reports a failed kernel (gpu::Runtime::finish, src/gpu/runtime.cpp:453-471).
#include "models/runtime.hpp"

#include "mako_attn.hpp"

#include <cuda_runtime_api.h>

#include <algorithm>
#include <format>
#include <stdexcept>

namespace mako::models {

namespace {
void cu(cudaError_t e, const char* what)
{
    if (e != cudaSuccess)
        throw std::runtime_error(std::format("{}: {}", what, cudaGetErrorString(e)));
}
} // namespace

struct Backend {
    attn::Attention attn{0, attn::Dtype::f16};
    cudaStream_t stream = nullptr;
};

TransformerRuntime::TransformerRuntime(mtl::Context& ctx, gpu::Telemetry) : ctx_(ctx), be_(std::make_unique<Backend>())
{
    cu(cudaStreamCreateWithFlags(&be_->stream, cudaStreamNonBlocking), "cudaStreamCreate");
    be_->attn.set_stream(be_->stream);
}

TransformerRuntime::~TransformerRuntime()
{
    cudaStreamSynchronize(be_->stream);
    for (auto& [name, b] : scratch_)
        cudaFree(b->device);
    cudaStreamDestroy(be_->stream);
}

MTL::Buffer* TransformerRuntime::scratch(const std::string& name, uint64_t bytes)
{
    auto it = scratch_.find(name);
    if (it == scratch_.end() || it->second->length() < bytes) {
        auto b = std::make_unique<MTL::Buffer>(std::max<uint64_t>(bytes, 16));
        cu(cudaMalloc(&b->device, b->length()), "cudaMalloc");
        if (it != scratch_.end()) {
            cu(cudaStreamSynchronize(be_->stream), "cudaStreamSynchronize");
            cudaFree(it->second->device);
        }
        it = scratch_.insert_or_assign(name, std::move(b)).first;
    }
    return it->second.get();
}

MTL::ComputeCommandEncoder* TransformerRuntime::encoder(MTL::CommandBuffer*, uint32_t, int)
{
    for (auto& [name, b] : scratch_)
        cu(cudaMemcpyAsync(b->device, b->contents(), b->length(), cudaMemcpyHostToDevice, be_->stream), "upload");
    return &enc_;
}

void TransformerRuntime::finish(MTL::CommandBuffer*)
{
    for (auto& [name, b] : scratch_)
        cu(cudaMemcpyAsync(b->contents(), b->device, b->length(), cudaMemcpyDeviceToHost, be_->stream), "download");
    cu(cudaStreamSynchronize(be_->stream), "command buffer");
    be_->attn.finish();
}

void TransformerRuntime::cube_select(MTL::ComputeCommandEncoder*&, MTL::Buffer* q, MTL::Buffer* k, uint32_t heads,
                                     uint32_t q_pad, uint32_t k_pad, uint32_t n_cubes, MTL::Buffer* cnt, uint32_t topk,
                                     MTL::Buffer*& sel, MTL::Buffer*& nsel, uint32_t local, uint32_t stride)
{
    uint16_t *s = nullptr, *ns = nullptr;
    be_->attn.cube_select(q->device, k->device, heads, q_pad, k_pad, n_cubes, static_cast<const uint32_t*>(cnt->device),
                          topk, s, ns, local, stride);
    // The library returns sel / nsel as its own scratch; the test reads them as runtime buffers.
    const uint64_t sel_bytes = uint64_t(heads) * n_cubes * std::min(topk, n_cubes) * 2,
                   nsel_bytes = uint64_t(heads) * n_cubes * 2;
    sel = scratch("c_sel", sel_bytes);
    nsel = scratch("c_nsel", nsel_bytes);
    cu(cudaMemcpyAsync(sel->device, s, sel_bytes, cudaMemcpyDeviceToDevice, be_->stream), "sel");
    cu(cudaMemcpyAsync(nsel->device, ns, nsel_bytes, cudaMemcpyDeviceToDevice, be_->stream), "nsel");
}

void TransformerRuntime::attention_sparse(MTL::ComputeCommandEncoder*&, MTL::Buffer* q, MTL::Buffer* k, MTL::Buffer* v,
                                          MTL::Buffer* o, uint32_t n_q, uint32_t q_pad, uint32_t n_k, uint32_t k_pad,
                                          uint32_t heads, uint32_t kv_heads, uint32_t width, uint32_t n_cubes,
                                          uint32_t topk, uint32_t dense0, uint32_t dense1, MTL::Buffer* sel,
                                          MTL::Buffer* nsel, MTL::Buffer* valid, MTL::Buffer* map)
{
    be_->attn.attention_sparse(q->device, k->device, v->device, static_cast<float*>(o->device), n_q, q_pad, n_k, k_pad,
                               heads, kv_heads, width, n_cubes, topk, dense0, dense1,
                               static_cast<const uint16_t*>(sel->device), static_cast<const uint16_t*>(nsel->device),
                               static_cast<const uint8_t*>(valid->device), static_cast<const int32_t*>(map->device));
}

} // namespace mako::models
