// Stand-in for mako-common's src/mtl/context.hpp (and the metal-cpp types it pulls in), enough for the reference's
// tests/sparse_attn_test.cpp to compile unmodified against a backend of this repository.  Test infrastructure only.
//
// A Buffer is Metal's shared storage mode as the test uses it: contents() is host memory the test writes before a
// command buffer and reads after finish().  The CUDA backend mirrors it in device memory (uploaded when an encoder
// opens, downloaded at finish); the oracle backend computes on the host copy directly.
#pragma once

#include <cstddef>
#include <cstdint>
#include <memory>
#include <vector>

namespace MTL {

class Buffer {
public:
    explicit Buffer(uint64_t bytes) : host_(bytes, std::byte{0}) {}
    void* contents() { return host_.data(); }
    uint64_t length() const { return host_.size(); }
    // The backend's copy (device memory for the CUDA backend; unused by the oracle backend).
    void* device = nullptr;

private:
    std::vector<std::byte> host_;
};

class ComputeCommandEncoder {
public:
    void endEncoding() {}
};

class CommandBuffer {};

class CommandQueue {
public:
    CommandBuffer* commandBuffer() { return &cb_; }

private:
    CommandBuffer cb_;
};

} // namespace MTL

namespace mako::mtl {

class Context {
public:
    MTL::CommandQueue* queue() { return &queue_; }

private:
    MTL::CommandQueue queue_;
};

} // namespace mako::mtl
