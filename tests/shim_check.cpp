// Host-side check of the C++ shim (include/mako_attn.hpp): it compiles against the C ABI, links libmako_attn.so and
// turns the library's statuses into std::runtime_error like TransformerRuntime does.  Needs no GPU: without a device
// the constructor must throw; with one, an argument the reference rejects (a head width of 96,
// src/models/runtime.cpp:266-267) must throw before anything is enqueued.
#include "mako_attn.hpp"

#include <cstdio>
#include <cstring>

int main(int argc, char**)
{
    // host code, no device needed: 3 x 10 x 10 patches -> 1 x 3 x 3 cubes, 50 dense rows after them
    const auto lay = mako::attn::cube_layout(3, 10, 10, 100, 50, 50, 0.15f);
    if (lay.info.n_cubes != 9 || lay.info.dense0 != 576 || lay.map.size() != 640 || lay.map[0] != 50 ||
        lay.cnt[2] != 24) {
        std::printf("cube_layout: unexpected layout\n");
        return 1;
    }
    try {
        mako::attn::Attention attn(0);
        if (argc > 100) {  // compiled, never run here: a one-rank group whose exchange is the identity
            mako::attn::Group g(attn, 0, 1, 1, [](const mako_ipc_handle& h) { return std::vector<mako_ipc_handle>{h}; });
            g.attention_decode_kv_sharded(nullptr, nullptr, nullptr, nullptr, 0, nullptr, 0, 1, 1, 128, 0);
        }
        try {
            attn.attention(nullptr, nullptr, nullptr, nullptr, 1, 64, 1, 128, 1, 1, 0, 0, 96);
        } catch (const std::runtime_error& e) {
            std::printf("rejected: %s\n", e.what());
            return std::strstr(e.what(), "heads of 96") ? 0 : 1;
        }
        std::printf("a head width of 96 was accepted\n");
        return 1;
    } catch (const std::runtime_error& e) {
        std::printf("no device: %s\n", e.what());
        return std::strlen(e.what()) ? 0 : 1;
    }
}
