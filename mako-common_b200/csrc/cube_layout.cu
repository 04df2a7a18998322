// The block-sparse attention's cube layout of a video sequence (host code): MiniMax-H3's sparse path puts the
// generated video tokens in 4 x 4 x 4 cubes of (frame, patch row, patch column) -- the grid padded to multiples of 4
// with rows that are no token -- followed by the sequence's other rows (text, conditioning, audio) as dense rows, and
// describes that order to the attention by three arrays (src/models/h3.cpp:510-546):
//   map   [q_pad]   int32  tile row -> model row (-1: a padding row)
//   valid [k_pad]   uint8  1 where the tile row is a token
//   cnt   [n_cubes] uint32 tokens of each cube
// plus the cube count, the dense row range, the top-k for a keep fraction and the neighbour stride of the `local`
// option (one frame-slab of cubes).  The caller copies the arrays to the device for mako_cube_select /
// mako_heads_partial / mako_attention_sparse.
#include "mako_attn.h"
#include "kernels.h"

#include <algorithm>
#include <cmath>

extern "C" int mako_cube_layout(uint32_t frames, uint32_t ph, uint32_t pw, uint32_t rows_per_frame,
                                uint32_t video_row0, uint32_t dense, float keep, int32_t* map, uint8_t* valid,
                                uint32_t* cnt, mako_cube_layout_info* info)
{
    constexpr uint32_t kCube = 4;
    if (!info)
        return mako::set_error(MAKO_EINVAL, "cube_layout: null info");
    if (rows_per_frame < uint64_t(ph) * pw)
        return mako::set_error(MAKO_EINVAL, "cube_layout: %u rows a frame for %u x %u patches", rows_per_frame, ph,
                               pw);
    if (!(keep > 0.0f) || keep > 1.0f)
        return mako::set_error(MAKO_EINVAL, "cube_layout: keep fraction %g (0, 1]", double(keep));
    const uint32_t fc = (frames + kCube - 1) / kCube, yc = (ph + kCube - 1) / kCube, xc = (pw + kCube - 1) / kCube;
    const uint64_t n = uint64_t(fc) * yc * xc;
    if (n > 4096)  // the reference's limit and message (src/models/h3.cpp:516-517)
        return mako::set_error(MAKO_EINVAL, "sparse attention: more than 4096 cubes");
    const uint64_t vrows = n * 64, rows = vrows + dense;
    if (rows > 0x7FFFFFFFull || uint64_t(video_row0) + uint64_t(frames) * rows_per_frame > 0x7FFFFFFFull)
        return mako::set_error(MAKO_EINVAL, "cube_layout: %llu rows", (unsigned long long)rows);
    info->n_cubes = uint32_t(n);
    info->rows = uint32_t(rows);
    info->q_pad = uint32_t((rows + 63) / 64 * 64);  // runtime.hpp's kAttnRows tiles
    info->k_pad = uint32_t((rows + 127) / 128 * 128);
    info->dense0 = uint32_t(vrows);
    info->dense1 = uint32_t(rows);
    info->topk = std::max<uint32_t>(1, uint32_t(std::ceil(double(keep) * double(n))));
    info->stride = yc * xc;
    if (!map || !valid || !cnt)  // sizes only
        return MAKO_OK;
    std::fill_n(map, info->q_pad, -1);
    std::fill_n(valid, info->k_pad, uint8_t(0));
    std::fill_n(cnt, n, 0u);
    for (uint32_t f = 0; f < frames; ++f)
        for (uint32_t y = 0; y < ph; ++y)
            for (uint32_t x = 0; x < pw; ++x) {
                const uint32_t cube = ((f / kCube) * yc + y / kCube) * xc + x / kCube;
                const uint32_t r = cube * 64 + ((f % kCube) * kCube + y % kCube) * kCube + x % kCube;
                map[r] = int32_t(video_row0 + f * rows_per_frame + y * pw + x);
                valid[r] = 1;
                ++cnt[cube];
            }
    for (uint32_t r = 0; r < dense; ++r) {
        map[vrows + r] = int32_t(r);
        valid[vrows + r] = 1;
    }
    mako::clear_error();
    return MAKO_OK;
}
