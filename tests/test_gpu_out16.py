"""16-bit attention output (MAKO_OPT_OUTPUT_16BIT): o in the call's input type, the values the reference's to_half /
to_bf16 conversion makes of its fp32 o before the output projection (src/gpu/runtime.cpp:164-190).  Each call runs
twice on the same inputs, fp32 then 16-bit: the 16-bit o must equal the fp32 o rounded to nearest even, bit for bit
(the kernels scale in fp32 and round once at the store), and rows or columns a call does not own stay untouched.
The fp32 results themselves are checked against the oracle in test_gpu_parity.py."""
import numpy as np
import pytest

import attn_cases as C

pytestmark = pytest.mark.gpu
SENT16 = 0x7BFF


def round16(x, dtype):
    """fp32 -> 16-bit bits, round to nearest even (the oracle's conversion)."""
    import oracle as O
    return O.to_bits(np.ascontiguousarray(x, np.float32), dtype)


def dev(bits, dtype):
    import torch
    t = torch.from_numpy(np.ascontiguousarray(bits).view(np.int16))
    return t.view(torch.bfloat16 if dtype == 1 else torch.float16).cuda()


def out_pair(rows, width, dtype):
    import torch
    o32 = torch.full((rows, width), 12345.0, dtype=torch.float32, device="cuda")
    o16 = torch.full((rows, width), SENT16, dtype=torch.int16, device="cuda")
    return o32, o16


def both(ctx, call, o32, o16, dtype):
    """call(o) once with fp32 o, once with the 16-bit option; returns (fp32 array, 16-bit bits)."""
    import torch
    import mako_attn
    call(o32)
    ctx.set_option(mako_attn.OPT_OUTPUT_16BIT, 1)
    try:
        call(o16.view(torch.bfloat16 if dtype == 1 else torch.float16))
    finally:
        ctx.set_option(mako_attn.OPT_OUTPUT_16BIT, 0)
    torch.cuda.synchronize()
    assert ctx.device_error() == 0
    return o32.cpu().numpy(), o16.cpu().numpy().view(np.uint16)




@pytest.mark.parametrize("dim", [64, 128, 256])
@pytest.mark.parametrize("kernel", [0, 1], ids=["auto", "mma"])
@pytest.mark.parametrize("dtype", [0, 1])
def test_dense_out16(ctx, kernel, dtype, dim):
    import mako_attn
    case = C.dense_case(seed=60 + dtype, heads=4, kv_heads=2, dim=dim, n_q=300, n_k=300, dtype=dtype)
    q, k, v = dev(case["q"], dtype), dev(case["k"], dtype), dev(case["v"], dtype)
    hw = 4 * dim
    width = hw + 8  # a wider o row: the columns past the heads stay untouched
    o32, o16 = out_pair(300 + 2, width, dtype)
    ctx.set_option(mako_attn.OPT_PREFILL_KERNEL, kernel)
    try:
        f32, b16 = both(ctx, lambda o: ctx.attention(q, k, v, o, 300, case["q_pad"], 300, case["k_pad"], 4, 2, 0,
                                                     0xFFFFFFFF, dim, width), o32, o16, dtype)
    finally:
        ctx.set_option(mako_attn.OPT_PREFILL_KERNEL, 0)
    np.testing.assert_array_equal(b16[:300, :hw], round16(f32[:300, :hw], dtype))
    assert np.all(b16[:300, hw:] == SENT16) and np.all(b16[300:] == SENT16)


@pytest.mark.parametrize("dim", [64, 128, 256])
def test_decode_out16(ctx, dim):
    """Batched decode: one split and several (the combine's store), a one-key and a zero-key sequence."""
    import torch
    dtype = 1
    rng = np.random.default_rng(70 + dim)
    B, H, KV, S = 4, 8, 2, 3000
    lens = np.array([3000, 1, 0, 333], np.int32)
    q = dev(round16(rng.standard_normal((B, H, dim)), dtype), dtype)
    k = dev(round16(rng.standard_normal((B, KV, S, dim)), dtype), dtype)
    v = dev(round16(rng.standard_normal((B, KV, S, dim)), dtype), dtype)
    kl = torch.from_numpy(lens).cuda()
    o32 = torch.full((B, H * dim), 12345.0, dtype=torch.float32, device="cuda")
    o16 = torch.full((B, H * dim), SENT16, dtype=torch.int16, device="cuda")
    f32, b16 = both(ctx, lambda o: ctx.attention_decode(q, k, v, o, kl, S, H, KV, dim, S), o32, o16, dtype)
    np.testing.assert_array_equal(b16, round16(f32, dtype))
    assert np.all(f32[2] == 0.0)


def test_single_query_out16(ctx):
    """attention() with one query goes to the split-KV decode kernel; o rows there may have any width."""
    dtype = 0
    case = C.dense_case(seed=75, heads=4, kv_heads=1, dim=128, n_q=1, n_k=900, dtype=dtype, q_pos0=899)
    q, k, v = dev(case["q"], dtype), dev(case["k"], dtype), dev(case["v"], dtype)
    width = 4 * 128 + 2
    o32, o16 = out_pair(1, width, dtype)
    f32, b16 = both(ctx, lambda o: ctx.attention(q, k, v, o, 1, case["q_pad"], 900, case["k_pad"], 4, 1, 899,
                                                 0xFFFFFFFF, 128, width), o32, o16, dtype)
    np.testing.assert_array_equal(b16[:, :512], round16(f32[:, :512], dtype))
    assert np.all(b16[:, 512:] == SENT16)


@pytest.mark.parametrize("dtype", [0, 1])
def test_block_sparse_out16(ctx, dtype):
    heads, n = 3, 1024
    nb = n // 64
    lists, counts = C.block_lists(90 + dtype, heads, nb, 0.2)
    case = C.dense_case(seed=91 + dtype, heads=heads, kv_heads=heads, dim=128, n_q=n, n_k=n, dtype=dtype)
    q, k, v = dev(case["q"], dtype), dev(case["k"], dtype), dev(case["v"], dtype)
    import torch
    o32, o16 = out_pair(n, heads * 128, dtype)
    f32, b16 = both(ctx, lambda o: ctx.attention_block_sparse(q, k, v, o, n, heads, heads,
                                                              torch.from_numpy(lists).cuda(),
                                                              torch.from_numpy(counts).cuda()), o32, o16, dtype)
    np.testing.assert_array_equal(b16, round16(f32, dtype))


def test_out16_rejections(ctx):
    import torch
    import mako_attn
    q = torch.zeros(4 * 64 * 128, dtype=torch.float16, device="cuda")
    o = torch.zeros(64 * 1024, dtype=torch.float16, device="cuda")
    ctx.set_option(mako_attn.OPT_OUTPUT_16BIT, 1)
    try:
        with pytest.raises(mako_attn.MakoError, match="a multiple of 8"):
            ctx.attention(q, q, q, o, 10, 64, 10, 64, 1, 1, 0, 0, 128, 132)
    finally:
        ctx.set_option(mako_attn.OPT_OUTPUT_16BIT, 0)
    with pytest.raises(mako_attn.MakoError, match="a multiple of 4"):
        ctx.attention(q, q, q, o.view(torch.float32), 10, 64, 10, 64, 1, 1, 0, 0, 128, 130)
