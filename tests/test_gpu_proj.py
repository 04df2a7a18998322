"""The output projection that consumes the attention's 16-bit output (mako_proj, the B200 form of Runtime::proj on a
BF16 / F16 matrix, src/gpu/runtime.cpp:164-190) against the oracle's double-precision GEMM on the same 16-bit
inputs, through the C ABI.  Tolerance: fp32 accumulation of k products of exactly representable terms, so relative L2
<= 1e-5 and every value within 1e-4 of the largest |y| (an fp32 sum of 1024 terms drifts by ~1e-6 relative)."""
import numpy as np
import pytest

import attn_cases as C

pytestmark = pytest.mark.gpu


def dev16(bits, dtype):
    import torch
    t = torch.from_numpy(np.ascontiguousarray(bits).view(np.int16))
    return t.view(torch.bfloat16 if dtype == 1 else torch.float16).cuda()


def check(got, want):
    err = np.asarray(got, np.float64) - np.asarray(want, np.float64)
    rel = float(np.sqrt(np.sum(err ** 2) / max(np.sum(np.asarray(want, np.float64) ** 2), 1e-30)))
    mx = float(np.max(np.abs(err))) / max(float(np.max(np.abs(want))), 1e-30)
    assert rel <= 1e-5 and mx <= 1e-4, f"rel-L2 {rel:.3e}, max-abs / max|y| {mx:.3e}"


@pytest.mark.parametrize("T,k,n,ldy,dtype", [
    (300, 256, 520, 0, 1),      # ragged rows and columns (a partial 32-column chunk), bf16
    (257, 512, 256, 264, 0),    # fp16, a row stride wider than n
    (1000, 1024, 768, 0, 1),    # several tiles each way
    (64, 4096, 64, 0, 1),       # one partial tile, long k (config 3's hidden size)
], ids=["ragged-bf16", "fp16-ldy", "tiles", "long-k"])
def test_proj_matches_oracle(ctx, oracle, T, k, n, ldy, dtype):
    import torch
    rng = np.random.default_rng(T + k + n)
    x = oracle.to_bits(C.normal(rng, (T, k)), dtype)
    w = oracle.to_bits(C.normal(rng, (n, k), scale=0.05), dtype)
    stride = ldy or n
    y = torch.full((T, stride), 12345.0, dtype=torch.float32, device="cuda")
    ctx.proj(dev16(w, dtype), dev16(x, dtype), y, T, k, n, ldy)
    torch.cuda.synchronize()
    assert ctx.device_error() == 0
    got = y.cpu().numpy()
    check(got[:, :n], oracle.proj(dtype, w, x, T, k, n))
    if stride > n:
        assert np.all(got[:, n:] == 12345.0), "columns past n were written"


@pytest.mark.parametrize("ctas", [1, 3])
def test_proj_few_ctas(ctx, oracle, ctas):
    """The persistent grid capped at a few CTAs (MAKO_OPT_GRID_CTAS): each CTA works through many output tiles,
    alternating its two TMEM accumulators, so a tile's epilogue overlaps the next tile's products."""
    import mako_attn
    ctx.set_option(mako_attn.OPT_GRID_CTAS, ctas)
    try:
        test_proj_matches_oracle(ctx, oracle, 1000, 1024, 768, 0, 1)
        test_proj_matches_oracle(ctx, oracle, 300, 256, 520, 0, 1)
    finally:
        ctx.set_option(mako_attn.OPT_GRID_CTAS, 0)


def test_attention_then_proj(ctx, oracle):
    """The consumer as the models call it: causal attention with 16-bit output (the reference's to_bf16 of o fused into
    the epilogue), then the projection straight from it; against the oracle's attention rounded to bf16 and its
    double GEMM."""
    import torch
    import mako_attn
    heads, kv_heads, dim, n_q = 4, 2, 128, 256
    case = C.dense_case(seed=70, heads=heads, kv_heads=kv_heads, dim=dim, n_q=n_q, n_k=n_q, dtype=1)
    width = heads * dim
    ctx.set_option(mako_attn.OPT_OUTPUT_16BIT, 1)
    try:
        o16 = torch.zeros((case["q_pad"], width), dtype=torch.bfloat16, device="cuda")
        ctx.attention(dev16(case["q"], 1), dev16(case["k"], 1), dev16(case["v"], 1), o16, n_q, case["q_pad"], n_q,
                      case["k_pad"], heads, kv_heads, 0, C.UINT32_MAX, dim)
    finally:
        ctx.set_option(mako_attn.OPT_OUTPUT_16BIT, 0)
    rng = np.random.default_rng(71)
    n = 384
    w = oracle.to_bits(C.normal(rng, (n, width), scale=0.05), 1)
    y = torch.zeros((n_q, n), dtype=torch.float32, device="cuda")
    ctx.proj(dev16(w, 1), o16, y, n_q, width, n)
    torch.cuda.synchronize()
    # the oracle's path: attention in double, rounded to bf16 (what the 16-bit output stores), then the GEMM
    o_ref = oracle.attention(1, case["q"], case["k"], case["v"], n_q, case["q_pad"], n_q, case["k_pad"], heads,
                             kv_heads, 0, C.UINT32_MAX, dim)
    o_bits = oracle.to_bits(o_ref.astype(np.float32), 1)
    want = oracle.proj(1, w, o_bits, n_q, width, n)
    got = y.cpu().numpy()
    # the 16-bit o may differ from the oracle's rounding by one bf16 ulp where the attention's own error crosses a
    # rounding boundary, so the product is compared at the attention's tolerance
    ok, stats = C.within(got, want, max_abs=2e-2, rel_l2=5e-3, row_rel=1e-2)
    assert ok, stats
    # and exactly what the GEMM makes of the kernel's own 16-bit o
    check(got, oracle.proj(1, w, o16.cpu().view(torch.int16).numpy().view(np.uint16), n_q, width, n))


def test_proj_rejects_k_off_64(ctx):
    import torch
    import mako_attn
    x = torch.zeros((4, 100), dtype=torch.bfloat16, device="cuda")
    w = torch.zeros((8, 100), dtype=torch.bfloat16, device="cuda")
    y = torch.zeros((4, 8), dtype=torch.float32, device="cuda")
    with pytest.raises(mako_attn.MakoError, match="k must be a multiple of 64"):
        ctx.proj(w, x, y, 4, 100, 8)
