"""The allocation-free decode entry point, mako_attention_decode_noalloc, against the oracle and against
mako_attention_decode.

The entry point exists for callers that cannot call cudaMalloc (device memory wholly committed to a fixed pool or
to a loan, or a loop that cannot let cudaMalloc / cudaFree synchronise the device): its split partials live in a
static device array inside the library instead of context scratch.  This file is named to be collected last, so a
run that stops at its first failure has run every other test before it; it also passes alone in a fresh process.
"""
import numpy as np
import pytest

import attn_cases as C

pytestmark = pytest.mark.gpu

SCRATCH_BYTES = 4 << 20  # the library's static array


def _dev(bits, dtype):
    import torch
    t = torch.from_numpy(np.ascontiguousarray(bits).view(np.int16))
    return t.view(torch.bfloat16 if dtype == 1 else torch.float16).cuda()


def default_plan(max_len, batch, kv_heads, heads, sms):
    """mako_attention_decode's split plan (decode_plan in csrc/decode.cu), restated: (keys a split, splits)."""
    group = heads // kv_heads
    rb = (group + 15) // 16
    rows = max_len * batch * kv_heads * rb
    c = -(-rows // (sms * 8))
    c = min(max(C.round_up(c, 64), 256), 2048)
    if max_len > c * 1024:
        c = -(-max_len // 1024)
    c = C.round_up(c, 64)
    return c, (-(-max_len // c) if max_len else 1)


def noalloc_plan(max_len, batch, kv_heads, heads, dim, sms):
    """The no-allocation entry point's plan: the default one, with the smallest chunk (a multiple of 64) whose
    partials fit the array when the default's do not."""
    chunk, ns = default_plan(max_len, batch, kv_heads, heads, sms)
    ns_max = SCRATCH_BYTES // (batch * heads * (dim * 4 + 8))
    if ns > ns_max:
        chunk = C.round_up(-(-max_len // ns_max), 64)
        ns = -(-max_len // chunk)
    return chunk, ns


def _run_both(ctx, oracle, case, chunk=None):
    import torch
    import mako_attn
    d = case["dtype"]
    q, k, v = _dev(case["q"], d), _dev(case["k"], d), _dev(case["v"], d)
    lens = torch.from_numpy(case["kv_len"]).cuda()
    max_len = int(case["kv_len"].max())
    shape = (lens.numel(), case["heads"] * case["dim"])
    # mako_attention_decode, with the same chunk when one is given (bit-identical results then prove the same plan)
    ref = torch.empty(shape, dtype=torch.float32, device="cuda")
    if chunk is not None:
        ctx.set_option(mako_attn.OPT_DECODE_CHUNK, chunk)
    try:
        ctx.attention_decode(q, k, v, ref, lens, max_len, case["heads"], case["kv_heads"], case["dim"],
                             case["k_stride"])
        torch.cuda.synchronize()
    finally:
        ctx.set_option(mako_attn.OPT_DECODE_CHUNK, 0)
    want = oracle.decode(d, case["q"], case["k"], case["v"], case["kv_len"], case["heads"], case["kv_heads"],
                         case["dim"], case["k_stride"])
    outs = []
    for call in range(2):  # the static array keeps the previous call's contents; results must not depend on them
        got = torch.full(shape, 12345.0, dtype=torch.float32, device="cuda")
        mako_attn.attention_decode_noalloc(q, k, v, got, lens, max_len, case["heads"], case["kv_heads"], case["dim"],
                                           case["k_stride"])
        torch.cuda.synchronize()
        g = got.cpu().numpy()
        ok, stats = C.within(g, want)
        assert ok, f"call {call} vs oracle: max-abs {stats[0]:.3e} rel-L2 {stats[1]:.3e} worst-row {stats[2]:.3e}"
        outs.append(g)
    return outs, ref.cpu().numpy()


@pytest.mark.parametrize("kw", [
    dict(seed=60, batch=8, heads=32, kv_heads=8, dim=128, lo=16384, hi=32768, dtype=0),  # config 2's shape
    dict(seed=61, batch=3, heads=16, kv_heads=2, dim=128, lo=1, hi=3000, dtype=1),
    dict(seed=62, batch=2, heads=8, kv_heads=8, dim=256, lo=100, hi=900, dtype=0),
], ids=["config2", "bf16-gqa", "d256"])
def test_noalloc_decode_matches_oracle_and_decode(ctx, oracle, kw):
    case = C.decode_case(**kw)
    outs, ref = _run_both(ctx, oracle, case)
    for g in outs:  # these plans fit the array unchanged: the same kernels on the same plan
        ok, stats = C.within(g, ref)
        assert ok, stats


def test_noalloc_decode_raises_the_chunk_to_fit(ctx, oracle):
    """32 sequences x 64 heads of up to 8000 keys: mako_attention_decode's plan on 148 SMs needs about 9 splits a row
    (about 9.6 MB of partials); the entry point takes splits of about 2700 keys instead (3 a row, 3.2 MB)."""
    import torch
    kw = dict(seed=63, batch=32, heads=64, kv_heads=4, dim=128, lo=6000, hi=8000, dtype=0)
    case = C.decode_case(**kw)
    max_len = int(case["kv_len"].max())
    sms = torch.cuda.get_device_properties(0).multi_processor_count
    chunk0, ns0 = default_plan(max_len, 32, 4, 64, sms)
    assert 32 * 64 * ns0 * (128 * 4 + 8) > SCRATCH_BYTES, "the case must overflow the default plan"
    chunk, ns = noalloc_plan(max_len, 32, 4, 64, 128, sms)
    assert chunk > chunk0 and ns < ns0 and 32 * 64 * ns * (128 * 4 + 8) <= SCRATCH_BYTES
    outs, ref = _run_both(ctx, oracle, case, chunk=chunk)
    for g in outs:  # bit for bit the decode kernel run on the raised chunk: the entry point used that plan
        assert np.array_equal(g, ref)


def test_noalloc_decode_rejects_partials_beyond_the_array(ctx):
    import torch
    import mako_attn
    # 4096 sequences x 32 heads x (4 * 128 + 8) bytes: above the 4 MiB array even with one split per sequence
    q = torch.zeros((4096, 32, 128), dtype=torch.float16, device="cuda")
    kv = torch.zeros((1, 8, 64, 128), dtype=torch.float16, device="cuda")
    lens = torch.zeros(4096, dtype=torch.int32, device="cuda")
    o = torch.zeros((4096, 32 * 128), dtype=torch.float32, device="cuda")
    with pytest.raises(mako_attn.MakoError, match="static scratch"):
        mako_attn.attention_decode_noalloc(q, kv, kv, o, lens, 64, 32, 8, 128, 64)
