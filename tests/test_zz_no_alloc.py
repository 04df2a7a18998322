"""The allocation-free decode entry point, mako_attention_decode_noalloc, against mako_attention_decode.

The entry point exists for callers that cannot call cudaMalloc (device memory wholly committed to a fixed pool or
to a loan, or a loop that cannot let cudaMalloc / cudaFree synchronise the device): its split partials live in a
static device array inside the library instead of context scratch.  This file is named to be collected last, so a
run that stops at its first failure has run every other test before it; it also passes alone in a fresh process.
"""
import numpy as np
import pytest

import attn_cases as C

pytestmark = pytest.mark.gpu


def _dev(bits, dtype):
    import torch
    t = torch.from_numpy(np.ascontiguousarray(bits).view(np.int16))
    return t.view(torch.bfloat16 if dtype == 1 else torch.float16).cuda()


@pytest.mark.parametrize("kw", [
    dict(seed=60, batch=8, heads=32, kv_heads=8, dim=128, lo=16384, hi=32768, dtype=0),  # config 2's shape
    dict(seed=61, batch=3, heads=16, kv_heads=2, dim=128, lo=1, hi=3000, dtype=1),
    dict(seed=62, batch=2, heads=8, kv_heads=8, dim=256, lo=100, hi=900, dtype=0),
], ids=["config2", "bf16-gqa", "d256"])
def test_noalloc_decode_matches_decode(ctx, kw):
    import torch
    import mako_attn
    case = C.decode_case(**kw)
    d = case["dtype"]
    q, k, v = _dev(case["q"], d), _dev(case["k"], d), _dev(case["v"], d)
    lens = torch.from_numpy(case["kv_len"]).cuda()
    max_len = int(case["kv_len"].max())
    shape = (lens.numel(), case["heads"] * case["dim"])
    want = torch.empty(shape, dtype=torch.float32, device="cuda")
    ctx.attention_decode(q, k, v, want, lens, max_len, case["heads"], case["kv_heads"], case["dim"], case["k_stride"])
    torch.cuda.synchronize()
    want = want.cpu().numpy()
    for call in range(2):  # the static array keeps the previous call's contents; results must not depend on them
        got = torch.full(shape, 12345.0, dtype=torch.float32, device="cuda")
        mako_attn.attention_decode_noalloc(q, k, v, got, lens, max_len, case["heads"], case["kv_heads"], case["dim"],
                                           case["k_stride"])
        torch.cuda.synchronize()
        ok, stats = C.within(got.cpu().numpy(), want)
        assert ok, f"call {call}: max-abs {stats[0]:.3e} rel-L2 {stats[1]:.3e} worst-row {stats[2]:.3e}"


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
