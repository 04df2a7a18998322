"""Parity of the CUDA path (through the C ABI) with the CPU oracle on the same seeded inputs.

Tolerance: max-abs <= 2e-3 and relative L2 <= 1e-3 against the double-accumulated oracle,
plus the reference test's worst-row relative L2 < 5e-3 (tests/sparse_attn_test.cpp:181).  Index and mask handling
is exact: cube selections bit for bit, rows outside the output untouched (sentinel 12345,
tests/sparse_attn_test.cpp:86,138-141,182).
"""
import numpy as np
import pytest

import attn_cases as C

pytestmark = pytest.mark.gpu
SENTINEL = 12345.0


def dev(bits, dtype):
    import torch
    t = torch.from_numpy(np.ascontiguousarray(bits).view(np.int16))
    return t.view(torch.bfloat16 if dtype == 1 else torch.float16).cuda()


def dev_raw(a):
    import torch
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def run_dense(ctx, case, kernel=0):
    import torch
    import mako_attn
    ctx.set_option(mako_attn.OPT_PREFILL_KERNEL, kernel)
    q, k, v = dev(case["q"], case["dtype"]), dev(case["k"], case["dtype"]), dev(case["v"], case["dtype"])
    width = case["heads"] * case["dim"]
    o = torch.full((case["q_pad"], width), SENTINEL, dtype=torch.float32, device="cuda")
    ctx.attention(q, k, v, o, case["n_q"], case["q_pad"], case["n_k"], case["k_pad"], case["heads"], case["kv_heads"],
                  case["q_pos0"], case["block"], case["dim"])
    torch.cuda.synchronize()
    return o.cpu().numpy()


def oracle_dense(oracle, case, rows=None):
    return oracle.attention(case["dtype"], case["q"], case["k"], case["v"], case["n_q"], case["q_pad"], case["n_k"],
                            case["k_pad"], case["heads"], case["kv_heads"], case["q_pos0"], case["block"], case["dim"],
                            rows=rows)


DENSE = [
    # config 1 exactly: causal GQA prefill fp16, B1 H16/8 D128 S512, seed 0
    ("config1", dict(seed=0, heads=16, kv_heads=8, dim=128, n_q=512, n_k=512, dtype=0)),
    ("config1-bf16", dict(seed=0, heads=16, kv_heads=8, dim=128, n_q=512, n_k=512, dtype=1)),
    ("ragged-causal", dict(seed=1, heads=4, kv_heads=4, dim=128, n_q=333, n_k=333, dtype=0)),
    ("bidir-gqa", dict(seed=2, heads=8, kv_heads=2, dim=128, n_q=200, n_k=450, block=0, dtype=1)),
    ("block-mask", dict(seed=3, heads=4, kv_heads=2, dim=128, n_q=300, n_k=300, block=77, dtype=0)),
    ("q-offset", dict(seed=4, heads=4, kv_heads=1, dim=128, n_q=70, n_k=600, q_pos0=530, dtype=0)),
    ("d64", dict(seed=5, heads=6, kv_heads=3, dim=64, n_q=257, n_k=257, dtype=0)),
    ("d64-bidir-bf16", dict(seed=6, heads=2, kv_heads=2, dim=64, n_q=130, n_k=130, block=0, dtype=1)),
    ("d64-gqa-long", dict(seed=11, heads=8, kv_heads=2, dim=64, n_q=1100, n_k=1100, dtype=1)),
    ("d64-offset-block", dict(seed=12, heads=4, kv_heads=4, dim=64, n_q=300, n_k=700, q_pos0=400, block=500,
                              dtype=0)),
    ("d256", dict(seed=7, heads=4, kv_heads=2, dim=256, n_q=190, n_k=190, dtype=0)),
    ("d256-bf16", dict(seed=8, heads=2, kv_heads=1, dim=256, n_q=64, n_k=300, block=0, dtype=1)),
    ("d256-gqa-long", dict(seed=13, heads=8, kv_heads=1, dim=256, n_q=900, n_k=900, dtype=1)),
    ("d256-offset-block", dict(seed=14, heads=3, kv_heads=3, dim=256, n_q=200, n_k=650, q_pos0=450, block=520,
                               dtype=0)),
    ("video-rms", dict(seed=9, heads=2, kv_heads=2, dim=128, n_q=1000, n_k=1000, block=0, dtype=1, qk_rms_norm=True)),
    ("config3-scale", dict(seed=10, heads=4, kv_heads=1, dim=128, n_q=700, n_k=700, dtype=1, scale=0.5)),
]


@pytest.mark.parametrize("name,kw", DENSE, ids=[n for n, _ in DENSE])
@pytest.mark.parametrize("kernel", [0, 1, 2], ids=["auto", "mma", "tcgen05"])
def test_dense(ctx, oracle, name, kw, kernel):
    """kernel 0: the default choice (tcgen05), 1: the portable mma.sync kernel, 2: tcgen05 explicitly."""
    case = C.dense_case(**kw)
    got = run_dense(ctx, case, kernel)
    assert ctx.device_error() == 0
    want = oracle_dense(oracle, case)
    ok, stats = C.within(got[:case["n_q"]], want)
    assert ok, f"{name}: max-abs {stats[0]:.3e} rel-L2 {stats[1]:.3e} worst-row {stats[2]:.3e}"
    assert np.all(got[case["n_q"]:] == SENTINEL), "rows past n_q were written"


def test_dense_no_keys_gives_zeros(ctx, oracle):
    case = C.dense_case(seed=12, heads=2, kv_heads=2, dim=128, n_q=64, n_k=0, dtype=0)
    got = run_dense(ctx, case)
    assert np.all(got[:64] == 0.0)


def test_single_query_routes_to_decode(ctx, oracle):
    import mako_attn
    for q_pos0, block in ((799, C.UINT32_MAX), (300, C.UINT32_MAX), (10, 5), (0, 0)):
        case = C.dense_case(seed=13, heads=8, kv_heads=2, dim=128, n_q=1, n_k=800, q_pos0=q_pos0, block=block,
                            dtype=0)
        got = run_dense(ctx, case)
        want = oracle_dense(oracle, case)
        ok, stats = C.within(got[:1], want)
        assert ok, f"pos {q_pos0} block {block}: {stats}"
        ctx.set_option(mako_attn.OPT_DECODE_ROUTE, 0)
        got2 = run_dense(ctx, case)
        ctx.set_option(mako_attn.OPT_DECODE_ROUTE, 1)
        ok, stats = C.within(got2[:1], want)
        assert ok, f"prefill kernel at n_q 1: {stats}"


def run_decode(ctx, case, max_len=None):
    import torch
    d = case["dtype"]
    q, k, v = dev(case["q"], d), dev(case["k"], d), dev(case["v"], d)
    lens = dev_raw(case["kv_len"])
    batch = lens.numel()
    o = torch.full((batch, case["heads"] * case["dim"]), SENTINEL, dtype=torch.float32, device="cuda")
    ctx.attention_decode(q, k, v, o, lens, int(case["kv_len"].max()) if max_len is None else max_len, case["heads"],
                         case["kv_heads"], case["dim"], case["k_stride"])
    torch.cuda.synchronize()
    return o.cpu().numpy()


DECODE = [
    ("config2-short", dict(seed=20, batch=8, heads=32, kv_heads=8, dim=128, lo=1000, hi=3000, dtype=0)),
    ("config2", dict(seed=21, batch=8, heads=32, kv_heads=8, dim=128, lo=16384, hi=32768, dtype=0)),
    ("ragged-tiny", dict(seed=22, batch=5, heads=4, kv_heads=4, dim=128, lo=1, hi=70, dtype=0)),
    ("bf16-gqa", dict(seed=23, batch=3, heads=16, kv_heads=2, dim=128, lo=500, hi=5000, dtype=1)),
    ("d64", dict(seed=24, batch=2, heads=8, kv_heads=1, dim=64, lo=100, hi=2000, dtype=0)),
    ("d256", dict(seed=25, batch=2, heads=4, kv_heads=2, dim=256, lo=100, hi=2000, dtype=1)),
    ("group32", dict(seed=26, batch=2, heads=32, kv_heads=1, dim=128, lo=300, hi=900, dtype=0)),
]


@pytest.mark.parametrize("name,kw", DECODE, ids=[n for n, _ in DECODE])
def test_decode(ctx, oracle, name, kw):
    case = C.decode_case(**kw)
    got = run_decode(ctx, case)
    want = oracle.decode(case["dtype"], case["q"], case["k"], case["v"], case["kv_len"], case["heads"],
                         case["kv_heads"], case["dim"], case["k_stride"])
    ok, stats = C.within(got, want)
    assert ok, f"{name}: max-abs {stats[0]:.3e} rel-L2 {stats[1]:.3e} worst-row {stats[2]:.3e}"


@pytest.mark.parametrize("chunk", [64, 256, 2048])
def test_decode_split_lengths(ctx, oracle, chunk):
    """The same result whatever the split length (many splits through the combine, or one split a sequence)."""
    import mako_attn
    case = C.decode_case(seed=28, batch=4, heads=16, kv_heads=4, dim=128, lo=100, hi=9000, dtype=0)
    ctx.set_option(mako_attn.OPT_DECODE_CHUNK, chunk)
    try:
        got = run_decode(ctx, case)
    finally:
        ctx.set_option(mako_attn.OPT_DECODE_CHUNK, 0)
    want = oracle.decode(0, case["q"], case["k"], case["v"], case["kv_len"], 16, 4, 128, case["k_stride"])
    ok, stats = C.within(got, want)
    assert ok, f"chunk {chunk}: {stats}"


def test_decode_zero_length_gives_zeros(ctx, oracle):
    case = C.decode_case(seed=27, batch=3, heads=4, kv_heads=2, dim=128, lo=10, hi=20, dtype=0)
    case["kv_len"][1] = 0
    got = run_decode(ctx, case)
    assert np.all(got[1] == 0.0)
    want = oracle.decode(0, case["q"], case["k"], case["v"], case["kv_len"], 4, 2, 128, case["k_stride"])
    assert C.within(got, want)[0]


@pytest.mark.parametrize("cap", [0, 700, 2500])
def test_decode_lengths_beyond_max_kv_len(ctx, oracle, cap):
    """A kv_len entry above max_kv_len is read as max_kv_len: no key past it is read (the split plan covers max_kv_len
    keys) and every o row is still written -- 0 when max_kv_len is 0."""
    case = C.decode_case(seed=29, batch=4, heads=8, kv_heads=2, dim=128, lo=300, hi=4000, dtype=0)
    got = run_decode(ctx, case, max_len=cap)
    assert not np.any(got == SENTINEL)
    capped = np.minimum(case["kv_len"], cap).astype(np.int32)
    want = oracle.decode(0, case["q"], case["k"], case["v"], capped, 8, 2, 128, case["k_stride"])
    if cap == 0:
        assert np.all(got == 0.0)
    ok, stats = C.within(got, want)
    assert ok, f"cap {cap}: {stats}"


def sparse_fixture_run(ctx, oracle, dtype=0, topk=3, local=0, stride=0, kernel=0):
    import torch
    import mako_attn
    ctx.set_option(mako_attn.OPT_PREFILL_KERNEL, kernel)
    fx = oracle.sparse_test_fixture()
    q, k, v = dev(fx["q"], dtype), dev(fx["k"], dtype), dev(fx["v"], dtype)
    cnt = dev_raw(fx["cnt"])
    valid, map_ = dev_raw(fx["valid"]), dev_raw(fx["map"])
    sel_t, nsel_t = ctx.cube_select(q, k, 2, 448, 512, 6, cnt, topk, local, stride)
    o = torch.full((448, 256), SENTINEL, dtype=torch.float32, device="cuda")
    ctx.attention_sparse(q, k, v, o, 444, 448, 444, 512, 2, 2, 256, 6, topk, 384, 444, sel_t, nsel_t, valid, map_)
    torch.cuda.synchronize()
    sel = sel_t.cpu().numpy().view(np.uint16)
    nsel = nsel_t.cpu().numpy().view(np.uint16)
    return fx, sel, nsel, o.cpu().numpy()


@pytest.mark.parametrize("kernel", [0, 1], ids=["auto", "mma"])
def test_sparse_reference_fixture(ctx, oracle, kernel):
    """tests/sparse_attn_test.cpp re-run through the C ABI: selection exact (vs the fp32 restatement and the
    reference's double procedure), attention within tolerance, unmapped rows untouched."""
    fx, sel, nsel, o = sparse_fixture_run(ctx, oracle, kernel=kernel)
    assert ctx.device_error() == 0
    want_sel, want_nsel, *_ = oracle.cube_select(0, fx["q"], fx["k"], 2, 448, 512, 6, fx["cnt"], 3, mode=1)
    dbl_sel, *_ = oracle.cube_select(0, fx["q"], fx["k"], 2, 448, 512, 6, fx["cnt"], 3, mode=0)
    np.testing.assert_array_equal(sel, want_sel)
    np.testing.assert_array_equal(sel, dbl_sel)
    np.testing.assert_array_equal(nsel, want_nsel)
    want = np.full((448, 256), SENTINEL, np.float32)
    oracle.attention_sparse(0, fx["q"], fx["k"], fx["v"], 444, 448, 444, 512, 2, 2, 256, 6, 3, 384, 444, sel, nsel,
                            fx["valid"], fx["map"], out=want)
    mapped = np.array([r for r in range(444) if fx["map"][r] >= 0])
    ok, stats = C.within(o[mapped], want[mapped])
    assert ok, f"max-abs {stats[0]:.3e} rel-L2 {stats[1]:.3e} worst-row {stats[2]:.3e}"
    untouched = [r for r in range(448) if r >= 444 or fx["map"][r] < 0]
    assert np.all(o[untouched] == SENTINEL)


def test_sparse_local_cubes(ctx, oracle):
    fx, sel, nsel, _ = sparse_fixture_run(ctx, oracle, topk=4, local=3, stride=1)
    want, *_ = oracle.cube_select(0, fx["q"], fx["k"], 2, 448, 512, 6, fx["cnt"], 4, local=3, stride=1)
    np.testing.assert_array_equal(sel, want)


def test_cube_select_large_bit_exact(ctx, oracle):
    """Many cubes, partial cubes, bf16: the selection equals the fp32 restatement bit for bit."""
    import torch
    rng = np.random.default_rng(30)
    heads, n_cubes, topk = 3, 300, 40
    n = n_cubes * 64
    cnt = rng.integers(1, 65, size=n_cubes).astype(np.uint32)
    cnt[::7] = 64
    valid = np.zeros(n, np.uint8)
    for c in range(n_cubes):
        valid[c * 64:c * 64 + cnt[c]] = 1
    for dtype in (0, 1):
        x = C.normal(rng, (2, heads, n, 128)) * valid[None, None, :, None]
        q, k = oracle.to_bits(x[0], dtype), oracle.to_bits(x[1], dtype)
        sel_t, _ = ctx.cube_select(dev(q, dtype), dev(k, dtype), heads, n, n, n_cubes, dev_raw(cnt), topk, 1, 0)
        torch.cuda.synchronize()
        sel = sel_t.cpu().numpy().view(np.uint16)
        want, *_ = oracle.cube_select(dtype, q, k, heads, n, n, n_cubes, cnt, topk, local=1, mode=1)
        np.testing.assert_array_equal(sel, want)


def planted_cubes(seed, n_cubes):
    """One head of n_cubes full cubes, fp16, N(0, 1) with planted edge cases: key cubes 100, 2000 and n - 1 copies of
    key cube 5, and 8..10 copies of 7 (tied scores in every row); query cube 3 is -inf in dimension 0 and 0 elsewhere
    (its scores are +inf or -inf by the sign of the key cube's dimension 0: tied +inf candidates, -inf never picked);
    query cube 11 is NaN (no candidate: every pick after the local ones is cube 0); cube 9 is empty (cnt 0, zero
    rows: a row and a column of zero scores, all tied)."""
    rng = np.random.default_rng(seed)
    n = n_cubes * 64
    x = C.normal(rng, (2, 1, n, 128))
    q, k = x[0], x[1]
    cube = lambda t, c: t[0, c * 64:(c + 1) * 64]  # noqa: E731
    for c in (100, 2000, n_cubes - 1):
        cube(k, c)[:] = cube(k, 5)
    for c in (8, 9, 10):
        cube(k, c)[:] = cube(k, 7)
    cube(q, 3)[:] = 0.0
    cube(q, 3)[:, 0] = -np.inf
    cube(q, 11)[:] = np.nan
    cube(q, 9)[:] = 0.0
    cube(k, 9)[:] = 0.0
    cnt = np.full(n_cubes, 64, np.uint32)
    cnt[9] = 0
    return oracle_bits(q, 0), oracle_bits(k, 0), cnt


@pytest.mark.parametrize("local,stride", [(0, 0), (3, 256), (3, 0)], ids=["by-score", "local3", "local3-stride0"])
def test_cube_topk_at_the_reference_bound(ctx, oracle, local, stride):
    """4096 cubes (the reference's limit, src/models/runtime.cpp:290) with H3's top-k, ceil(0.15 * 4096) = 615
    (src/models/h3.cpp:520), and the planted ties, infinities, NaNs and empty cube of planted_cubes: the selection
    equals the fp32 restatement's repeated argmax bit for bit."""
    import torch
    n_cubes, topk = 4096, 615
    n = n_cubes * 64
    q, k, cnt = planted_cubes(31, n_cubes)
    want, want_n, _, _, sc = oracle.cube_select(0, q, k, 1, n, n, n_cubes, cnt, topk, local, stride, mode=1)
    # the planted cases reach the selection as intended
    assert np.array_equal(sc[0, :, 5], sc[0, :, 100], equal_nan=True)
    assert np.array_equal(sc[0, :, 7], sc[0, :, 10], equal_nan=True)
    assert np.any(sc[0, 3] == np.inf) and np.any(sc[0, 3] == -np.inf)
    assert np.all(np.isnan(sc[0, 11])) and np.all(sc[0, 9] == 0.0)
    sel_t, nsel_t = ctx.cube_select(dev(q, 0), dev(k, 0), 1, n, n, n_cubes, dev_raw(cnt), topk, local, stride)
    torch.cuda.synchronize()
    sel, nsel = sel_t.cpu().numpy().view(np.uint16), nsel_t.cpu().numpy().view(np.uint16)
    np.testing.assert_array_equal(nsel, want_n)
    np.testing.assert_array_equal(sel, want)
    nf = 0 if not local else 1 + (11 >= stride) + (11 + stride < n_cubes)  # query cube 11's forced entries
    assert np.all(sel[0, 11, nf:] == 0)  # nothing above -inf: cube 0 repeated


@pytest.mark.parametrize("kernel", [0, 1], ids=["auto", "mma"])
def test_block_sparse_lists(ctx, oracle, kernel):
    """Config 4's mask format (int32 sorted kept-block lists + counts) at a reduced length."""
    import torch
    import mako_attn
    ctx.set_option(mako_attn.OPT_PREFILL_KERNEL, kernel)
    heads, n, dtype = 4, 2048, 1
    nb = n // 64
    lists, counts = C.block_lists(40, heads, nb, 0.15)
    counts[1, 3] = 0  # a query block that keeps nothing: zeros
    case = C.dense_case(seed=41, heads=heads, kv_heads=heads, dim=128, n_q=n, n_k=n, dtype=dtype)
    q, k, v = dev(case["q"], dtype), dev(case["k"], dtype), dev(case["v"], dtype)
    o = torch.full((n, heads * 128), SENTINEL, dtype=torch.float32, device="cuda")
    ctx.attention_block_sparse(q, k, v, o, n, heads, heads, dev_raw(lists), dev_raw(counts))
    torch.cuda.synchronize()
    got = o.cpu().numpy()
    want = oracle.attention_sparse(dtype, case["q"], case["k"], case["v"], n, case["q_pad"], n, case["k_pad"], heads,
                                   heads, heads * 128, nb, lists.shape[-1], n, n, lists.astype(np.uint16),
                                   counts.astype(np.uint16), np.ones(case["k_pad"], np.uint8),
                                   np.arange(case["q_pad"], dtype=np.int32))[:n]
    ok, stats = C.within(got, want)
    assert ok, f"max-abs {stats[0]:.3e} rel-L2 {stats[1]:.3e} worst-row {stats[2]:.3e}"
    assert np.all(got[3 * 64:4 * 64, 128:256] == 0.0)
    assert ctx.device_error() == 0
    ctx.set_option(mako_attn.OPT_PREFILL_KERNEL, 0)


@pytest.mark.parametrize("dtype", [0, 1])
def test_block_sparse_irregular_lists(ctx, oracle, dtype):
    """Lists of different lengths within a tile (the shorter one padded with empty passes), a repeated entry (counted
    twice, as the reference's pass list does), entries >= n_cubes (skipped), an odd block count and GQA."""
    import torch
    heads, kv_heads, n = 4, 2, 1344  # 21 blocks: the last tile's second cube does not exist
    nb = n // 64
    rng = np.random.default_rng(90 + dtype)
    max_list = 9
    lists = rng.integers(0, nb, size=(heads, nb, max_list)).astype(np.int32)
    counts = rng.integers(0, max_list + 1, size=(heads, nb)).astype(np.int32)
    lists[0, 0, :3] = [5, 5, 5]
    counts[0, 0] = 3
    lists[1, 2, 1] = nb + 7  # out of range: skipped
    lists[2, 4, 0] = 70000
    counts[1, 2] = max(counts[1, 2], 2)
    counts[2, 4] = max(counts[2, 4], 1)
    counts[3, 5] = -4  # a negative count keeps nothing
    case = C.dense_case(seed=91, heads=heads, kv_heads=kv_heads, dim=128, n_q=n, n_k=n, dtype=dtype)
    case["k"], case["v"], case["k_pad"] = case["k"][:, :n], case["v"][:, :n], n  # this form's rows: [kv_heads][n]
    q, k, v = dev(case["q"], dtype), dev(case["k"], dtype), dev(case["v"], dtype)
    o = torch.full((n, heads * 128), SENTINEL, dtype=torch.float32, device="cuda")
    ctx.attention_block_sparse(q, k, v, o, n, heads, kv_heads, dev_raw(lists), dev_raw(counts))
    torch.cuda.synchronize()
    assert ctx.device_error() == 0
    got = o.cpu().numpy()
    sel = np.where(lists >= 0, np.minimum(lists, 65535), 65535).astype(np.uint16)
    nsel = np.clip(counts, 0, None).astype(np.uint16)
    want = oracle.attention_sparse(dtype, case["q"], case["k"], case["v"], n, case["q_pad"], n, case["k_pad"], heads,
                                   kv_heads, heads * 128, nb, max_list, n, n, sel, nsel,
                                   np.ones(case["k_pad"], np.uint8), np.arange(case["q_pad"], dtype=np.int32))[:n]
    ok, stats = C.within(got, want)
    assert ok, f"max-abs {stats[0]:.3e} rel-L2 {stats[1]:.3e} worst-row {stats[2]:.3e}"
    assert np.all(got[5 * 64:6 * 64, 3 * 128:4 * 128] == 0.0)


def ramp_keys(k_bits, dtype, n_k, block_rows, top):
    """K rows scaled up key block by key block (factor 1 at the first block to `top` at the last), so that a row's
    running maximum rises by more than the lazy-rescale threshold (8 in log2 units) several times along its keys:
    the rescale of O and, in the kernels that split a row's passes over two warpgroups, the hand-over of the maximum
    between them are exercised."""
    import oracle as O
    k = O.from_bits(k_bits, dtype)
    blocks = np.arange(k.shape[1]) // block_rows
    last = max(1, (n_k - 1) // block_rows)
    fac = 1.0 + (top - 1.0) * np.minimum(blocks, last) / last
    return O.to_bits(k * fac[None, :, None].astype(np.float32), dtype)


@pytest.mark.parametrize("dim", [128, 256])
@pytest.mark.parametrize("dtype", [0, 1])
def test_dense_rising_scores(ctx, oracle, dim, dtype):
    """Causal prefill whose scores grow along the keys (the running maximum is raised mid-row, O rescaled)."""
    case = C.dense_case(seed=140 + dim + dtype, heads=4, kv_heads=2, dim=dim, n_q=1000, n_k=1000, dtype=dtype)
    case["k"] = ramp_keys(case["k"], dtype, case["n_k"], 64, 10.0)
    got = run_dense(ctx, case)
    assert ctx.device_error() == 0
    want = oracle_dense(oracle, case)
    ok, stats = C.within(got[:case["n_q"]], want)
    assert ok, f"max-abs {stats[0]:.3e} rel-L2 {stats[1]:.3e} worst-row {stats[2]:.3e}"


@pytest.mark.parametrize("dtype", [0, 1])
def test_block_sparse_rising_scores(ctx, oracle, dtype):
    """Block-sparse lists (ascending) over keys whose scores grow cube by cube: the running maximum handed from
    pass to pass is raised several times within a row, and O is rescaled between the two parities' products."""
    import torch
    heads, n = 2, 2048
    nb = n // 64
    lists, counts = C.block_lists(150 + dtype, heads, nb, 0.3)
    case = C.dense_case(seed=151 + dtype, heads=heads, kv_heads=heads, dim=128, n_q=n, n_k=n, dtype=dtype)
    case["k"] = ramp_keys(case["k"], dtype, n, 64, 10.0)
    q, k, v = dev(case["q"], dtype), dev(case["k"], dtype), dev(case["v"], dtype)
    o = torch.full((n, heads * 128), SENTINEL, dtype=torch.float32, device="cuda")
    ctx.attention_block_sparse(q, k, v, o, n, heads, heads, dev_raw(lists), dev_raw(counts))
    torch.cuda.synchronize()
    assert ctx.device_error() == 0
    got = o.cpu().numpy()
    want = oracle.attention_sparse(dtype, case["q"], case["k"], case["v"], n, case["q_pad"], n, case["k_pad"], heads,
                                   heads, heads * 128, nb, lists.shape[-1], n, n, lists.astype(np.uint16),
                                   counts.astype(np.uint16), np.ones(case["k_pad"], np.uint8),
                                   np.arange(case["q_pad"], dtype=np.int32))[:n]
    ok, stats = C.within(got, want)
    assert ok, f"max-abs {stats[0]:.3e} rel-L2 {stats[1]:.3e} worst-row {stats[2]:.3e}"


V_FACTORS = (2.0 ** -24, 2.0 ** -3, 1.0, 2.0 ** 18)  # per kv head: tiny, at the unscaled range's edge, plain, huge


def scale_v_heads(v_bits, dtype, factors):
    """V of kv head i multiplied by factors[i] (exact in the 16-bit type: powers of two)."""
    import oracle as O
    v = O.from_bits(v_bits, dtype)
    return O.to_bits(v * np.asarray(factors, np.float32)[:, None, None], dtype)


def per_head(o, heads, dim, kv_of, factors):
    """o's columns of head h divided by its kv head's factor, so that one tolerance applies to every head."""
    o = np.array(o, np.float64)
    for h in range(heads):
        o[..., h * dim:(h + 1) * dim] /= factors[kv_of(h)]
    return o


@pytest.mark.parametrize("dim", [128, 256])
def test_bf16_v_magnitudes(ctx, oracle, dim):
    """bf16 V whose kv heads span 2^-24 .. 2^18: the fp16 copy P.V reads keeps heads in range unscaled and
    converts the others with a power of two, head by head; every head's output within tolerance of the oracle."""
    heads, kvh = 8, len(V_FACTORS)
    case = C.dense_case(seed=160 + dim, heads=heads, kv_heads=kvh, dim=dim, n_q=700, n_k=900, dtype=1)
    case["v"] = scale_v_heads(case["v"], 1, V_FACTORS)
    got = run_dense(ctx, case)
    assert ctx.device_error() == 0
    want = oracle_dense(oracle, case)
    kv_of = lambda h: h // (heads // kvh)
    ok, stats = C.within(per_head(got[:case["n_q"]], heads, dim, kv_of, V_FACTORS),
                         per_head(want, heads, dim, kv_of, V_FACTORS))
    assert ok, f"max-abs {stats[0]:.3e} rel-L2 {stats[1]:.3e} worst-row {stats[2]:.3e}"


def test_block_sparse_bf16_v_magnitudes(ctx, oracle):
    """The block-sparse path's fp16 copy of V, heads from 2^-24 to 2^18 (see test_bf16_v_magnitudes)."""
    import torch
    heads, n = len(V_FACTORS), 1024
    nb = n // 64
    lists, counts = C.block_lists(170, heads, nb, 0.3)
    case = C.dense_case(seed=171, heads=heads, kv_heads=heads, dim=128, n_q=n, n_k=n, dtype=1)
    case["v"] = scale_v_heads(case["v"], 1, V_FACTORS)
    q, k, v = dev(case["q"], 1), dev(case["k"], 1), dev(case["v"], 1)
    o = torch.full((n, heads * 128), SENTINEL, dtype=torch.float32, device="cuda")
    ctx.attention_block_sparse(q, k, v, o, n, heads, heads, dev_raw(lists), dev_raw(counts))
    torch.cuda.synchronize()
    assert ctx.device_error() == 0
    want = oracle.attention_sparse(1, case["q"], case["k"], case["v"], n, case["q_pad"], n, case["k_pad"], heads,
                                   heads, heads * 128, nb, lists.shape[-1], n, n, lists.astype(np.uint16),
                                   counts.astype(np.uint16), np.ones(case["k_pad"], np.uint8),
                                   np.arange(case["q_pad"], dtype=np.int32))[:n]
    kv_of = lambda h: h
    ok, stats = C.within(per_head(o.cpu().numpy(), heads, 128, kv_of, V_FACTORS),
                         per_head(want, heads, 128, kv_of, V_FACTORS))
    assert ok, f"max-abs {stats[0]:.3e} rel-L2 {stats[1]:.3e} worst-row {stats[2]:.3e}"


def h3_layout(seed, frames, ph, pw, dense, heads, kv_heads, dtype):
    """A cube layout as H3 builds it (src/models/h3.cpp:510-546), from the library's mako_cube_layout: 4x4x4 cubes
    over (frame, patch row, patch column) with partial cubes at the grid edges (their rows scattered, not leading),
    then the dense rows; map sends each tile row to its model row (video rows after the dense ones)."""
    import mako_attn
    rng = np.random.default_rng(seed)
    map_, valid, cnt, info = mako_attn.cube_layout(frames, ph, pw, ph * pw, dense, dense, 0.15)
    n_cubes, vrows, rows, q_pad, k_pad = info.n_cubes, info.dense0, info.rows, info.q_pad, info.k_pad
    x = C.normal(rng, (3, max(heads, kv_heads), k_pad, 128)) * valid[None, None, :, None]
    q = oracle_bits(x[0, :heads, :q_pad], dtype)
    k = oracle_bits(x[1, :kv_heads], dtype)
    v = oracle_bits(x[2, :kv_heads], dtype)
    n_out = dense + frames * ph * pw
    return dict(q=q, k=k, v=v, valid=valid, map=map_, cnt=cnt, n_cubes=n_cubes, rows=rows, q_pad=q_pad,
                k_pad=k_pad, dense0=vrows, dense1=rows, n_out=n_out, heads=heads, kv_heads=kv_heads, dtype=dtype)


def oracle_bits(x, dtype):
    import oracle as O
    return O.to_bits(x, dtype)


@pytest.mark.parametrize("kernel", [0, 1], ids=["auto", "mma"])
@pytest.mark.parametrize("dtype", [0, 1])
def test_sparse_h3_layout(ctx, oracle, kernel, dtype):
    """Odd cube count (a tile half with no cube), partial edge cubes, dense rows, a permuted output map, GQA, the
    local option -- cube_select then attention_sparse against the oracle."""
    import torch
    import mako_attn
    L = h3_layout(70 + dtype, frames=3, ph=10, pw=10, dense=100, heads=4, kv_heads=2, dtype=dtype)
    assert L["n_cubes"] % 2 == 1
    topk = 3
    q, k, v = dev(L["q"], dtype), dev(L["k"], dtype), dev(L["v"], dtype)
    # cube_select pools q and k of the same head, so it runs on a kv-head-wide copy of q's first heads
    sel_t, nsel_t = ctx.cube_select(q[:2], k, 2, L["q_pad"], L["k_pad"], L["n_cubes"], dev_raw(L["cnt"]), topk, 1, 0)
    sel2 = sel_t.cpu().numpy().view(np.uint16)
    want_sel, *_ = oracle.cube_select(dtype, L["q"][:2], L["k"], 2, L["q_pad"], L["k_pad"], L["n_cubes"], L["cnt"],
                                      topk, local=1, mode=1)
    np.testing.assert_array_equal(sel2, want_sel)
    # per-head selection for all 4 q heads: heads 2, 3 reuse heads 0, 1's lists (any list is a valid input)
    sel = np.concatenate([sel2, sel2], axis=0)
    nsel = np.concatenate([nsel_t.cpu().numpy().view(np.uint16)] * 2, axis=0)
    ctx.set_option(mako_attn.OPT_PREFILL_KERNEL, kernel)
    width = 4 * 128
    o = torch.full((L["n_out"] + 3, width), SENTINEL, dtype=torch.float32, device="cuda")
    ctx.attention_sparse(q, k, v, o, L["rows"], L["q_pad"], L["rows"], L["k_pad"], 4, 2, width, L["n_cubes"], topk,
                         L["dense0"], L["dense1"], dev_raw(sel), dev_raw(nsel), dev_raw(L["valid"]), dev_raw(L["map"]))
    torch.cuda.synchronize()
    ctx.set_option(mako_attn.OPT_PREFILL_KERNEL, 0)
    assert ctx.device_error() == 0
    got = o.cpu().numpy()
    want = np.full((L["n_out"] + 3, width), SENTINEL, np.float32)
    oracle.attention_sparse(dtype, L["q"], L["k"], L["v"], L["rows"], L["q_pad"], L["rows"], L["k_pad"], 4, 2, width,
                            L["n_cubes"], topk, L["dense0"], L["dense1"], sel, nsel, L["valid"], L["map"], out=want)
    ok, stats = C.within(got[:L["n_out"]], want[:L["n_out"]])
    assert ok, f"max-abs {stats[0]:.3e} rel-L2 {stats[1]:.3e} worst-row {stats[2]:.3e}"
    assert np.all(got[L["n_out"]:] == SENTINEL)


# The persistent kernels take one work item per CTA on the small problems above (fewer items than SMs); with the grid
# capped at a few CTAs each CTA works through many items, so the state carried from one item to the next (barrier
# phases, the next item's Q, the epilogue overlapping the next item's first products) is exercised too.
FEW_CTAS = 3


@pytest.fixture
def few_ctas(ctx):
    import mako_attn
    ctx.set_option(mako_attn.OPT_GRID_CTAS, FEW_CTAS)
    yield
    ctx.set_option(mako_attn.OPT_GRID_CTAS, 0)


@pytest.mark.parametrize("name,kw", [c for c in DENSE if c[0] in ("config1", "ragged-causal", "bidir-gqa", "block-mask",
                                                                    "q-offset", "d64-gqa-long", "d256", "d256-gqa-long",
                                                                    "d256-offset-block")],
                         ids=lambda c: c if isinstance(c, str) else "")
def test_dense_few_ctas(ctx, oracle, few_ctas, name, kw):
    test_dense(ctx, oracle, name, kw, 0)


@pytest.mark.parametrize("dim", [128, 256])
def test_dense_rising_scores_few_ctas(ctx, oracle, few_ctas, dim):
    test_dense_rising_scores(ctx, oracle, dim, 1)


def test_block_sparse_few_ctas(ctx, oracle, few_ctas):
    test_block_sparse_lists(ctx, oracle, 0)
    test_block_sparse_rising_scores(ctx, oracle, 1)


@pytest.mark.parametrize("dtype", [0, 1])
def test_block_sparse_irregular_few_ctas(ctx, oracle, few_ctas, dtype):
    test_block_sparse_irregular_lists(ctx, oracle, dtype)


def test_sparse_h3_layout_few_ctas(ctx, oracle, few_ctas):
    test_sparse_h3_layout(ctx, oracle, 0, 1)


def test_sparse_reference_fixture_few_ctas(ctx, oracle, few_ctas):
    test_sparse_reference_fixture(ctx, oracle, 0)


def test_argument_errors(ctx):
    import torch
    import mako_attn
    q = torch.zeros(64 * 128, dtype=torch.float16, device="cuda")
    o = torch.zeros(64 * 128, dtype=torch.float32, device="cuda")
    with pytest.raises(mako_attn.MakoError, match="heads of 96"):
        ctx.attention(q, q, q, o, 10, 64, 10, 64, 1, 1, 0, 0, 96)
    with pytest.raises(mako_attn.MakoError, match="q_pad"):
        ctx.attention(q, q, q, o, 10, 32, 10, 64, 1, 1, 0, 0, 128)
    with pytest.raises(mako_attn.MakoError, match="cube_select"):
        ctx.cube_select(q, q, 1, 64, 128, 5000, o, 3)
    with pytest.raises(mako_attn.MakoError, match="multiple of 64"):
        ctx.attention_sparse(q, q, q, o, 10, 60, 10, 128, 1, 1, 128, 0, 1, 0, 10, None, None, o, o)
