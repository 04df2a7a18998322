"""The head-tile producers (TransformerRuntime::heads / heads_norm / heads_partial, src/models/runtime.cpp:215-260,
and heads_clear) through the C ABI against the oracle's double restatement, rounded to the tile's 16-bit type.

Bar: every element within one unit in the last place of the 16-bit result, or within 1e-5 where the result nearly
cancels (a rotation u c - v s of inputs of a few units: fp32 rounding of the terms then exceeds an ulp of the tiny
result), since the device computes in fp32 with its own summation order and fused multiply-adds and the oracle in
double; at least 99% of the elements bit-identical; rows outside the written range untouched (sentinel)."""
import numpy as np
import pytest

import attn_cases as C

pytestmark = pytest.mark.gpu


def tdev(a):
    import torch
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def y_tile(heads, n_pad, dim, dtype, fill=0x7BFF):
    import torch
    t = torch.full((heads, n_pad, dim), fill, dtype=torch.int16, device="cuda")
    return t.view(torch.bfloat16 if dtype == 1 else torch.float16)


def bits(t):
    import torch
    return t.view(torch.int16).cpu().numpy().view(np.uint16)


def ulp_check(got_bits, want_f32, dtype, mask=None):
    import oracle as O
    want_bits = O.to_bits(want_f32, dtype)
    g = O.from_bits(got_bits, dtype).astype(np.float64)
    w = O.from_bits(want_bits, dtype).astype(np.float64)
    if mask is not None:
        g, w, gb, wb = g[mask], w[mask], got_bits[mask], want_bits[mask]
    else:
        gb, wb = got_bits, want_bits
    # one ulp of the 16-bit type at the reference value's magnitude
    mant = 7 if dtype == 1 else 10
    e = np.floor(np.log2(np.maximum(np.abs(w), 2.0 ** -14)))
    ulp = 2.0 ** (e - mant)
    far = np.abs(g - w) > np.maximum(ulp * 1.0001, 1e-5)
    exact = float(np.mean(gb == wb)) if gb.size else 1.0
    return int(far.sum()), exact


def angles(rng, rows, pairs):
    a = rng.uniform(-np.pi, np.pi, size=(rows, pairs))
    return np.stack([np.cos(a), np.sin(a)], axis=-1).astype(np.float32)


PARTIAL = [
    # qwen text q: gated layout (stride 2 D), full-width norm, partial rotation
    ("qwen-q", dict(dim=128, heads=4, stride=256, col0=0, rot=32, norm=True, T=70, n_pad=128, dtype=0)),
    # h3: 128-wide heads, 96 rotated, norm, permuted map with empty rows
    ("h3-mapped", dict(dim=128, heads=3, stride=128, col0=384, rot=96, norm=True, T=96, n_pad=128, dtype=1, map=True)),
    # v tiles: no norm, no rotation
    ("v", dict(dim=128, heads=2, stride=128, col0=256, rot=0, norm=False, T=33, n_pad=64, dtype=0)),
    # other widths: 64, 96 (scalar loads), 256
    ("d64", dict(dim=64, heads=2, stride=64, col0=0, rot=64, norm=True, T=40, n_pad=64, dtype=1)),
    ("d96-unaligned", dict(dim=96, heads=2, stride=100, col0=3, rot=48, norm=True, T=17, n_pad=32, dtype=0)),
    ("d256", dict(dim=256, heads=2, stride=256, col0=0, rot=128, norm=True, T=50, n_pad=64, dtype=1)),
]


@pytest.mark.parametrize("name,kw", PARTIAL, ids=[n for n, _ in PARTIAL])
def test_heads_partial(ctx, oracle, name, kw):
    rng = np.random.default_rng(hash(name) % 2 ** 32)
    dim, H, stride, col0, rot, T, n_pad, dtype = (kw[k] for k in ("dim", "heads", "stride", "col0", "rot", "T",
                                                                  "n_pad", "dtype"))
    ld = col0 + stride * H + 5
    src_rows = T + 7
    x = (rng.standard_normal((src_rows, ld)) * 3.0).astype(np.float32)
    cs = angles(rng, src_rows, max(rot // 2, 1))
    w = rng.uniform(0.5, 1.5, dim).astype(np.float32) if kw["norm"] else None
    m = None
    if kw.get("map"):
        m = rng.permutation(src_rows)[:T].astype(np.int32)
        m[::9] = -1
    y = y_tile(H, n_pad, dim, dtype)
    ctx.heads_partial(tdev(x), ld, col0, stride, dim, rot, H, T, n_pad, tdev(cs) if rot else None,
                      tdev(w) if w is not None else None, 1e-6, y, tdev(m) if m is not None else None)
    import torch
    torch.cuda.synchronize()
    got = bits(y)
    want = oracle.heads(x, ld, col0, stride, dim, rot, 1 if rot else 0, T, H, n_pad, cs=cs, cs_row=rot // 2, w=w,
                        eps=1e-6 if kw["norm"] else 0.0, map_=m)
    far, exact = ulp_check(got[:, :T], want[:, :T], dtype)
    assert far == 0 and exact >= 0.99, f"{far} elements beyond one ulp, {exact:.4f} bit-identical"
    assert np.all(got[:, T:] == 0x7BFF), "rows past T are the caller's"
    if m is not None:
        assert np.all(got[:, :T][:, m < 0] == 0), "rows the map leaves empty are zero"


@pytest.mark.parametrize("rope", [0, 1, 2])
@pytest.mark.parametrize("dtype", [0, 1])
def test_heads_and_clear(ctx, oracle, rope, dtype):
    import torch
    rng = np.random.default_rng(100 + rope + 3 * dtype)
    H, T, n_pad, ld, col0 = 3, 45, 128, 3 * 128 + 64, 64
    x = rng.standard_normal((T, ld)).astype(np.float32)
    cs = angles(rng, T, 64)
    y = y_tile(H, n_pad, 128, dtype)
    ctx.heads(tdev(x), ld, col0, H, T, n_pad, tdev(cs) if rope else None, rope, y)
    torch.cuda.synchronize()
    got = bits(y)
    want = oracle.heads(x, ld, col0, 128, 128, 128, rope, T, H, n_pad, cs=cs, cs_row=64)
    far, exact = ulp_check(got[:, :T], want[:, :T], dtype)
    assert far == 0 and exact >= 0.99, (far, exact)
    assert np.all(got[:, T:] == 0), "heads() zeroes the rows past T"


def test_heads_norm_rows_from_row0(ctx, oracle):
    import torch
    rng = np.random.default_rng(7)
    H, T, n_pad, row0, ld = 2, 20, 64, 30, 256
    x = rng.standard_normal((T, ld)).astype(np.float32) * 5
    cs = angles(rng, T, 64)
    w = rng.uniform(0.5, 1.5, 128).astype(np.float32)
    y = y_tile(H, n_pad, 128, 0)
    ctx.heads_norm(tdev(x), ld, 0, H, T, n_pad, tdev(cs), 2, tdev(w), 1e-5, row0, y)
    torch.cuda.synchronize()
    got = bits(y)
    want = oracle.heads(x, ld, 0, 128, 128, 128, 2, T, H, n_pad, row0=row0, cs=cs, cs_row=64, w=w, eps=1e-5)
    far, exact = ulp_check(got[:, row0:row0 + T], want[:, row0:row0 + T], 0)
    assert far == 0 and exact >= 0.99, (far, exact)
    assert np.all(got[:, :row0] == 0x7BFF) and np.all(got[:, row0 + T:] == 0x7BFF)


def test_heads_clear_and_errors(ctx):
    import torch
    import mako_attn
    y = y_tile(3, 64, 96, 1)
    ctx.heads_clear(y, 96, 64, 40, 3)
    torch.cuda.synchronize()
    got = bits(y)
    assert np.all(got[:, 40:] == 0) and np.all(got[:, :40] == 0x7BFF)
    x = torch.zeros(1024, dtype=torch.float32, device="cuda")
    with pytest.raises(mako_attn.MakoError, match="heads of 300 with 0 rotated"):
        ctx.heads_partial(x, 300, 0, 300, 300, 0, 1, 1, 64, None, None, 0.0, y)
    with pytest.raises(mako_attn.MakoError, match="heads of 128 with 3 rotated"):
        ctx.heads_partial(x, 128, 0, 128, 128, 3, 1, 1, 64, x, None, 0.0, y)
    with pytest.raises(mako_attn.MakoError, match="beyond n_pad"):
        ctx.heads_partial(x, 128, 0, 128, 128, 0, 1, 65, 64, None, None, 0.0, y)


@pytest.mark.parametrize("dtype", [0, 1])
def test_h3_sparse_block(ctx, oracle, dtype):
    """One sparse attention block of H3 (src/models/h3.cpp:343-362) on a layout from mako_cube_layout: fp32 qkv rows
    -> heads_partial through the cube map (q and k RMS-normed, 96 of 128 values rotated; v plain) -> heads_clear of
    the tiles' padding rows -> cube_select with local = 3 and the layout's frame-slab stride -> attention_sparse back
    into model row order.  Partial cubes at every grid edge and 63 dense rows.  Each stage is checked against the
    oracle on the device's own inputs: tiles within one ulp, selection bit for bit, output within the attention
    tolerance, every model row written and rows past them untouched."""
    import torch
    import mako_attn
    rng = np.random.default_rng(300 + dtype)
    frames, ph, pw, dense, H = 5, 10, 12, 63, 4
    rpf = ph * pw
    m, valid, cnt, L = mako_attn.cube_layout(frames, ph, pw, rpf, dense, dense, 0.25)
    assert (L.n_cubes, L.topk, L.stride) == (18, 5, 9)
    S, rows, q_pad, k_pad = dense + frames * rpf, L.rows, L.q_pad, L.k_pad
    ld = 3 * H * 128
    x = (rng.standard_normal((S, ld)) * 2.0).astype(np.float32)
    cs = angles(rng, S, 48)
    wq, wk = (rng.uniform(0.5, 1.5, 128).astype(np.float32) for _ in range(2))
    tiles = [y_tile(H, q_pad, 128, dtype), y_tile(H, k_pad, 128, dtype), y_tile(H, k_pad, 128, dtype)]
    args = [(0, 96, q_pad, wq, 1e-6), (H * 128, 96, k_pad, wk, 1e-6), (2 * H * 128, 0, k_pad, None, 0.0)]
    xd, csd, md = tdev(x), tdev(cs), tdev(m)
    for t, (col0, rot, n_pad, w, eps) in zip(tiles, args):
        ctx.heads_partial(xd, ld, col0, 128, 128, rot, H, rows, n_pad, csd if rot else None,
                          tdev(w) if w is not None else None, eps, t, md)
        ctx.heads_clear(t, 128, n_pad, rows, H)
    torch.cuda.synchronize()
    tb = [bits(t) for t in tiles]
    for got, (col0, rot, n_pad, w, eps) in zip(tb, args):
        want = oracle.heads(x, ld, col0, 128, 128, rot, 1 if rot else 0, rows, H, n_pad, cs=cs, cs_row=48, w=w,
                            eps=eps, map_=m)
        far, exact = ulp_check(got[:, :rows], want[:, :rows], dtype)
        assert far == 0 and exact >= 0.99, f"{far} elements beyond one ulp, {exact:.4f} bit-identical"
        assert np.all(got[:, rows:] == 0)
    qt, kt, vt = tiles
    sel_t, nsel_t = ctx.cube_select(qt, kt, H, q_pad, k_pad, L.n_cubes, tdev(cnt), L.topk, 3, L.stride)
    torch.cuda.synchronize()
    sel = sel_t.cpu().numpy().view(np.uint16)
    nsel = nsel_t.cpu().numpy().view(np.uint16)
    want_sel, want_nsel, *_ = oracle.cube_select(dtype, tb[0], tb[1], H, q_pad, k_pad, L.n_cubes, cnt, L.topk,
                                                 local=3, stride=L.stride, mode=1)
    np.testing.assert_array_equal(sel, want_sel)
    np.testing.assert_array_equal(nsel, want_nsel)
    width = H * 128
    o = torch.full((S + 2, width), 12345.0, dtype=torch.float32, device="cuda")
    ctx.attention_sparse(qt, kt, vt, o, rows, q_pad, rows, k_pad, H, H, width, L.n_cubes, L.topk, L.dense0, L.dense1,
                         sel_t, nsel_t, tdev(valid), md)
    torch.cuda.synchronize()
    assert ctx.device_error() == 0
    got = o.cpu().numpy()
    want = np.full((S + 2, width), 12345.0, np.float32)
    oracle.attention_sparse(dtype, tb[0], tb[1], tb[2], rows, q_pad, rows, k_pad, H, H, width, L.n_cubes, L.topk,
                            L.dense0, L.dense1, sel, nsel, valid, m, out=want)
    assert not np.any(want[:S] == 12345.0), "the layout maps every model row"
    ok, stats = C.within(got[:S], want[:S])
    assert ok, f"max-abs {stats[0]:.3e} rel-L2 {stats[1]:.3e} worst-row {stats[2]:.3e}"
    assert np.all(got[S:] == 12345.0)


BULK = [
    # 16-byte aligned rows (128-bit loads).  A partial last block of rows, heads % 8 != 0, map holes, 96 of 128
    # values rotated.
    ("q-norm-rot96-map", dict(api="partial", dim=128, heads=11, stride=128, col0=4, rot=96, norm=True, T=203,
                              n_pad=256, dtype=1, map=True)),
    # heads not adjacent (stride 2 D), partial rotation
    ("gated-q-rot64", dict(api="partial", dim=128, heads=9, stride=256, col0=0, rot=64, norm=True, T=77, n_pad=128,
                           dtype=0, map=False)),
    # adjacent-pair rotation with the norm (heads_norm)
    ("pairs-norm", dict(api="norm", dim=128, heads=6, stride=128, col0=8, rot=128, norm=True, T=150, n_pad=192,
                        dtype=1, map=False)),
    # no rotation, no norm (v tiles), 64-wide heads; 96-wide heads rotated
    ("v-d64", dict(api="partial", dim=64, heads=20, stride=64, col0=8, rot=0, norm=False, T=1000, n_pad=1024,
                   dtype=1, map=False)),
    ("k-d96", dict(api="partial", dim=96, heads=5, stride=96, col0=0, rot=96, norm=True, T=40, n_pad=64, dtype=0,
                   map=True)),
]


@pytest.mark.parametrize("name,kw", BULK, ids=[n for n, _ in BULK])
def test_heads_aligned_rows(ctx, oracle, name, kw):
    import torch
    rng = np.random.default_rng(hash(name) % 2 ** 32)
    dim, H, stride, col0, rot, T, n_pad, dtype = (kw[k] for k in ("dim", "heads", "stride", "col0", "rot", "T",
                                                                  "n_pad", "dtype"))
    ld = col0 + stride * H + 12
    assert ld % 4 == 0 and col0 % 4 == 0 and stride % 4 == 0
    src_rows = T + 9
    x = (rng.standard_normal((src_rows, ld)) * 2.0).astype(np.float32)
    w = rng.uniform(0.5, 1.5, dim).astype(np.float32) if kw["norm"] else None
    m = None
    if kw["map"]:
        m = rng.permutation(src_rows)[:T].astype(np.int32)
        m[::7] = -1
    y = y_tile(H, n_pad, dim, dtype)
    if kw["api"] == "norm":
        cs = angles(rng, src_rows, 64)
        ctx.heads_norm(tdev(x), ld, col0, H, T, n_pad, tdev(cs), 2, tdev(w), 1e-6, 0, y)
        want = oracle.heads(x, ld, col0, 128, 128, 128, 2, T, H, n_pad, cs=cs, cs_row=64, w=w, eps=1e-6)
    else:
        cs = angles(rng, src_rows, max(rot // 2, 1))
        ctx.heads_partial(tdev(x), ld, col0, stride, dim, rot, H, T, n_pad, tdev(cs) if rot else None,
                          tdev(w) if w is not None else None, 1e-6, y, tdev(m) if m is not None else None)
        want = oracle.heads(x, ld, col0, stride, dim, rot, 1 if rot else 0, T, H, n_pad, cs=cs, cs_row=rot // 2, w=w,
                            eps=1e-6 if kw["norm"] else 0.0, map_=m)
    torch.cuda.synchronize()
    assert ctx.device_error() == 0
    got = bits(y)
    far, exact = ulp_check(got[:, :T], want[:, :T], dtype)
    assert far == 0 and exact >= 0.99, f"{far} elements beyond one ulp, {exact:.4f} bit-identical"
    assert np.all(got[:, T:] == 0x7BFF), "rows past T are the caller's"
    if m is not None:
        assert np.all(got[:, :T][:, m < 0] == 0), "rows the map leaves empty are zero"
