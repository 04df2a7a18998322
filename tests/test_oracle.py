"""Pins the CPU oracle before any GPU result is trusted against it (no GPU needed).

The reference cannot be built here (Metal only), so the pins are: (1) the reference test's own checks re-run on its
own fixture (tests/sparse_attn_test.cpp:46-208 -- selection by sorted double scores, the local-cube order); (2) an
independent numpy float64 restatement of the mask rules (src/kernels/ops.metal:161,289) and of the sparse key sets
(tests/sparse_attn_test.cpp:143-155, ops.metal:1079-1110); (3) the committed golden vectors (tests/golden/).
"""
import os

import numpy as np
import pytest

import attn_cases as C

GOLDEN = os.path.join(os.path.dirname(__file__), "golden", "sparse_attn_fixture.npz")


def np_attention(dtype, q, k, v, n_q, q_pad, n_k, k_pad, heads, kv_heads, q_pos0, block, dim, oracle):
    """Independent float64 restatement: full score matrix, boolean mask, masked softmax."""
    qf = oracle.from_bits(q, dtype).reshape(heads, q_pad, dim).astype(np.float64)
    kf = oracle.from_bits(k, dtype).reshape(kv_heads, k_pad, dim).astype(np.float64)
    vf = oracle.from_bits(v, dtype).reshape(kv_heads, k_pad, dim).astype(np.float64)
    pos = q_pos0 + np.arange(n_q, dtype=np.int64)[:, None]
    j = np.arange(n_k, dtype=np.int64)[None, :]
    vis = (j <= pos) | ((pos >= block) & (j >= block))
    out = np.zeros((n_q, heads * dim))
    if n_k == 0:
        return out
    scale = np.float64(np.float32(1.0) / np.sqrt(np.float32(dim)))
    for h in range(heads):
        kvh = h // (heads // kv_heads)
        s = qf[h, :n_q] @ kf[kvh, :n_k].T * scale
        s = np.where(vis, s, -np.inf)
        mx = np.max(s, axis=1, keepdims=True)
        mx = np.where(np.isfinite(mx), mx, 0.0)
        e = np.exp(s - mx)
        den = e.sum(axis=1, keepdims=True)
        o = np.where(den > 0, (e @ vf[kvh, :n_k]) / np.where(den > 0, den, 1.0), 0.0)
        out[:, h * dim:(h + 1) * dim] = o
    return out


@pytest.mark.parametrize("kw", [
    dict(heads=4, kv_heads=2, dim=64, n_q=70, n_k=70, block=C.UINT32_MAX),                # causal, ragged, GQA
    dict(heads=2, kv_heads=2, dim=128, n_q=65, n_k=130, block=0),                          # bidirectional
    dict(heads=2, kv_heads=1, dim=128, n_q=40, n_k=200, q_pos0=150, block=C.UINT32_MAX),  # decode-like offset
    dict(heads=2, kv_heads=2, dim=256, n_q=96, n_k=96, block=50),                          # image block
    dict(heads=3, kv_heads=1, dim=64, n_q=33, n_k=0, block=C.UINT32_MAX),                  # no keys: zeros
])
@pytest.mark.parametrize("dtype", [0, 1])
def test_dense_oracle_matches_numpy(oracle, kw, dtype):
    case = C.dense_case(seed=11, dtype=dtype, **kw)
    args = [case[x] for x in ("q", "k", "v", "n_q", "q_pad", "n_k", "k_pad", "heads", "kv_heads", "q_pos0", "block",
                              "dim")]
    got = oracle.attention(dtype, *args)
    want = np_attention(dtype, *args, oracle=oracle)
    assert np.max(np.abs(got - want)) < 1e-5


def test_decode_oracle_is_dense_with_one_query(oracle):
    case = C.decode_case(seed=3, batch=3, heads=4, kv_heads=2, dim=128, lo=1, hi=300, dtype=0)
    got = oracle.decode(0, case["q"], case["k"], case["v"], case["kv_len"], 4, 2, 128, case["k_stride"])
    for b in range(3):
        L = int(case["kv_len"][b])
        q = case["q"][b].reshape(4, 1, 128)
        want = oracle.attention(0, q, case["k"][b], case["v"][b], 1, 1, L, case["k_stride"], 4, 2, L - 1,
                                C.UINT32_MAX, 128)
        np.testing.assert_array_equal(got[b], want[0])


def test_reference_fixture_shape(oracle):
    fx = oracle.sparse_test_fixture()
    assert fx["cnt"].tolist() == [64, 64, 64, 64, 64, 20]
    assert int(fx["valid"].sum()) == 5 * 64 + 20 + 60
    assert int((fx["map"] >= 0).sum()) == 400
    # invalid rows are zero, valid rows drawn
    qf = oracle.from_bits(fx["q"], 0)
    assert np.all(qf[:, 340:384] == 0) and np.all(qf[:, 444:] == 0) and np.all(qf[:, 0] != 0)


def test_selection_matches_reference_test_procedure(oracle):
    """tests/sparse_attn_test.cpp:103-128: pooled means in double (each row / cnt), double dot products, sorted by
    (-score, index), the first topk -- against both oracle modes."""
    fx = oracle.sparse_test_fixture()
    D, heads, cubes, topk = 128, 2, 6, 3
    kf = oracle.from_bits(fx["k"], 0).astype(np.float64)
    qf = np.zeros_like(kf)
    qf[:, :448] = oracle.from_bits(fx["q"], 0)
    want = np.zeros((heads, cubes, topk), np.uint16)
    for hh in range(heads):
        qp = np.zeros((cubes, D))
        kp = np.zeros((cubes, D))
        for c in range(cubes):
            for r in range(int(fx["cnt"][c])):
                qp[c] += qf[hh, c * 64 + r] / fx["cnt"][c]
                kp[c] += kf[hh, c * 64 + r] / fx["cnt"][c]
        for qc in range(cubes):
            sc = sorted((-float(qp[qc] @ kp[kc]), kc) for kc in range(cubes))
            want[hh, qc] = [kc for _, kc in sc[:topk]]
    for mode in (0, 1):
        sel, nsel, *_ = oracle.cube_select(0, fx["q"], fx["k"], heads, 448, 512, cubes, fx["cnt"], topk, mode=mode)
        np.testing.assert_array_equal(sel, want)
        assert np.all(nsel == topk)


def test_local_selection_order(oracle):
    """tests/sparse_attn_test.cpp:184-208: with local=3, stride=1 the query cube and its neighbours lead; no cube
    twice."""
    fx = oracle.sparse_test_fixture()
    sel, *_ = oracle.cube_select(0, fx["q"], fx["k"], 2, 448, 512, 6, fx["cnt"], 4, local=3, stride=1)
    for hh in range(2):
        for qc in range(6):
            e = sel[hh, qc].tolist()
            want = [qc] + ([qc - 1] if qc >= 1 else []) + ([qc + 1] if qc + 1 < 6 else [])
            assert e[:len(want)] == want
            assert len(set(e)) == 4


def test_local_stride_zero_repeats_the_cube(oracle):
    """ops.metal:975-989 with stride 0: all three local picks are the query cube itself (kept, as the reference)."""
    fx = oracle.sparse_test_fixture()
    sel, *_ = oracle.cube_select(0, fx["q"], fx["k"], 2, 448, 512, 6, fx["cnt"], 5, local=3, stride=0)
    for qc in range(6):
        assert sel[0, qc, :3].tolist() == [qc, qc, qc]
        assert qc not in sel[0, qc, 3:].tolist()


def np_sparse_rows(oracle, fx, sel, nsel, n_q, heads, n_cubes, dense0, dense1, n_k):
    """The reference test's key sets (tests/sparse_attn_test.cpp:143-173), generalised by ops.metal:1079-1110
    (validity applies to the dense rows too; the dense tiles see every valid key below n_k)."""
    D = 128
    qf = oracle.from_bits(fx["q"], 0).astype(np.float64)
    kf = oracle.from_bits(fx["k"], 0).astype(np.float64)
    vf = oracle.from_bits(fx["v"], 0).astype(np.float64)
    valid = fx["valid"]
    out = {}
    scale = float(np.float32(1) / np.sqrt(np.float32(D)))
    for hh in range(heads):
        for r in range(n_q):
            if fx["map"][r] < 0:
                continue
            if r // 64 < n_cubes:
                keys = [j for c in sel[hh, r // 64, :nsel[hh, r // 64]] for j in range(c * 64, c * 64 + 64) if valid[j]]
                keys += [j for j in range(dense0, dense1) if valid[j]]
            else:
                keys = [j for j in range(n_k) if valid[j]]
            s = kf[hh, keys] @ qf[hh, r] * scale
            w = np.exp(s - s.max())
            out[(hh, r)] = (w / w.sum()) @ vf[hh, keys]
    return out


def test_sparse_oracle_matches_reference_key_sets(oracle):
    fx = oracle.sparse_test_fixture()
    sel, nsel, *_ = oracle.cube_select(0, fx["q"], fx["k"], 2, 448, 512, 6, fx["cnt"], 3)
    o = np.full((448, 256), 12345.0, np.float32)
    oracle.attention_sparse(0, fx["q"], fx["k"], fx["v"], 444, 448, 444, 512, 2, 2, 256, 6, 3, 384, 444, sel, nsel,
                            fx["valid"], fx["map"], out=o)
    want = np_sparse_rows(oracle, fx, sel, nsel, 444, 2, 6, 384, 444, 444)
    for (hh, r), w in want.items():
        np.testing.assert_allclose(o[r, hh * 128:(hh + 1) * 128], w, atol=1e-6)
    # rows never mapped keep the sentinel (tests/sparse_attn_test.cpp:138-141)
    untouched = [r for r in range(448) if r >= 444 or fx["map"][r] < 0]
    assert np.all(o[untouched] == 12345.0)


def test_golden_vectors(oracle):
    """The committed vectors (tests/golden/make_golden.py) still come out of the oracle."""
    import hashlib
    g = np.load(GOLDEN)
    fx = oracle.sparse_test_fixture()
    for name in ("q", "k", "v", "valid", "map", "cnt"):
        assert hashlib.sha256(np.ascontiguousarray(fx[name]).tobytes()).hexdigest() == str(g["sha_" + name])
    sel, nsel, *_ = oracle.cube_select(0, fx["q"], fx["k"], 2, 448, 512, 6, fx["cnt"], 3)
    np.testing.assert_array_equal(sel, g["sel"])
    np.testing.assert_array_equal(nsel, g["nsel"])
    sel4, *_ = oracle.cube_select(0, fx["q"], fx["k"], 2, 448, 512, 6, fx["cnt"], 4, local=3, stride=1)
    np.testing.assert_array_equal(sel4, g["sel_local"])
    o = np.full((448, 256), 12345.0, np.float32)
    oracle.attention_sparse(0, fx["q"], fx["k"], fx["v"], 444, 448, 444, 512, 2, 2, 256, 6, 3, 384, 444, sel, nsel,
                            fx["valid"], fx["map"], out=o)
    np.testing.assert_allclose(o[g["o_rows"]], g["o_sub"], rtol=0, atol=1e-6)


def test_heads_oracle_matches_numpy(oracle):
    """The producers' restatement against an independent numpy float64 one, with known-answer cases: a rotation by
    zero is the identity, by a right angle turns (u, v) into (-v, u), and the RMS norm with unit weights gives unit
    RMS rows."""
    import numpy as np
    rng = np.random.default_rng(3)
    T, H, dim, stride, col0, rot = 6, 2, 64, 80, 8, 48
    ld = col0 + stride * H
    x = rng.standard_normal((T, ld)).astype(np.float32)
    a = rng.uniform(-3, 3, (T, rot // 2))
    cs = np.stack([np.cos(a), np.sin(a)], -1).astype(np.float32)
    w = rng.uniform(0.5, 1.5, dim).astype(np.float32)
    got = oracle.heads(x, ld, col0, stride, dim, rot, 1, T, H, 8, cs=cs, cs_row=rot // 2, w=w, eps=1e-6)
    for h in range(H):
        v = x[:, col0 + h * stride: col0 + h * stride + dim].astype(np.float64)
        v = v / np.sqrt((v * v).mean(-1, keepdims=True) + 1e-6) * w
        o = v.copy()
        c, s = cs[..., 0].astype(np.float64), cs[..., 1].astype(np.float64)
        o[:, :rot // 2] = v[:, :rot // 2] * c - v[:, rot // 2:rot] * s
        o[:, rot // 2:rot] = v[:, rot // 2:rot] * c + v[:, :rot // 2] * s
        np.testing.assert_allclose(got[h, :T], o, rtol=1e-6, atol=1e-6)
    # identity rotation, right-angle rotation, unit RMS
    zero = np.zeros((T, 32, 2), np.float32)
    zero[..., 0] = 1.0
    y0 = oracle.heads(x, ld, 0, 64, 64, 64, 1, T, 1, T, cs=zero, cs_row=32)
    np.testing.assert_array_equal(y0[0], x[:, :64])
    quarter = np.zeros((T, 32, 2), np.float32)
    quarter[..., 1] = 1.0
    yq = oracle.heads(x, ld, 0, 64, 64, 64, 2, T, 1, T, cs=quarter, cs_row=32)
    np.testing.assert_allclose(yq[0][:, 0::2], -x[:, 1:64:2], atol=1e-6)
    np.testing.assert_allclose(yq[0][:, 1::2], x[:, 0:64:2], atol=1e-6)
    yn = oracle.heads(x, ld, 0, 64, 64, 0, 0, T, 1, T, w=np.ones(64, np.float32), eps=1e-12)
    np.testing.assert_allclose(np.sqrt((yn[0].astype(np.float64) ** 2).mean(-1)), 1.0, rtol=1e-6)


def test_proj_restatement(oracle):
    """The oracle's double GEMM against numpy's float64 product of the same 16-bit values."""
    rng = np.random.default_rng(5)
    for dtype in (0, 1):
        x = oracle.to_bits(rng.standard_normal((37, 128)).astype(np.float32), dtype)
        w = oracle.to_bits(rng.standard_normal((45, 128)).astype(np.float32), dtype)
        want = oracle.from_bits(x, dtype).astype(np.float64) @ oracle.from_bits(w, dtype).astype(np.float64).T
        got = oracle.proj(dtype, w, x, 37, 128, 45)
        assert np.allclose(got, want.astype(np.float32), rtol=1e-6, atol=1e-6)
        rows = np.array([3, 30], np.uint32)
        part = oracle.proj(dtype, w, x, 37, 128, 45, rows=rows)
        assert np.array_equal(part[rows], got[rows]) and not np.any(part[5])
