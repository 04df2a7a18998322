"""ctypes wrapper around the CPU oracle (liboracle.so) -- TEST INFRASTRUCTURE ONLY.

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg import this module; the CUDA product path
never does.  Every function takes numpy arrays holding the raw 16-bit patterns the device reads (fp16 or bf16) and
mirrors one extern "C" function of attn_oracle.cpp, which cites the reference lines it restates.
"""
from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "liboracle.so")

F16, BF16 = 0, 1

_lib = None


def build() -> str:
    """Compiles liboracle.so with the Makefile beside this file (a no-op when it is current)."""
    subprocess.run(["make", "-s", "-C", HERE], check=True)
    return LIB_PATH


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            build()
        L = ctypes.CDLL(LIB_PATH)
        u32, i32, ptr = ctypes.c_uint32, ctypes.c_int, ctypes.c_void_p
        L.oracle_threads.argtypes = [i32]
        L.oracle_threads.restype = i32
        L.oracle_attention.argtypes = [i32, ptr, ptr, ptr, ptr] + [u32] * 10 + [ptr, u32, i32]
        L.oracle_decode.argtypes = [i32, ptr, ptr, ptr, ptr, u32, ptr, u32, u32, u32, u32, i32]
        L.oracle_attention_sparse.argtypes = ([i32, ptr, ptr, ptr, ptr] + [u32] * 11 + [ptr] * 4 + [ptr, u32, i32])
        L.oracle_cube_select.argtypes = ([i32, ptr, ptr] + [u32] * 4 + [ptr] + [u32] * 3 + [i32] + [ptr] * 5)
        L.oracle_sparse_test_fixture.argtypes = [ptr] * 6
        L.oracle_heads.argtypes = [ptr, ctypes.c_uint64] + [u32] * 9 + [ptr, u32, ptr, ctypes.c_float, ptr, ptr]
        L.oracle_heads.restype = None
        L.oracle_proj.argtypes = [i32, ptr, ptr, ptr] + [u32] * 4 + [ptr, u32, i32]
        L.oracle_proj.restype = None
        for f in (L.oracle_attention, L.oracle_decode, L.oracle_attention_sparse, L.oracle_cube_select,
                  L.oracle_sparse_test_fixture):
            f.restype = None
        _lib = L
    return _lib


def _p(a):
    return None if a is None else a.ctypes.data_as(ctypes.c_void_p)


def _c(a, dtype):
    return np.ascontiguousarray(a, dtype=dtype)


def threads(n: int = 0) -> int:
    """Sets (n > 0) and returns the OpenMP thread count the oracle uses."""
    return lib().oracle_threads(n)


# ---- 16-bit encodings ---------------------------------------------------------------------------------------------

def to_f16_bits(x: np.ndarray) -> np.ndarray:
    return np.asarray(x, dtype=np.float32).astype(np.float16).view(np.uint16)


def to_bf16_bits(x: np.ndarray) -> np.ndarray:
    """Round to nearest even, NaN kept NaN (the rule of src/models/runtime.cpp:31-40)."""
    u = np.asarray(x, dtype=np.float32).view(np.uint32).astype(np.uint64)
    nan = ((u & 0x7F800000) == 0x7F800000) & ((u & 0x007FFFFF) != 0)
    r = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16) & 0xFFFF
    r = np.where(nan, ((u >> 16) | 0x40) & 0xFFFF, r)
    return r.astype(np.uint16)


def to_bits(x: np.ndarray, dtype: int) -> np.ndarray:
    return to_bf16_bits(x) if dtype == BF16 else to_f16_bits(x)


def from_bits(b: np.ndarray, dtype: int) -> np.ndarray:
    b = np.asarray(b, dtype=np.uint16)
    if dtype == BF16:
        return (b.astype(np.uint32) << 16).view(np.float32)
    return b.view(np.float16).astype(np.float32)


# ---- the restated reference ---------------------------------------------------------------------------------------

def attention(dtype, q, k, v, n_q, q_pad, n_k, k_pad, heads, kv_heads, q_pos0, block, dim, width=None, rows=None,
              out=None, nthreads=0):
    """Dense masked attention; returns o [n_q][width] float32 (rows not computed stay as `out` had them, or 0)."""
    width = heads * dim if width is None else width
    q, k, v = _c(q, np.uint16), _c(k, np.uint16), _c(v, np.uint16)
    assert q.size >= heads * q_pad * dim and k.size >= kv_heads * k_pad * dim and v.size >= kv_heads * k_pad * dim
    o = np.zeros((n_q, width), np.float32) if out is None else out
    assert o.dtype == np.float32 and o.flags.c_contiguous and o.size >= n_q * width
    r = None if rows is None else _c(rows, np.uint32)
    lib().oracle_attention(dtype, _p(q), _p(k), _p(v), _p(o), n_q, q_pad, n_k, k_pad, heads, kv_heads, q_pos0,
                           block & 0xFFFFFFFF, dim, width, _p(r), 0 if r is None else r.size, nthreads)
    return o


def decode(dtype, q, k, v, kv_len, heads, kv_heads, dim, k_stride, nthreads=0):
    """One query per sequence over its cache; returns o [batch][heads*dim] float32."""
    kv_len = _c(kv_len, np.int32)
    batch = kv_len.size
    q, k, v = _c(q, np.uint16), _c(k, np.uint16), _c(v, np.uint16)
    assert q.size >= batch * heads * dim and k.size >= batch * kv_heads * k_stride * dim
    o = np.zeros((batch, heads * dim), np.float32)
    lib().oracle_decode(dtype, _p(q), _p(k), _p(v), _p(o), batch, _p(kv_len), heads, kv_heads, dim, k_stride,
                        nthreads)
    return o


def attention_sparse(dtype, q, k, v, n_q, q_pad, n_k, k_pad, heads, kv_heads, width, n_cubes, max_sel, dense0,
                     dense1, sel, nsel, valid, map_, out=None, rows=None, nthreads=0):
    """Block-sparse attention (D 128); writes into `out` ([rows][width] float32, default zeros of max(map)+1 rows)."""
    q, k, v = _c(q, np.uint16), _c(k, np.uint16), _c(v, np.uint16)
    sel, nsel = _c(sel, np.uint16), _c(nsel, np.uint16)
    valid, map_ = _c(valid, np.uint8), _c(map_, np.int32)
    assert valid.size >= k_pad and map_.size >= q_pad
    if out is None:
        out = np.zeros((max(int(map_.max()) + 1, 1), width), np.float32)
    assert out.dtype == np.float32 and out.flags.c_contiguous
    r = None if rows is None else _c(rows, np.uint32)
    lib().oracle_attention_sparse(dtype, _p(q), _p(k), _p(v), _p(out), n_q, q_pad, n_k, k_pad, heads, kv_heads,
                                  width, n_cubes, max_sel, dense0, dense1, _p(sel), _p(nsel), _p(valid), _p(map_),
                                  _p(r), 0 if r is None else r.size, nthreads)
    return out


def cube_select(dtype, q, k, heads, q_pad, k_pad, n_cubes, cnt, topk, local=0, stride=0, mode=1):
    """Returns (sel [heads][n_cubes][min(topk,n_cubes)] u16, nsel [heads][n_cubes] u16, qp, kp, sc); qp/kp/sc are the
    fp32 intermediates (mode 1) or None (mode 0, double)."""
    q, k = _c(q, np.uint16), _c(k, np.uint16)
    cnt = _c(cnt, np.uint32)
    kk = min(topk, n_cubes)
    sel = np.zeros((heads, n_cubes, kk), np.uint16)
    nsel = np.zeros((heads, n_cubes), np.uint16)
    qp = kp = sc = None
    if mode == 1:
        qp = np.zeros((heads, n_cubes, 128), np.float32)
        kp = np.zeros_like(qp)
        sc = np.zeros((heads, n_cubes, n_cubes), np.float32)
    lib().oracle_cube_select(dtype, _p(q), _p(k), heads, q_pad, k_pad, n_cubes, _p(cnt), topk, local, stride, mode,
                             _p(sel), _p(nsel), _p(qp), _p(kp), _p(sc))
    return sel, nsel, qp, kp, sc


SPARSE_TEST = dict(D=128, heads=2, cubes=6, dense=60, topk=3, n=444, q_pad=448, k_pad=512, dense0=384, dense1=444)


def sparse_test_fixture():
    """The fixture of the reference's tests/sparse_attn_test.cpp:46-86 (libstdc++ normal draws, see the C source)."""
    f = SPARSE_TEST
    q = np.zeros((f["heads"], f["q_pad"], 128), np.uint16)
    k = np.zeros((f["heads"], f["k_pad"], 128), np.uint16)
    v = np.zeros_like(k)
    valid = np.zeros(f["k_pad"], np.uint8)
    map_ = np.zeros(f["q_pad"], np.int32)
    cnt = np.zeros(f["cubes"], np.uint32)
    lib().oracle_sparse_test_fixture(_p(q), _p(k), _p(v), _p(valid), _p(map_), _p(cnt))
    return dict(q=q, k=k, v=v, valid=valid, map=map_, cnt=cnt, **f)


# ---- split-KV partials and their log-sum-exp merge (numpy float64; the KV-sharded decode's two halves) -----------

def decode_partial(dtype, q, k, v, kv_len, heads, kv_heads, dim, k_stride, start=None):
    """Per (sequence, head) over keys [start[b], start[b] + kv_len[b]) of the cache: (o, m, l) with
    m = max of the scores in log2 units (q.k * fp32(1/sqrt(dim)) * log2(e)), l = sum 2^(s - m), o = sum 2^(s - m) v
    (unnormalised); an empty range gives m = -inf, l = 0, o = 0.  The decode's softmax (tests/sparse_attn_test.cpp:
    131-180) split into parts so that merge_partials recovers it."""
    kv_len = np.asarray(kv_len, np.int64)
    batch = kv_len.size
    start = np.zeros(batch, np.int64) if start is None else np.asarray(start, np.int64)
    qf = from_bits(np.asarray(q).reshape(batch, heads, dim), dtype).astype(np.float64)
    kf = from_bits(np.asarray(k).reshape(batch, kv_heads, k_stride, dim), dtype)
    vf = from_bits(np.asarray(v).reshape(batch, kv_heads, k_stride, dim), dtype)
    scale = float(np.float32(1.0) / np.sqrt(np.float32(dim))) * np.log2(np.e)
    group = heads // kv_heads
    o = np.zeros((batch, heads, dim))
    m = np.full((batch, heads), -np.inf)
    l = np.zeros((batch, heads))
    for b in range(batch):
        s0, n = int(start[b]), int(kv_len[b])
        if n <= 0:
            continue
        for h in range(heads):
            kk = kf[b, h // group, s0:s0 + n].astype(np.float64)
            vv = vf[b, h // group, s0:s0 + n].astype(np.float64)
            s = kk @ qf[b, h] * scale
            m[b, h] = s.max()
            p = np.exp2(s - m[b, h])
            l[b, h] = p.sum()
            o[b, h] = p @ vv
    return o, m, l


def merge_partials(parts):
    """Log-sum-exp merge of [(o, m, l), ...] into the normalised output [batch][heads * dim]."""
    M = np.max(np.stack([m for _, m, _ in parts]), axis=0)
    tot = np.zeros_like(M)
    acc = np.zeros_like(parts[0][0])
    for o, m, l in parts:
        w = np.where(m == -np.inf, 0.0, np.exp2(np.where(m == -np.inf, 0.0, m - np.where(M == -np.inf, 0.0, M))))
        tot += l * w
        acc += o * w[..., None]
    out = np.where(tot[..., None] > 0, acc / np.where(tot > 0, tot, 1.0)[..., None], 0.0)
    return out.reshape(out.shape[0], -1).astype(np.float32)


# ---- head-tile producers ------------------------------------------------------------------------------------------

def heads(x, ld, col0, stride, dim, rot, rope, rows, heads_, n_pad, row0=0, cs=None, cs_row=0, w=None, eps=0.0,
          map_=None, out=None):
    """heads_half / heads_norm_half / heads_partial restated (attn_oracle.cpp: oracle_heads); returns the float32
    values [heads][n_pad][dim] before 16-bit rounding (rows not written stay as `out` had them, or 0)."""
    x = _c(x, np.float32)
    y = np.zeros((heads_, n_pad, dim), np.float32) if out is None else out
    assert y.dtype == np.float32 and y.flags.c_contiguous
    cs = None if cs is None else _c(cs, np.float32)
    w = None if w is None else _c(w, np.float32)
    m = None if map_ is None else _c(map_, np.int32)
    lib().oracle_heads(_p(x), ld, col0, stride, dim, rot, rope, rows, heads_, n_pad, row0, _p(cs), cs_row, _p(w),
                       eps, _p(m), _p(y))
    return y


def proj(dtype, w, x, T, k, n, rows=None, nthreads=0):
    """The output projection in double: y [T][n] float32 (rows not in `rows` left 0) from 16-bit patterns x [T][k]
    and w [n][k]."""
    w, x = _c(w, np.uint16), _c(x, np.uint16)
    y = np.zeros((T, n), np.float32)
    r = None if rows is None else _c(rows, np.uint32)
    lib().oracle_proj(dtype, _p(w), _p(x), _p(y), T, k, n, n, _p(r), 0 if r is None else len(r), nthreads)
    return y
