"""Seeded synthetic inputs and comparison helpers shared by the parity tests, smoke() and bench.py.

Inputs are i.i.d. N(0, 1) float32 from numpy's PCG64 generator (np.random.default_rng(seed)), optionally scaled or
RMS-normalised per row, rounded to fp16 / bf16 bit patterns exactly as the device reads them.  Padded rows are
zero, as the reference's producers leave them (src/kernels/ops.metal:45-52).
"""
from __future__ import annotations

import numpy as np

import oracle as O

UINT32_MAX = 0xFFFFFFFF

# North-star tolerance against the fp32/double-accumulated oracle, plus the reference test's own per-row bound
# (tests/sparse_attn_test.cpp:181).
MAX_ABS = 2e-3
REL_L2 = 1e-3
ROW_REL_L2 = 5e-3


def round_up(x: int, m: int) -> int:
    return (x + m - 1) // m * m


def normal(rng, shape, scale=1.0, rms_norm=False):
    x = rng.standard_normal(shape, dtype=np.float32)
    if rms_norm:
        x = x / np.sqrt(np.mean(x.astype(np.float64) ** 2, axis=-1, keepdims=True)).astype(np.float32)
    return (x * np.float32(scale)).astype(np.float32)


def head_tiles(rng, heads, n, pad, dim, dtype, scale=1.0, rms_norm=False):
    """[heads][pad][dim] bit patterns; rows >= n zero."""
    t = np.zeros((heads, pad, dim), np.float32)
    t[:, :n] = normal(rng, (heads, n, dim), scale, rms_norm)
    return O.to_bits(t, dtype)


def compare(got: np.ndarray, want: np.ndarray):
    """(max-abs error, global relative L2, worst per-row relative L2); rows = last axis."""
    g = np.asarray(got, np.float64)
    w = np.asarray(want, np.float64)
    err = g - w
    max_abs = float(np.max(np.abs(err))) if err.size else 0.0
    rel = float(np.sqrt(np.sum(err ** 2) / max(np.sum(w ** 2), 1e-30)))
    e2 = np.sum(err.reshape(-1, err.shape[-1]) ** 2, axis=-1)
    n2 = np.sum(w.reshape(-1, w.shape[-1]) ** 2, axis=-1)
    row = float(np.max(np.sqrt(e2 / np.maximum(n2, 1e-30)))) if e2.size else 0.0
    return max_abs, rel, row


def within(got, want, max_abs=MAX_ABS, rel_l2=REL_L2, row_rel=ROW_REL_L2):
    a, r, w = compare(got, want)
    return (a <= max_abs and r <= rel_l2 and w <= row_rel), (a, r, w)


def dense_case(seed, heads, kv_heads, dim, n_q, n_k, dtype, q_pos0=0, block=UINT32_MAX, scale=1.0, rms_norm=False,
               qk_rms_norm=False):
    rng = np.random.default_rng(seed)
    q_pad, k_pad = round_up(max(n_q, 1), 64), round_up(max(n_k, 1), 128)
    q = head_tiles(rng, heads, n_q, q_pad, dim, dtype, scale, rms_norm or qk_rms_norm)
    k = head_tiles(rng, kv_heads, n_k, k_pad, dim, dtype, scale, rms_norm or qk_rms_norm)
    v = head_tiles(rng, kv_heads, n_k, k_pad, dim, dtype, scale, rms_norm)
    return dict(q=q, k=k, v=v, n_q=n_q, q_pad=q_pad, n_k=n_k, k_pad=k_pad, heads=heads, kv_heads=kv_heads,
                q_pos0=q_pos0, block=block, dim=dim, dtype=dtype)


def decode_case(seed, batch, heads, kv_heads, dim, lo, hi, dtype, k_stride=None):
    rng = np.random.default_rng(seed)
    lens = rng.integers(lo, hi + 1, size=batch).astype(np.int32)
    k_stride = int(round_up(int(lens.max()), 64)) if k_stride is None else k_stride
    q = O.to_bits(normal(rng, (batch, heads, dim)), dtype)
    k = np.zeros((batch, kv_heads, k_stride, dim), np.uint16)
    v = np.zeros_like(k)
    for b in range(batch):
        k[b, :, :lens[b]] = O.to_bits(normal(rng, (kv_heads, int(lens[b]), dim)), dtype)
        v[b, :, :lens[b]] = O.to_bits(normal(rng, (kv_heads, int(lens[b]), dim)), dtype)
    return dict(q=q, k=k, v=v, kv_len=lens, heads=heads, kv_heads=kv_heads, dim=dim, k_stride=k_stride, dtype=dtype)


def block_lists(seed, heads, n_blocks, frac):
    """Config 4's mask: per (head, query block) its diagonal block plus ceil(frac * (n_blocks - 1)) others drawn
    uniformly without replacement, as int32 sorted lists [heads][n_blocks][keep] and counts [heads][n_blocks]."""
    rng = np.random.default_rng(seed)
    extra = int(np.ceil(frac * (n_blocks - 1)))
    keep = extra + 1
    lists = np.zeros((heads, n_blocks, keep), np.int32)
    for h in range(heads):
        for t in range(n_blocks):
            others = np.delete(np.arange(n_blocks), t)
            pick = rng.choice(others, size=extra, replace=False)
            lists[h, t] = np.sort(np.concatenate([[t], pick]))
    counts = np.full((heads, n_blocks), keep, np.int32)
    return lists, counts
