"""The sharded forms' kernels on one GPU, with the second rank stood in for by host writes.

Rank 0 of a group of 2 runs for real; rank 1's exchange area is a plain device buffer, and what rank 1 would have sent
(its decode rows, its barrier flags) is written into rank 0's area by the host before the call.  So every wait in the
call is already satisfied when it starts -- no kernel here waits on another launch -- and the test checks what rank 0
computed, what it stored into "rank 1's" memory, and the merged result against the oracle.  The last test leaves the
flags unset on purpose: the bounded waits run out (about a second each), the device error flag reports it and the
context stays usable.
"""
import numpy as np
import pytest

import attn_cases as C

pytestmark = pytest.mark.gpu

ROWS_CAP = 64
STRIDE = 260  # floats per exchanged decode row (kXchgStride)
SENTINEL = 12345.0


def dev(bits, dtype):
    import torch
    t = torch.from_numpy(np.ascontiguousarray(bits).view(np.int16))
    return t.view(torch.bfloat16 if dtype == 1 else torch.float16).cuda()


def rows_offset(rows_cap):
    return (256 + 2 * 8 * rows_cap * 4 + 255) // 256 * 256


class Pair:
    """Rank 0's real group and a stand-in area for rank 1."""

    def __init__(self, ctx):
        import torch
        import mako_attn
        self.g = mako_attn.Group(ctx, 0, 2, ROWS_CAP)
        self.area0, nbytes = self.g.area()
        self.fake1 = torch.zeros(nbytes // 4, dtype=torch.int32, device="cuda")
        self.g.connect_ptrs([self.area0, self.fake1.data_ptr()])
        self.own = mako_attn.device_view(self.area0, (nbytes // 4,), "<i4")
        self.epoch = 0

    def next_epoch(self):
        self.epoch += 1
        return self.epoch

    def close(self):
        self.g.close()


def set_barrier_flags(pair, epoch):
    """Rank 1's enter and done flags for `epoch` in rank 0's area."""
    par = epoch & 1
    for kind in (0, 1):
        pair.own[(par * 2 + kind) * 8 + 1] = epoch


@pytest.mark.parametrize("n,ctas", [(300, 0), (1100, 3)], ids=["one_item_per_cta", "few_ctas"])
def test_gather_stores_the_slice_into_every_rank(ctx, oracle, n, ctas):
    """The head-sharded kernel's output slices in both ranks' o.  few_ctas: the persistent grid capped at three CTAs
    (MAKO_OPT_GRID_CTAS), so that each CTA stores many items' boxes through its staging buffers."""
    import torch
    import mako_attn
    from mako_attn.shard import head_shard
    d = C.dense_case(seed=51, heads=8, kv_heads=4, dim=128, n_q=n, n_k=n, dtype=1)
    head0, hl, kv0, kvl = head_shard(8, 4, 2, 0)
    q = dev(d["q"][head0:head0 + hl], 1)
    k, v = dev(d["k"][kv0:kv0 + kvl], 1), dev(d["v"][kv0:kv0 + kvl], 1)
    want = oracle.attention(1, d["q"], d["k"], d["v"], n, d["q_pad"], n, d["k_pad"], 8, 4, 0, C.UINT32_MAX, 128)
    pair = Pair(ctx)
    ctx.set_option(mako_attn.OPT_GRID_CTAS, ctas)
    try:
        for _ in range(2):  # two calls: both barrier parities
            o0 = torch.full((n, 1024), SENTINEL, dtype=torch.float32, device="cuda")
            o1 = torch.full((n, 1024), SENTINEL, dtype=torch.float32, device="cuda")
            set_barrier_flags(pair, pair.next_epoch())
            pair.g.attention_gather(q, k, v, [o0.data_ptr(), o1.data_ptr()], n, d["q_pad"], n, d["k_pad"], hl, kvl,
                                    head0, 1024)
            torch.cuda.synchronize()
            assert ctx.device_error() == 0
            g0, g1 = o0.cpu().numpy(), o1.cpu().numpy()
            ok, stats = C.within(g0[:, :512], want[:, :512])
            assert ok, stats
            assert np.array_equal(g0[:, :512], g1[:, :512]), "the peer's copy differs from the local one"
            assert np.all(g0[:, 512:] == SENTINEL) and np.all(g1[:, 512:] == SENTINEL), "columns of other heads"
            # this rank released its flags in the peer's area
            flags1 = pair.fake1.cpu().numpy()
            par = pair.epoch & 1
            assert flags1[(par * 2) * 8 + 0] == pair.epoch and flags1[(par * 2 + 1) * 8 + 0] == pair.epoch
    finally:
        ctx.set_option(mako_attn.OPT_GRID_CTAS, 0)
        pair.close()


@pytest.mark.parametrize("dtype", [0, 1])
def test_decode_kv_sharded_merges_the_peer_rows(ctx, oracle, dtype):
    import torch
    from mako_attn.shard import kv_shard
    c = C.decode_case(seed=52 + dtype, batch=3, heads=8, kv_heads=2, dim=128, lo=200, hi=5000, dtype=dtype)
    B, H, KV, D = 3, 8, 2, 128
    want = oracle.decode(dtype, c["q"], c["k"], c["v"], c["kv_len"], H, KV, D, c["k_stride"])
    sh = [kv_shard(int(n), 2, 0) for n in c["kv_len"]]
    s1 = [kv_shard(int(n), 2, 1) for n in c["kv_len"]]
    # rank 0's shard, re-based at row 0 of its own cache
    n0 = np.array([n for _, n in sh], np.int32)
    stride0 = C.round_up(int(n0.max()), 64)
    k0 = np.zeros((B, KV, stride0, D), np.uint16)
    v0 = np.zeros_like(k0)
    for b, (s, n) in enumerate(sh):
        k0[b, :, :n] = c["k"][b, :, s:s + n]
        v0[b, :, :n] = c["v"][b, :, s:s + n]
    o1_, m1, l1 = oracle.decode_partial(dtype, c["q"], c["k"], c["v"], [n for _, n in s1], H, KV, D, c["k_stride"],
                                        start=[s for s, _ in s1])
    m0_want = oracle.decode_partial(dtype, c["q"], c["k"], c["v"], n0, H, KV, D, c["k_stride"], start=[s for s, _ in sh])
    pair = Pair(ctx)
    try:
        q = dev(c["q"], dtype)
        k, v = dev(k0, dtype), dev(v0, dtype)
        kvl = torch.from_numpy(n0).cuda()
        off = rows_offset(ROWS_CAP) // 4
        for _ in range(2):
            epoch = pair.next_epoch()
            par = epoch & 1
            # rank 1's rows and flags, as its kernel would have stored them into rank 0's area
            rows = np.zeros((B * H, STRIDE), np.float32)
            rows[:, :D] = o1_.reshape(B * H, D)
            rows[:, D] = m1.reshape(-1)
            rows[:, D + 1] = l1.reshape(-1)
            base = off + ((par * 8 + 1) * ROWS_CAP) * STRIDE
            pair.own[base:base + B * H * STRIDE] = torch.from_numpy(rows.view(np.int32).reshape(-1)).cuda()
            fb = 64 + (par * 8 + 1) * ROWS_CAP
            pair.own[fb:fb + B * H] = epoch
            o = torch.full((B, H * D), SENTINEL, dtype=torch.float32, device="cuda")
            pair.g.attention_decode_kv_sharded(q, k, v, o, kvl, int(n0.max()), H, KV, D, stride0)
            torch.cuda.synchronize()
            assert ctx.device_error() == 0
            ok, stats = C.within(o.cpu().numpy(), want)
            assert ok, f"merged: {stats}"
            # what rank 0 pushed into rank 1's area: its rows (normalised they must match its shard's attention)
            a1 = pair.fake1.cpu().numpy()
            pushed = a1[off + ((par * 8 + 0) * ROWS_CAP) * STRIDE:][:B * H * STRIDE].view(np.float32).reshape(B * H,
                                                                                                      STRIDE)
            assert np.all(a1[64 + (par * 8) * ROWS_CAP:][:B * H] == epoch), "flags released in the peer's area"
            mine = pushed[:, :D] / pushed[:, D + 1:D + 2]
            ref = m0_want[0].reshape(B * H, D) / m0_want[2].reshape(B * H, 1)
            ok, stats = C.within(mine, ref)
            assert ok, f"pushed rows: {stats}"
            assert np.allclose(pushed[:, D], m0_want[1].reshape(-1), atol=1e-3)
    finally:
        pair.close()


def test_waits_that_run_out_report_and_leave_the_context_usable(ctx, oracle):
    """Nothing sets rank 1's flags: the barriers give up after their bound, the error flag says so, and the next
    ordinary call on the same context is correct."""
    import torch
    d = C.dense_case(seed=53, heads=2, kv_heads=2, dim=128, n_q=64, n_k=64, dtype=0)
    pair = Pair(ctx)
    try:
        q, k, v = dev(d["q"], 0), dev(d["k"], 0), dev(d["v"], 0)
        o0 = torch.zeros((64, 256), dtype=torch.float32, device="cuda")
        o1 = torch.zeros((64, 256), dtype=torch.float32, device="cuda")
        pair.next_epoch()
        pair.g.attention_gather(q, k, v, [o0.data_ptr(), o1.data_ptr()], 64, d["q_pad"], 64, d["k_pad"], 2, 2, 0, 256)
        torch.cuda.synchronize()
        assert ctx.device_error() == 30
        o = torch.zeros((64, 256), dtype=torch.float32, device="cuda")
        ctx.attention(q, k, v, o, 64, d["q_pad"], 64, d["k_pad"], 2, 2)
        torch.cuda.synchronize()
        want = oracle.attention(0, d["q"], d["k"], d["v"], 64, d["q_pad"], 64, d["k_pad"], 2, 2, 0, C.UINT32_MAX, 128)
        ok, stats = C.within(o.cpu().numpy(), want)
        assert ok and ctx.device_error() == 0, stats
    finally:
        pair.close()
