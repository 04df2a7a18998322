"""The sharded forms' host logic on CPU ranks (gloo, world size 2): each rank takes its share of the work by the plan
in mako_attn/shard.py, computes it with the oracle, and the ranks exchange their pieces; the assembled result must be
the unsharded oracle's.  This checks that the plans cover every head and key exactly once and that the
log-sum-exp merge the KV-sharded decode kernel performs recovers the full softmax.  No GPU is involved."""
import os
import socket

import numpy as np
import pytest

import attn_cases as C


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, root):
    import sys
    for p in (os.path.join(root, "mako-common_b200"), os.path.join(root, "oracle"), os.path.join(root, "tests")):
        sys.path.insert(0, p)
    import torch.distributed as dist
    import attn_cases as C
    import oracle as O
    from mako_attn.shard import head_shard, kv_shard

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    O.threads(1)
    try:
        # KV-sharded decode: each rank's contiguous key range of every sequence
        c = C.decode_case(seed=41, batch=3, heads=8, kv_heads=2, dim=128, lo=50, hi=700, dtype=0)
        starts, counts = zip(*[kv_shard(int(n), world, rank) for n in c["kv_len"]])
        part = O.decode_partial(0, c["q"], c["k"], c["v"], counts, 8, 2, 128, c["k_stride"], start=starts)
        parts = [None] * world
        dist.all_gather_object(parts, part)
        got = O.merge_partials(parts)
        want = O.decode(0, c["q"], c["k"], c["v"], c["kv_len"], 8, 2, 128, c["k_stride"])
        ok, stats = C.within(got, want, max_abs=1e-5, rel_l2=1e-6, row_rel=1e-5)
        assert ok, f"decode merge: {stats}"

        # head-sharded prefill: this rank's kv heads with their query heads, columns placed at head0 * dim
        d = C.dense_case(seed=42, heads=8, kv_heads=4, dim=128, n_q=150, n_k=150, dtype=1)
        head0, hl, kv0, kvl = head_shard(8, 4, world, rank)
        mine = O.attention(1, d["q"][head0:head0 + hl], d["k"][kv0:kv0 + kvl], d["v"][kv0:kv0 + kvl], d["n_q"],
                           d["q_pad"], d["n_k"], d["k_pad"], hl, kvl, 0, C.UINT32_MAX, 128)
        pieces = [None] * world
        dist.all_gather_object(pieces, (head0, mine))
        full = np.zeros((d["n_q"], 8 * 128), np.float32)
        for h0, m in pieces:
            full[:, h0 * 128:h0 * 128 + m.shape[1]] = m
        want = O.attention(1, d["q"], d["k"], d["v"], d["n_q"], d["q_pad"], d["n_k"], d["k_pad"], 8, 4, 0,
                           C.UINT32_MAX, 128)
        assert np.array_equal(full, want), "head-sharded pieces differ from the unsharded oracle"
    finally:
        dist.destroy_process_group()


def test_sharded_plans_over_two_gloo_ranks(oracle):
    import torch.multiprocessing as mp
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    mp.start_processes(_worker, args=(2, _free_port(), root), nprocs=2, join=True, start_method="spawn")


def test_shard_plans_partition():
    from mako_attn.shard import head_shard, kv_shard
    for n, g in [(0, 2), (1, 2), (262144, 8), (1001, 3), (7, 8)]:
        ranges = [kv_shard(n, g, r) for r in range(g)]
        assert sum(c for _, c in ranges) == n
        pos = 0
        for s, c in ranges:
            assert s == pos and c >= 0
            pos += c
        assert max(c for _, c in ranges) - min(c for _, c in ranges) <= 1
    for H, KV, G in [(24, 24, 8), (64, 16, 8), (32, 8, 4), (16, 8, 2)]:
        covered = []
        for r in range(G):
            h0, hl, k0, kl = head_shard(H, KV, G, r)
            assert hl == kl * (H // KV) and h0 == k0 * (H // KV)
            covered += list(range(h0, h0 + hl))
        assert covered == list(range(H))
    with pytest.raises(ValueError):
        head_shard(24, 24, 5, 0)
