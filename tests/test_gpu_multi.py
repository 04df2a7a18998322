"""The sharded forms across real GPUs: one process per GPU (spawned here), exchange areas and outputs mapped through
CUDA IPC, handles passed over a gloo process group.  Each rank checks the gathered output / merged decode against the
unsharded oracle, over two calls (both flag parities).  Skipped with fewer than two GPUs."""
import os
import socket

import numpy as np
import pytest

pytestmark = [pytest.mark.gpu, pytest.mark.timeout(600)]


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, root):
    import sys
    for p in (os.path.join(root, "mako-common_b200"), os.path.join(root, "oracle"), os.path.join(root, "tests")):
        sys.path.insert(0, p)
    import torch
    import torch.distributed as dist
    import attn_cases as C
    import mako_attn
    import oracle as O
    from mako_attn.shard import head_shard, kv_shard

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    torch.cuda.set_device(rank)
    dist.init_process_group("gloo", rank=rank, world_size=world)

    def exchange(b):
        out = [None] * world
        dist.all_gather_object(out, b)
        return out

    def dev(bits, dtype):
        t = torch.from_numpy(np.ascontiguousarray(bits).view(np.int16))
        return t.view(torch.bfloat16 if dtype == 1 else torch.float16).cuda()

    ctx = mako_attn.Context(rank)
    group = mako_attn.Group(ctx, rank, world, 256, exchange)
    obuf = None
    try:
        # head-sharded prefill with the fused gather
        H, KV, n = 2 * world, world, 520
        d = C.dense_case(seed=61, heads=H, kv_heads=KV, dim=128, n_q=n, n_k=n, dtype=1)
        head0, hl, kv0, kvl = head_shard(H, KV, world, rank)
        q = dev(d["q"][head0:head0 + hl], 1)
        k, v = dev(d["k"][kv0:kv0 + kvl], 1), dev(d["v"][kv0:kv0 + kvl], 1)
        want = O.attention(1, d["q"], d["k"], d["v"], n, d["q_pad"], n, d["k_pad"], H, KV, 0, C.UINT32_MAX, 128)
        width = H * 128
        obuf = mako_attn.PeerBuffer(ctx, n * width * 4, rank, exchange, shape=(n, width))
        for _ in range(2):
            obuf.tensor.fill_(12345.0)
            group.attention_gather(q, k, v, obuf.ptrs, n, d["q_pad"], n, d["k_pad"], hl, kvl, head0, width)
            torch.cuda.synchronize()
            assert ctx.device_error() == 0, "a wait ran out"
            ok, stats = C.within(obuf.tensor.cpu().numpy(), want)
            assert ok, f"rank {rank} gather: {stats}"
            dist.barrier()

        # KV-sharded decode of long sequences
        c = C.decode_case(seed=62, batch=2, heads=32, kv_heads=8, dim=128, lo=3000, hi=20000, dtype=0)
        shards = [kv_shard(int(L), world, rank) for L in c["kv_len"]]
        nloc = np.array([m for _, m in shards], np.int32)
        stride = C.round_up(int(nloc.max()), 64)
        kl = np.zeros((2, 8, stride, 128), np.uint16)
        vl = np.zeros_like(kl)
        for b, (s, m) in enumerate(shards):
            kl[b, :, :m] = c["k"][b, :, s:s + m]
            vl[b, :, :m] = c["v"][b, :, s:s + m]
        want = O.decode(0, c["q"], c["k"], c["v"], c["kv_len"], 32, 8, 128, c["k_stride"])
        qd, kd, vd = dev(c["q"], 0), dev(kl, 0), dev(vl, 0)
        lens = torch.from_numpy(nloc).cuda()
        for _ in range(2):
            o = torch.full((2, 32 * 128), 12345.0, dtype=torch.float32, device="cuda")
            group.attention_decode_kv_sharded(qd, kd, vd, o, lens, int(nloc.max()), 32, 8, 128, stride)
            torch.cuda.synchronize()
            assert ctx.device_error() == 0, "a wait ran out"
            ok, stats = C.within(o.cpu().numpy(), want)
            assert ok, f"rank {rank} decode: {stats}"
        dist.barrier()
    finally:
        torch.cuda.synchronize()
        dist.barrier()  # no rank unmaps while another may still store into its memory
        if obuf is not None:
            obuf.close()
        group.close()
        ctx.close()
        dist.destroy_process_group()


def test_sharded_forms_across_gpus(oracle):
    import torch
    n = torch.cuda.device_count() if torch.cuda.is_available() else 0
    if n < 2:
        pytest.skip("needs two or more GPUs")
    world = 8 if n >= 8 else (4 if n >= 4 else 2)
    import torch.multiprocessing as mp
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    mp.start_processes(_worker, args=(world, _free_port(), root), nprocs=world, join=True, start_method="spawn")
