"""The attention calls are stream-ordered, allocate nothing once their scratch has grown and synchronise nothing, so a
serving loop can capture them in a CUDA graph.  After one eager call of each shape, a graph holding a batched decode,
a causal prefill and a block-sparse call (bf16: the V pre-pass is in the graph too) replays on new inputs written
into the same buffers, and its outputs equal, bit for bit, eager calls on those inputs."""
import numpy as np
import pytest

import attn_cases as C

pytestmark = pytest.mark.gpu


def test_capture_and_replay(ctx):
    import torch
    g0 = torch.Generator().manual_seed(5)

    def randn(*shape):
        return torch.randn(*shape, generator=g0).to(torch.bfloat16).cuda()

    # decode: 4 sequences, 8 q / 2 kv heads of 128, cache of 2048 rows
    B, H, KV, D, S = 4, 8, 2, 128, 2048
    dq, dk, dv = randn(B, H, D), randn(B, KV, S, D), randn(B, KV, S, D)
    lens = torch.tensor([2048, 1, 700, 1500], dtype=torch.int32, device="cuda")
    do = torch.empty(B, H * D, device="cuda")
    # causal prefill: 4 q / 2 kv heads, 600 rows
    n, hq, hk = 600, 4, 2
    q_pad, k_pad = C.round_up(n, 64), C.round_up(n, 128)
    pq, pk, pv = randn(hq, q_pad, D), randn(hk, k_pad, D), randn(hk, k_pad, D)
    po = torch.empty(n, hq * D, device="cuda")
    # block-sparse: 2 heads, 512 rows, config 4's list format
    sh, sn = 2, 512
    lists, counts = C.block_lists(9, sh, sn // 64, 0.3)
    lists_d, counts_d = torch.from_numpy(lists).cuda(), torch.from_numpy(counts).cuda()
    sq, sk, sv = randn(sh, sn, D), randn(sh, sn, D), randn(sh, sn, D)
    so = torch.empty(sn, sh * D, device="cuda")
    inputs = [dq, dk, dv, pq, pk, pv, sq, sk, sv]
    outputs = [do, po, so]

    def calls():
        ctx.attention_decode(dq, dk, dv, do, lens, S, H, KV, D, S)
        ctx.attention(pq, pk, pv, po, n, q_pad, n, k_pad, hq, hk, 0, 0xFFFFFFFF, D)
        ctx.attention_block_sparse(sq, sk, sv, so, sn, sh, sh, lists_d, counts_d)

    calls()  # grows the context's scratch
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        calls()
    for t in inputs:  # new values in the captured buffers
        t.copy_(randn(*t.shape))
    graph.replay()
    torch.cuda.synchronize()
    replayed = [o.clone() for o in outputs]
    calls()
    torch.cuda.synchronize()
    assert ctx.device_error() == 0
    for got, want in zip(replayed, outputs):
        assert torch.isfinite(want).all()
        assert torch.equal(got, want)
    del graph
