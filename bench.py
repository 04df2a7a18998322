#!/usr/bin/env python
"""Benchmark of the B200 attention path (one JSON line on stdout, rank 0).

  python bench.py [--gpus N] [--steps K] [--warmup W] [--workload NAME] [--impl mako|reference]

Workloads (synthetic seeded data -- no dataset is involved):
  decode         configs[1]: GQA decode fp16, batch 8, 32 q / 8 kv heads, D 128, KV lengths U[16384, 32768]
  prefill        configs[2]: causal GQA prefill bf16, batch 2 (folded into heads), 32 / 8 heads, D 128, S 8192
  sparse         configs[3]: block-sparse bf16, 24 heads, D 128, S 16384, 64x64 blocks, diagonal + 15% per row
  bidir          configs[4]: bidirectional bf16, 24 heads, D 128, N 75600, RMS-normalised q and k  (default: the
                 north star's head-sharded scaling config)
  prefill_small  configs[0]: causal GQA prefill fp16, 16 / 8 heads, D 128, S 512
  decode_long    configs[1]'s variant: one sequence of 262144 fp16 keys, 32 / 8 heads, D 128
  heads          the head-tile producers (RMS norm + RoPE into bf16 tiles) at configs[2]'s shape
  prefill_d256   not a BASELINE config: causal GQA prefill bf16 with Qwen3.5's 256-wide gated-attention heads,
                 16 / 2 heads, S 8192
  proj           the output projection after configs[2]'s attention: 16384 x 4096 bf16 o times a 4096 x 4096 bf16
                 matrix (the consumer of the attention's 16-bit output)
A step is one call of the public C ABI (include/mako_attn.h) over one batch held in HBM; `value` is device time
(CUDA events on the launching stream, max over ranks; L2 flushed between steps by a 256 MB write followed by a
256 MB read, so that the step finds neither its inputs nor the flush's dirty lines in L2, except for an HBM-bound
step whose inputs exceed 4x the 126 MB L2, `config.l2` says which); `e2e` is the same metric with the step's inputs
copied from pinned host memory and its output read back inside the timed region (on one GPU the dense and block-sparse
workloads split a large step into calls over groups of heads whose copies overlap the other groups' attention;
`e2e.pipelined` says how, and `e2e.matches_one_call_output` that the output read back equals the one-call step's bit
for bit).  With N > 1 the decode / prefill_small / prefill_d256 / sparse workloads run one replica per GPU (weak
scaling); prefill and bidir shard the heads over the GPUs with the output all-gather fused into the attention kernel,
and decode_long shards the keys with a cross-GPU log-sum-exp combine (strong scaling: `value` is the one problem's
work over the slowest rank's time).

--impl reference times the reference's scalar attention restated on the CPU (oracle/, all host threads) on a
bounded sample of the same workload: the reference itself is Metal-only and cannot run here.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import sys
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
for p in (os.path.join(ROOT, "mako-common_b200"), os.path.join(ROOT, "oracle"), os.path.join(ROOT, "tests")):
    if p not in sys.path:
        sys.path.insert(0, p)

UINT32_MAX = 0xFFFFFFFF
L2_FLUSH_BYTES = 256 << 20  # > 126 MB L2
L2_BYTES = 126 << 20
# The flush: a write larger than L2 evicts the previous step's lines; the read after it evicts the flush's own dirty
# lines, whose write-back would otherwise land inside the next timed step.
L2_FLUSH_NOTE = "flushed between steps (256 MB write, then a 256 MB read: no input and no dirty line left in L2)"


def peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            m = json.load(f)
        return float(m["hbm_gbs"]), float(m["bf16_tflops"]), "measured"
    except Exception:
        return 6650.0, 1590.0, "fallback"


def round_up(x, m):
    return (x + m - 1) // m * m


# ---- workloads ------------------------------------------------------------------------------------------------------

def l2_flushed(W):
    """Whether L2 is flushed (L2_FLUSH_NOTE) between timed steps of W, recorded in W.config["l2"]: yes, except for
    an HBM-bound step whose inputs are more than 4x the L2 -- it cannot hit L2 across steps."""
    in_bytes = sum(t.numel() * t.element_size() for t in W.inputs)
    if W.bound == "hbm" and in_bytes >= 4 * L2_BYTES:
        W.config["l2"] = (f"not flushed: the step's inputs ({in_bytes / 1e6:.0f} MB per GPU) are more than 4x the "
                          "126 MB L2")
        return False
    return True


class Workload:
    """Holds device inputs, knows its algorithmic work, runs one step through the C ABI."""
    name = ""
    metric = ""
    unit = ""
    bound = "tensor"
    dtype = "bf16"

    scaling = "weak"  # "weak": every rank runs the whole workload (replicas); "strong": ranks share one problem

    def work(self) -> float:  # algorithmic units (bytes or FLOP) this rank's part of a step does
        raise NotImplementedError

    def total_work(self, world: int) -> float:  # units the whole job does per step
        return self.work() * world

    def setup(self, ctx, world, rank, exchange):  # multi-GPU state (sharded workloads)
        pass

    def close(self):
        pass

    def to_metric(self, units_per_s: float) -> float:
        return units_per_s / (1e9 if self.bound == "hbm" else 1e12)


DEVICE = "cuda"  # "cpu" for the reference arm, which needs no GPU


def gen_heads(first, count, rows, dim, dtype, seed, scale=1.0, rms_norm=False, row0=0, chunk=4096):
    """[count][rows][dim] of heads first .. first + count - 1, rows row0 .. row0 + rows - 1 of each head's stream: each
    4096-row chunk of a head has its own seed, so a rank generates only its share and every GPU count sees the same
    values."""
    import torch
    out = torch.empty((count, rows, dim), dtype=dtype, device=DEVICE)
    for i in range(count):
        c0, c1 = row0 // chunk, (row0 + rows + chunk - 1) // chunk
        parts = []
        for c in range(c0, c1):
            g = torch.Generator(device="cpu")
            g.manual_seed(seed * 1000003 + (first + i) * 4099 + c)
            parts.append(torch.randn((chunk, dim), generator=g, dtype=torch.float32))
        x = torch.cat(parts)[row0 - c0 * chunk:row0 - c0 * chunk + rows]
        if rms_norm:
            x = x * torch.rsqrt((x * x).mean(dim=-1, keepdim=True))
        out[i] = (x * scale).to(dtype).to(DEVICE)
    return out


def gen(shape, dtype, seed, scale=1.0, rms_norm=False):
    """Seeded N(0, 1) from torch's CPU generator (the same values for both arms), moved to DEVICE."""
    import torch
    g = torch.Generator(device="cpu")
    g.manual_seed(seed)
    x = torch.randn(shape, generator=g, dtype=torch.float32)
    if rms_norm:
        x = x * torch.rsqrt((x * x).mean(dim=-1, keepdim=True))
    return (x * scale).to(dtype).to(DEVICE)


class Decode(Workload):
    name, metric, unit, bound, dtype = "decode", "decode KV-read GB/s (GQA, split-KV)", "GB/s", "hbm", "fp16"

    def __init__(self, seed=0):
        import numpy as np
        import torch
        self.B, self.H, self.KV, self.D = 8, 32, 8, 128
        rng = np.random.default_rng(seed)
        self.lens = rng.integers(16384, 32768 + 1, size=self.B).astype(np.int32)
        self.S = int(round_up(int(self.lens.max()), 64))
        self.q = gen((self.B, self.H, self.D), torch.float16, seed + 1)
        self.k = gen((self.B, self.KV, self.S, self.D), torch.float16, seed + 2)
        self.v = gen((self.B, self.KV, self.S, self.D), torch.float16, seed + 3)
        for b in range(self.B):  # rows past a sequence's length are zero, as a cache leaves them
            self.k[b, :, self.lens[b]:] = 0
            self.v[b, :, self.lens[b]:] = 0
        self.kv_len = torch.from_numpy(self.lens).to(DEVICE)
        self.o = torch.empty((self.B, self.H * self.D), dtype=torch.float32, device=DEVICE)
        self.inputs = [self.q, self.k, self.v]
        self.outputs = [self.o]
        self.launches_per_step = 2
        self.config = {"workload": "decode (configs[1])", "batch": self.B, "q_heads": self.H, "kv_heads": self.KV,
                       "head_dim": self.D, "kv_len": [int(x) for x in self.lens], "kv_len_seed": seed,
                       "cache_rows": self.S, "dtype": "fp16", "l2": L2_FLUSH_NOTE}

    def work(self):
        return float(sum(2 * self.KV * int(L) * self.D * 2 for L in self.lens) + self.B * self.H * self.D * (2 + 4))

    def step(self, ctx):
        ctx.attention_decode(self.q, self.k, self.v, self.o, self.kv_len, int(self.lens.max()), self.H, self.KV,
                             self.D, self.S)

    # CPU sample: the whole workload (the oracle decode is a few seconds on a host)
    def cpu_sample(self, O, threads, target_s=None):
        import numpy as np
        nb = self.B  # the whole batch: a few tenths of a second on a host
        q = self.q[:nb].cpu().view(torch_int16()).numpy().view(np.uint16)
        k = self.k[:nb].cpu().view(torch_int16()).numpy().view(np.uint16)
        v = self.v[:nb].cpu().view(torch_int16()).numpy().view(np.uint16)
        lens = self.lens[:nb]

        def run():
            return O.decode(0, q, k, v, lens, self.H, self.KV, self.D, self.S, nthreads=threads)
        work = float(sum(2 * self.KV * int(L) * self.D * 2 for L in lens) + nb * self.H * self.D * 6)
        return run, work, f"batch {nb} of {self.B} (all heads, full lengths)"

    def check(self, O):
        import numpy as np
        b = [0, self.B - 1]
        got = self.o[b].cpu().numpy()
        q = self.q[b].cpu().view(torch_int16()).numpy().view(np.uint16)
        k = self.k[b].cpu().view(torch_int16()).numpy().view(np.uint16)
        v = self.v[b].cpu().view(torch_int16()).numpy().view(np.uint16)
        want = O.decode(0, q, k, v, self.lens[b], self.H, self.KV, self.D, self.S)
        return got, want, "sequences 0 and 7"


class HeadGroupE2E:
    """The end-to-end leg at N = 1 as one call per group of heads (e2e_groups: q head and kv head ranges; e2e_call:
    the call for one group into its own [S][group heads * D] output block), pipelined over three streams: a group's
    q, k and v are copied in on one stream, attended on the launching stream and read back on a third, so that the
    copies of one group overlap the attention of another."""

    def e2e_host_outputs(self):
        """Pinned host buffers for the output, one block per call (and the device blocks the calls write)."""
        import torch
        self.o_groups = [torch.empty((self.S, (h1 - h0) * self.D), dtype=torch.float32, device=DEVICE)
                         for h0, h1, _, _ in self.e2e_groups()]
        return [torch.empty(t.shape, dtype=t.dtype, pin_memory=True) for t in self.o_groups]

    def e2e_note(self):
        n = len(self.e2e_groups())
        if n == 1:
            return "one call a step: q, k and v copied in, attended, o read back, one after another"
        return (f"{n} calls a step, one per group of heads: a group's q, k and v copied in on one stream, attended on "
                "the launching stream, its o read back on a third, each waiting only for its own group's previous "
                "stage")

    def e2e_step(self, ctx, host_in, host_out, main, s_in, s_out):
        import torch
        hq, hk, hv = host_in
        s_in.wait_stream(main)  # the step's start: the previous step's calls have read q, k and v
        for (h0, h1, k0, k1), og, ho in zip(self.e2e_groups(), self.o_groups, host_out):
            with torch.cuda.stream(s_in):
                self.q[h0:h1].copy_(hq[h0:h1], non_blocking=True)
                self.k[k0:k1].copy_(hk[k0:k1], non_blocking=True)
                self.v[k0:k1].copy_(hv[k0:k1], non_blocking=True)
            main.wait_stream(s_in)
            self.e2e_call(ctx, h0, h1, k0, k1, og, main)
            s_out.wait_stream(main)
            with torch.cuda.stream(s_out):
                ho.copy_(og, non_blocking=True)
        main.wait_stream(s_out)

    def e2e_matches(self, host_out):
        """The pipelined calls' output equals the one-call step's o bit for bit (heads are independent)."""
        import torch
        o = self.o.cpu()
        return all(torch.equal(ho, o[:, h0 * self.D:h1 * self.D])
                   for (h0, h1, _, _), ho in zip(self.e2e_groups(), host_out))


class Prefill(HeadGroupE2E, Workload):
    """Dense masked prefill; batch folded into heads (head h of batch b is head b * H + h).  With N > 1 GPUs the heads
    are sharded (whole GQA groups per rank, mako_attn/shard.py) and every rank's output slice is stored into every
    rank's o by the kernel itself (mako_attention_gather): strong scaling of one problem."""
    bound = "tensor"

    def __init__(self, name, metric, B, H, KV, D, S, dtype, scale, block, seed, rms_qk=False, cfg="", world=1,
                 rank=0, sharded=False):
        import torch
        from mako_attn.shard import head_shard
        self.name, self.metric, self.unit = name, metric, "TFLOP/s"
        self.B, self.H, self.KV, self.D, self.S, self.block = B, H, KV, D, S, block
        self.tdtype = torch.bfloat16 if dtype == "bf16" else torch.float16
        self.dtype = dtype
        self.seed, self.scale, self.rms_qk = seed, scale, rms_qk
        self.heads_all, self.kv_all = B * H, B * KV
        self.world, self.rank = world, rank
        self.head0, self.heads, self.kv0, self.kv_heads = head_shard(self.heads_all, self.kv_all, world, rank)
        # sharded: one problem at every N (its heads shared out when N > 1); else one replica per GPU
        self.scaling = "strong" if sharded else "weak"
        self.q_pad, self.k_pad = round_up(S, 64), round_up(S, 128)
        self.q = torch.zeros((self.heads, self.q_pad, D), dtype=self.tdtype, device=DEVICE)
        self.k = torch.zeros((self.kv_heads, self.k_pad, D), dtype=self.tdtype, device=DEVICE)
        self.v = torch.zeros_like(self.k)
        self.q[:, :S] = gen_heads(self.head0, self.heads, S, D, self.tdtype, seed + 1, scale, rms_qk)
        self.k[:, :S] = gen_heads(self.kv0, self.kv_heads, S, D, self.tdtype, seed + 2, scale, rms_qk)
        self.v[:, :S] = gen_heads(self.kv0, self.kv_heads, S, D, self.tdtype, seed + 3, scale)
        self.width = self.heads_all * D
        self.obuf = self.group = None
        self.o = torch.empty((S, self.width), dtype=torch.float32, device=DEVICE) if world == 1 else None
        self.inputs = [self.q, self.k, self.v]
        self.outputs = [self.o]
        self.config = {"workload": cfg, "batch": B, "q_heads": H, "kv_heads": KV, "head_dim": D, "seq_len": S,
                       "mask": "causal" if block == UINT32_MAX else ("bidirectional" if block == 0 else f"block {block}"),
                       "dtype": dtype, "input_scale": scale, "rms_norm_qk": rms_qk, "seed": seed,
                       "l2": L2_FLUSH_NOTE}
        if world > 1:
            self.config["sharding"] = (f"heads: {self.heads} q / {self.kv_heads} kv heads per rank, output slices "
                                       "stored into every rank's o by the attention kernel (fused all-gather)")

    def setup(self, ctx, world, rank, exchange):
        if world == 1:
            return
        import mako_attn
        self.group = mako_attn.Group(ctx, rank, world, 1, exchange)
        self.obuf = mako_attn.PeerBuffer(ctx, self.S * self.width * 4, rank, exchange, shape=(self.S, self.width))
        self.o = self.obuf.tensor
        self.outputs = [self.o]

    def close(self):
        import torch
        torch.cuda.synchronize()
        if self.obuf is not None:
            self.obuf.close()
        if self.group is not None:
            self.group.close()

    def visible(self, i):
        return self.S if (i >= self.block) else min(self.S, i + 1)

    def _pairs(self):
        if self.block == UINT32_MAX:
            return self.S * (self.S + 1) / 2
        if self.block == 0:
            return float(self.S) * self.S
        return float(sum(self.visible(i) for i in range(self.S)))

    def work(self):
        return 4.0 * self.D * self.heads * self._pairs()

    def total_work(self, world):
        return 4.0 * self.D * self.heads_all * self._pairs() if world > 1 else self.work() * world

    def step(self, ctx):
        if self.group is None:
            ctx.attention(self.q, self.k, self.v, self.o, self.S, self.q_pad, self.S, self.k_pad, self.heads,
                          self.kv_heads, 0, self.block, self.D)
        else:
            self.group.attention_gather(self.q, self.k, self.v, self.obuf.ptrs, self.S, self.q_pad, self.S,
                                        self.k_pad, self.heads, self.kv_heads, self.head0, self.width, 0, self.block)

    # -- the end-to-end leg at N = 1: whole GQA groups of heads, one call each (HeadGroupE2E)
    E2E_GROUPS = 8              # calls a step at most
    E2E_GROUP_BYTES = 32 << 20  # inputs a call at least: a smaller step is not worth splitting

    def e2e_groups(self):
        """(q head range, kv head range) of each call: the kv heads in up to E2E_GROUPS runs."""
        g = self.heads // self.kv_heads
        in_bytes = sum(t.numel() * t.element_size() for t in self.inputs)
        n = max(1, min(self.E2E_GROUPS, self.kv_heads, in_bytes // self.E2E_GROUP_BYTES))
        cut = [round(i * self.kv_heads / n) for i in range(n + 1)]
        return [(a * g, b * g, a, b) for a, b in zip(cut, cut[1:]) if b > a]

    def e2e_call(self, ctx, h0, h1, k0, k1, o, stream):
        ctx.attention(self.q[h0:h1], self.k[k0:k1], self.v[k0:k1], o, self.S, self.q_pad, self.S, self.k_pad, h1 - h0,
                      k1 - k0, 0, self.block, self.D, width=(h1 - h0) * self.D, stream=stream)

    def sample_rows(self, n):
        import numpy as np
        return np.unique(np.linspace(0, self.S - 1, n).astype(np.uint32))

    def _bits(self):
        """All heads' inputs as 16-bit patterns on the host (regenerated when this rank holds a shard)."""
        import numpy as np
        code = 1 if self.dtype == "bf16" else 0
        f = lambda t: t.cpu().view(torch_int16()).numpy().view(np.uint16)  # noqa: E731
        if self.world == 1:
            return code, f(self.q), f(self.k), f(self.v)
        global DEVICE
        dev, DEVICE = DEVICE, "cpu"
        try:
            q = np.zeros((self.heads_all, self.q_pad, self.D), np.uint16)
            k = np.zeros((self.kv_all, self.k_pad, self.D), np.uint16)
            v = np.zeros_like(k)
            q[:, :self.S] = f(gen_heads(0, self.heads_all, self.S, self.D, self.tdtype, self.seed + 1, self.scale,
                                        self.rms_qk))
            k[:, :self.S] = f(gen_heads(0, self.kv_all, self.S, self.D, self.tdtype, self.seed + 2, self.scale,
                                        self.rms_qk))
            v[:, :self.S] = f(gen_heads(0, self.kv_all, self.S, self.D, self.tdtype, self.seed + 3, self.scale))
        finally:
            DEVICE = dev
        return code, q, k, v

    def cpu_sample(self, O, threads, target_s=10.0):
        code, q, k, v = self._bits()
        # rows per second on this host, from a small probe, then a sample sized for ~target_s
        probe = self.sample_rows(8)
        t0 = time.perf_counter()
        O.attention(code, q, k, v, self.S, self.q_pad, self.S, self.k_pad, self.heads_all, self.kv_all, 0,
                    self.block, self.D, rows=probe, nthreads=threads)
        dt = max(time.perf_counter() - t0, 1e-3)
        n = int(min(self.S, max(8, len(probe) * target_s / dt)))
        rows = self.sample_rows(n)
        work = float(sum(4 * self.D * self.heads_all * self.visible(int(i)) for i in rows))

        def run():
            return O.attention(code, q, k, v, self.S, self.q_pad, self.S, self.k_pad, self.heads_all, self.kv_all, 0,
                               self.block, self.D, rows=rows, nthreads=threads)
        return run, work, f"{len(rows)} of {self.S} query rows (evenly spaced), all {self.heads_all} heads; " \
                          "rate extrapolated linearly in rows"

    def check(self, O):
        code, q, k, v = self._bits()
        rows = self.sample_rows(24)
        want = O.attention(code, q, k, v, self.S, self.q_pad, self.S, self.k_pad, self.heads_all, self.kv_all, 0,
                           self.block, self.D, rows=rows)
        what = f"{len(rows)} query rows x all heads" + (" (the gathered o of rank 0)" if self.world > 1 else "")
        return self.o.cpu().numpy()[rows], want[rows], what


class DecodeLong(Workload):
    """BASELINE config 2's single-sequence variant: one query per head over a 262144-token fp16 cache, 32 q / 8 kv
    heads.  With N > 1 GPUs each rank holds a contiguous 1/N of the keys and mako_attention_decode_kv_sharded merges
    the ranks' partial rows over NVLink (strong scaling of one problem)."""
    name, metric, unit, bound, dtype = "decode_long", "decode KV-read GB/s (GQA, split-KV)", "GB/s", "hbm", "fp16"

    def __init__(self, seed=0, world=1, rank=0, L=262144):
        import torch
        from mako_attn.shard import kv_shard
        self.H, self.KV, self.D, self.L, self.seed = 32, 8, 128, L, seed
        self.world, self.rank = world, rank
        self.start, self.n = kv_shard(L, world, rank)
        self.stride = round_up(max(self.n, 1), 64)
        self.scaling = "strong"  # one sequence at every N (its keys shared out when N > 1)
        self.q = gen_heads(0, 1, self.H, self.D, torch.float16, seed + 1)  # [1][H][D]
        self.k = torch.zeros((1, self.KV, self.stride, self.D), dtype=torch.float16, device=DEVICE)
        self.v = torch.zeros_like(self.k)
        self.k[0, :, :self.n] = gen_heads(0, self.KV, self.n, self.D, torch.float16, seed + 2, row0=self.start)
        self.v[0, :, :self.n] = gen_heads(0, self.KV, self.n, self.D, torch.float16, seed + 3, row0=self.start)
        self.kv_len = torch.tensor([self.n], dtype=torch.int32, device=DEVICE)
        self.o = torch.empty((1, self.H * self.D), dtype=torch.float32, device=DEVICE)
        self.inputs, self.outputs = [self.q, self.k, self.v], [self.o]
        self.group = None
        self.config = {"workload": "decode_long (configs[1], 262144-token single-sequence variant)", "batch": 1,
                       "q_heads": self.H, "kv_heads": self.KV, "head_dim": self.D, "kv_len": L, "dtype": "fp16",
                       "l2": L2_FLUSH_NOTE}
        if world > 1:
            self.config["sharding"] = (f"keys: {self.n} of {L} per rank; partial rows pushed to every rank over "
                                       "NVLink and merged by log-sum-exp in one kernel")

    def setup(self, ctx, world, rank, exchange):
        if world > 1:
            import mako_attn
            self.group = mako_attn.Group(ctx, rank, world, self.H, exchange)

    def close(self):
        import torch
        torch.cuda.synchronize()
        if self.group is not None:
            self.group.close()

    def work(self):
        return float(2 * self.KV * self.n * self.D * 2 + self.H * self.D * (2 + 4))

    def total_work(self, world):
        return float(2 * self.KV * self.L * self.D * 2 + self.H * self.D * (2 + 4)) if world > 1 else \
            self.work() * world

    def step(self, ctx):
        if self.group is None:
            ctx.attention_decode(self.q, self.k, self.v, self.o, self.kv_len, self.n, self.H, self.KV, self.D,
                                 self.stride)
        else:
            self.group.attention_decode_kv_sharded(self.q, self.k, self.v, self.o, self.kv_len, self.n, self.H,
                                                   self.KV, self.D, self.stride)

    def _full(self):
        import numpy as np
        import torch
        global DEVICE
        f = lambda t: t.cpu().view(torch_int16()).numpy().view(np.uint16)  # noqa: E731
        dev, DEVICE = DEVICE, "cpu"
        try:
            q = f(self.q)
            k = f(gen_heads(0, self.KV, self.L, self.D, torch.float16, self.seed + 2))[None]
            v = f(gen_heads(0, self.KV, self.L, self.D, torch.float16, self.seed + 3))[None]
        finally:
            DEVICE = dev
        return q, k, v

    def cpu_sample(self, O, threads, target_s=None):
        import numpy as np
        q, k, v = self._full()
        lens = np.array([self.L], np.int32)

        def run():
            return O.decode(0, q, k, v, lens, self.H, self.KV, self.D, self.L, nthreads=threads)
        return run, float(2 * self.KV * self.L * self.D * 2 + self.H * self.D * 6), "the whole sequence, all heads"

    def check(self, O):
        import numpy as np
        q, k, v = self._full()
        want = O.decode(0, q, k, v, np.array([self.L], np.int32), self.H, self.KV, self.D, self.L)
        return self.o.cpu().numpy(), want, "all 32 heads" + (" (rank 0's merged o)" if self.world > 1 else "")


class Proj(Workload):
    """The output projection after configs[2]'s attention: the 16-bit o of batch 2 x 8192 tokens x 32 heads of 128
    (x [16384][4096] bf16) times the 4096 x 4096 bf16 matrix, fp32 y (mako_proj; Runtime::proj as
    src/models/qwen_text.cpp:312 calls it).  Tensor-bound: 2 T k n FLOP."""
    name, metric, unit, bound, dtype = "proj", "output projection TFLOP/s (bf16 GEMM after the attention)", \
        "TFLOP/s", "tensor", "bf16"

    def __init__(self, seed=0):
        import torch
        self.T, self.k, self.n = 2 * 8192, 32 * 128, 32 * 128
        self.x = gen((self.T, self.k), torch.bfloat16, seed + 1, 0.5)
        self.w = gen((self.n, self.k), torch.bfloat16, seed + 2, 0.02)
        self.y = torch.empty((self.T, self.n), dtype=torch.float32, device=DEVICE)
        self.inputs, self.outputs = [self.x, self.w], [self.y]
        self.config = {"workload": "proj (configs[2]'s output projection: 16384 tokens x 4096 -> 4096, bf16)",
                       "T": self.T, "k": self.k, "n": self.n, "dtype": "bf16", "seed": seed,
                       "l2": L2_FLUSH_NOTE}

    def work(self):
        return 2.0 * self.T * self.k * self.n

    def step(self, ctx):
        ctx.proj(self.w, self.x, self.y, self.T, self.k, self.n)

    def _bits(self):
        import numpy as np
        f = lambda t: t.cpu().view(torch_int16()).numpy().view(np.uint16)  # noqa: E731
        return f(self.x), f(self.w)

    def cpu_sample(self, O, threads, target_s=10.0):
        import numpy as np
        x, w = self._bits()
        t0 = time.perf_counter()
        O.proj(1, w, x, self.T, self.k, self.n, rows=np.arange(4, dtype=np.uint32), nthreads=threads)
        dt = max(time.perf_counter() - t0, 1e-3)
        rows = np.unique(np.linspace(0, self.T - 1, int(min(self.T, max(4, 4 * target_s / dt)))).astype(np.uint32))

        def run():
            return O.proj(1, w, x, self.T, self.k, self.n, rows=rows, nthreads=threads)
        return run, 2.0 * len(rows) * self.k * self.n, f"{len(rows)} of {self.T} rows (evenly spaced), all " \
                                                        f"{self.n} columns; rate extrapolated linearly in rows"

    def check(self, O):
        import numpy as np
        x, w = self._bits()
        rows = np.linspace(0, self.T - 1, 24).astype(np.uint32)
        want = O.proj(1, w, x, self.T, self.k, self.n, rows=rows)
        return self.y.cpu().numpy()[rows], want[rows], f"{len(rows)} rows x all columns"

    tolerance = "relative L2 <= 1e-5 against the double-precision GEMM of the same bf16 inputs"

    def within(self, got, want):
        import numpy as np
        err = np.asarray(got, np.float64) - np.asarray(want, np.float64)
        return float(np.sqrt(np.sum(err ** 2) / max(np.sum(np.asarray(want, np.float64) ** 2), 1e-30))) <= 1e-5


class Sparse(HeadGroupE2E, Workload):
    name, metric, unit, bound, dtype = "sparse", "block-sparse attention TFLOP/s on kept blocks", "TFLOP/s", \
        "tensor", "bf16"

    def __init__(self, seed=0):
        import torch
        import attn_cases as C
        self.H, self.D, self.S, self.frac = 24, 128, 16384, 0.15
        self.nb = self.S // 64
        lists, counts = C.block_lists(seed, self.H, self.nb, self.frac)
        self.lists_np, self.counts_np = lists, counts
        self.lists, self.counts = torch.from_numpy(lists).to(DEVICE), torch.from_numpy(counts).to(DEVICE)
        self.q = gen((self.H, self.S, self.D), torch.bfloat16, seed + 1)
        self.k = gen((self.H, self.S, self.D), torch.bfloat16, seed + 2)
        self.v = gen((self.H, self.S, self.D), torch.bfloat16, seed + 3)
        self.o = torch.empty((self.S, self.H * self.D), dtype=torch.float32, device=DEVICE)
        self.inputs, self.outputs = [self.q, self.k, self.v], [self.o]
        self.launches_per_step = 1
        self.config = {"workload": "sparse (configs[3])", "heads": self.H, "head_dim": self.D, "seq_len": self.S,
                       "block": 64, "kept_per_query_block": int(lists.shape[-1]), "keep_fraction": self.frac,
                       "mask": "int32 sorted kept-block lists + counts", "dtype": "bf16", "seed": seed,
                       "l2": L2_FLUSH_NOTE}

    def work(self):
        return float(int(self.counts_np.sum()) * 4 * 64 * 64 * self.D)

    def step(self, ctx):
        ctx.attention_block_sparse(self.q, self.k, self.v, self.o, self.S, self.H, self.H, self.lists, self.counts)

    # -- the end-to-end leg at N = 1: groups of heads, one call each (HeadGroupE2E)
    E2E_GROUPS = 8

    def e2e_groups(self):
        cut = [round(i * self.H / self.E2E_GROUPS) for i in range(self.E2E_GROUPS + 1)]
        return [(a, b, a, b) for a, b in zip(cut, cut[1:]) if b > a]

    def e2e_call(self, ctx, h0, h1, k0, k1, o, stream):
        ctx.attention_block_sparse(self.q[h0:h1], self.k[h0:h1], self.v[h0:h1], o, self.S, h1 - h0, h1 - h0,
                                   self.lists[h0:h1], self.counts[h0:h1], stream=stream)

    def _args(self, O):
        import numpy as np
        f = lambda t: t.cpu().view(torch_int16()).numpy().view(np.uint16)  # noqa: E731
        return (1, f(self.q), f(self.k), f(self.v), self.S, self.S, self.S, self.S, self.H, self.H, self.H * self.D,
                self.nb, self.lists_np.shape[-1], self.S, self.S, self.lists_np.astype(np.uint16),
                self.counts_np.astype(np.uint16), np.ones(self.S, np.uint8), np.arange(self.S, dtype=np.int32))

    def cpu_sample(self, O, threads, target_s=10.0):
        import numpy as np
        args = self._args(O)
        out = np.zeros((self.S, self.H * self.D), np.float32)
        probe = np.arange(0, self.S, self.S // 8, dtype=np.uint32)
        t0 = time.perf_counter()
        O.attention_sparse(*args, out=out, rows=probe, nthreads=threads)
        dt = max(time.perf_counter() - t0, 1e-3)
        n = int(min(self.S, max(8, len(probe) * target_s / dt)))
        rows = np.unique(np.linspace(0, self.S - 1, n).astype(np.uint32))
        kept = self.counts_np.sum(axis=0)  # per query block, over heads
        work = float(sum(int(kept[r // 64]) * 64 * 4 * self.D for r in rows))

        def run():
            return O.attention_sparse(*args, out=out, rows=rows, nthreads=threads)
        return run, work, f"{len(rows)} of {self.S} query rows, all heads; rate extrapolated linearly in rows"

    def check(self, O):
        import numpy as np
        rows = np.linspace(0, self.S - 1, 24).astype(np.uint32)
        out = np.zeros((self.S, self.H * self.D), np.float32)
        O.attention_sparse(*self._args(O), out=out, rows=rows)
        return self.o.cpu().numpy()[rows], out[rows], f"{len(rows)} query rows x all heads"


class Heads(Workload):
    """Head-tile producers at configs[2]'s 8B-model shape: per sequence (batch 2, 8192 tokens) the q, k and v tiles
    from fp32 projection rows -- q and k RMS-normed with their norm weights and rotated over all 128 values, v as is
    -- into bf16 [heads][8192][128] tiles (TransformerRuntime::heads_partial, as src/models/qwen_text.cpp:415-417
    calls it).  HBM-bound: bytes = fp32 rows read + bf16 tiles written + angle rows read."""
    name, metric, unit, bound, dtype = "heads", "head-tile producer GB/s (RMS norm + RoPE)", "GB/s", "hbm", "bf16"
    graph = True  # six short calls a step

    def __init__(self, seed=0):
        import torch
        self.B, self.T, self.H, self.KV, self.D = 2, 8192, 32, 8, 128
        g = torch.Generator(device="cpu")
        g.manual_seed(seed)
        B, T, H, KV, D = self.B, self.T, self.H, self.KV, self.D
        self.xq = torch.randn((B * T, H * D), generator=g).to(DEVICE)
        self.xk = torch.randn((B * T, KV * D), generator=g).to(DEVICE)
        self.xv = torch.randn((B * T, KV * D), generator=g).to(DEVICE)
        pos = torch.arange(T, dtype=torch.float64)[:, None]
        inv = 1.0 / (1.0e6 ** (torch.arange(D // 2, dtype=torch.float64) / (D // 2)))
        ang = pos * inv[None, :]
        self.cs = torch.stack([torch.cos(ang), torch.sin(ang)], -1).to(torch.float32).contiguous().to(DEVICE)
        self.wq = (1.0 + 0.1 * torch.randn(D, generator=g)).to(DEVICE)
        self.wk = (1.0 + 0.1 * torch.randn(D, generator=g)).to(DEVICE)
        self.qh = torch.empty((B * H, T, D), dtype=torch.bfloat16, device=DEVICE)
        self.kh = torch.empty((B * KV, T, D), dtype=torch.bfloat16, device=DEVICE)
        self.vh = torch.empty((B * KV, T, D), dtype=torch.bfloat16, device=DEVICE)
        self.inputs = [self.xq, self.xk, self.xv, self.cs, self.wq, self.wk]
        self.outputs = [self.qh, self.kh, self.vh]
        self.eps = 1e-6
        self.config = {"workload": "heads (configs[2] shape: batch 2, 8192 tokens, 32 q / 8 kv heads, D 128)",
                       "norm": "RMS on q and k (eps 1e-6)", "rotation": "all 128 values, halves", "tiles": "bf16",
                       "calls_per_step": 6, "l2": L2_FLUSH_NOTE}

    def work(self):
        B, T, H, KV, D = self.B, self.T, self.H, self.KV, self.D
        rows = B * T * (H + 2 * KV) * D
        return float(rows * 4 + rows * 2 + 2 * B * T * (D // 2) * 8)  # x read, tiles written, angles (q, k calls)

    def step(self, ctx):
        B, T, H, KV, D = self.B, self.T, self.H, self.KV, self.D
        for b in range(B):
            rows = slice(b * T, (b + 1) * T)
            ctx.heads_partial(self.xq[rows], H * D, 0, D, D, D, H, T, T, self.cs, self.wq, self.eps,
                              self.qh[b * H:(b + 1) * H])
            ctx.heads_partial(self.xk[rows], KV * D, 0, D, D, D, KV, T, T, self.cs, self.wk, self.eps,
                              self.kh[b * KV:(b + 1) * KV])
            ctx.heads_partial(self.xv[rows], KV * D, 0, D, D, 0, KV, T, T, None, None, 0.0,
                              self.vh[b * KV:(b + 1) * KV])

    def cpu_sample(self, O, threads, target_s=None):
        xq = self.xq[:self.T].cpu().numpy()
        cs = self.cs.cpu().numpy()
        wq = self.wq.cpu().numpy()
        T, H, D = self.T, self.H, self.D

        def run():
            return O.heads(xq, H * D, 0, D, D, D, 1, T, H, T, cs=cs, cs_row=D // 2, w=wq, eps=self.eps)
        rows = T * H * D
        return run, float(rows * 6 + T * (D // 2) * 8), "the q tiles of sequence 0 (8192 tokens x 32 heads)"

    tolerance = "one bf16 ulp of the oracle's value (or 1e-5 where it nearly cancels)"

    def within(self, got, want):
        import numpy as np
        w = np.asarray(want, np.float64)
        ulp = 2.0 ** (np.floor(np.log2(np.maximum(np.abs(w), 2.0 ** -14))) - 7)
        return bool(np.all(np.abs(np.asarray(got, np.float64) - w) <= np.maximum(ulp * 1.0001, 1e-5)))

    def check(self, O):
        import numpy as np
        T, H, D = self.T, self.H, self.D
        xq = self.xq[:T].cpu().numpy()
        want = O.heads(xq, H * D, 0, D, D, D, 1, T, H, T, cs=self.cs.cpu().numpy(), cs_row=D // 2,
                       w=self.wq.cpu().numpy(), eps=self.eps)
        want = O.from_bits(O.to_bits(want, 1), 1)  # the oracle's values rounded to the tiles' bf16
        got = self.qh[:H].float().cpu().numpy()
        return got.reshape(H * T, D), want.reshape(H * T, D), "the q tiles of sequence 0 against the oracle in bf16"


def torch_int16():
    import torch
    return torch.int16


def make_workload(name, world=1, rank=0):
    """The workload of `name` as rank `rank` of `world` sees it.  decode, sparse, prefill_small and prefill_d256 run
    one replica per GPU; prefill and bidir shard heads, decode_long shards keys (one problem across the GPUs)."""
    if name == "decode":
        return Decode()
    if name == "decode_long":
        return DecodeLong(world=world, rank=rank)
    if name == "prefill":
        return Prefill("prefill", "prefill attention TFLOP/s (causal GQA)", 2, 32, 8, 128, 8192, "bf16", 0.5,
                       UINT32_MAX, 0, cfg="prefill (configs[2])", world=world, rank=rank, sharded=True)
    if name == "prefill_small":
        return Prefill("prefill_small", "prefill attention TFLOP/s (causal GQA)", 1, 16, 8, 128, 512, "fp16", 1.0,
                       UINT32_MAX, 0, cfg="prefill_small (configs[0])")
    if name == "prefill_d256":
        return Prefill("prefill_d256", "prefill attention TFLOP/s (causal GQA, 256-wide heads)", 1, 16, 2, 256, 8192,
                       "bf16", 0.5, UINT32_MAX, 0,
                       cfg="prefill_d256 (Qwen3.5 gated-attention head shape, synthetic; not a BASELINE config)")
    if name == "bidir":
        return Prefill("bidir", "bidirectional attention TFLOP/s (video DiT)", 1, 24, 24, 128, 75600, "bf16", 1.0, 0,
                       0, rms_qk=True, cfg="bidir (configs[4])", world=world, rank=rank, sharded=True)
    if name == "sparse":
        return Sparse()
    if name == "heads":
        return Heads()
    if name == "proj":
        return Proj()
    raise SystemExit(f"unknown workload {name}")


# ---- clocks ---------------------------------------------------------------------------------------------------------

class Clocks:
    """SM clock and throttle reasons sampled through NVML every 5 ms by a background thread; the summary keeps the
    samples taken between mark_start() and mark_stop() (the timed region), else all of them."""
    REASONS = {"hw_slowdown": 0x8, "sw_thermal_slowdown": 0x20, "hw_thermal_slowdown": 0x40, "sw_power_cap": 0x4}

    def __init__(self, index):
        import threading
        self.samples, self.window, self.ok = [], [None, None], False
        try:
            import pynvml
            pynvml.nvmlInit()
            self.nv = pynvml
            self.h = pynvml.nvmlDeviceGetHandleByIndex(index)
            self.max_sm = pynvml.nvmlDeviceGetMaxClockInfo(self.h, pynvml.NVML_CLOCK_SM)
            self.ok = True
        except Exception as e:  # no NVML: reported, the run continues
            self.err = str(e)
        self.stop_flag = threading.Event()
        self.t = threading.Thread(target=self._loop, daemon=True)

    def _loop(self):
        while not self.stop_flag.is_set():
            try:
                sm = self.nv.nvmlDeviceGetClockInfo(self.h, self.nv.NVML_CLOCK_SM)
                rs = self.nv.nvmlDeviceGetCurrentClocksEventReasons(self.h)
                self.samples.append((time.perf_counter(), sm, rs))
            except Exception:
                pass
            time.sleep(0.005)

    def start(self):
        if self.ok:
            self.t.start()

    def mark_start(self):
        self.window[0] = time.perf_counter()

    def mark_stop(self):
        self.window[1] = time.perf_counter()

    def stop(self):
        if not self.ok:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [f"nvml unavailable: {self.err}"]}
        self.stop_flag.set()
        self.t.join(timeout=1)
        t0, t1 = self.window
        inside = [s for s in self.samples if t0 is not None and t1 is not None and t0 <= s[0] <= t1]
        use = inside or self.samples
        reasons = sorted(n for n, bit in self.REASONS.items() if any(s[2] & bit for s in use))
        return {"sm_mhz": statistics.median(s[1] for s in use) if use else None, "sm_max_mhz": self.max_sm,
                "reasons": reasons, "samples": len(use),
                "window": "timed region" if inside else "whole run (timed region shorter than one sample)"}


def merge_clocks(per_rank):
    """One clocks record from every rank's: sm_mhz the lowest per-rank median (the slowest GPU sets a step timed as
    the max over ranks), the per-rank medians beside it, and the throttle reasons any rank saw."""
    mhz = [c.get("sm_mhz") for c in per_rank]
    known = [m for m in mhz if m is not None]
    out = dict(per_rank[0])
    out["sm_mhz"] = min(known) if known else None
    out["per_rank_sm_mhz"] = mhz
    out["reasons"] = sorted({r for c in per_rank for r in c.get("reasons", [])})
    out["samples"] = sum(c.get("samples") or 0 for c in per_rank)
    return out


# ---- runs -----------------------------------------------------------------------------------------------------------

def dist_setup():
    import torch
    import torch.distributed as dist
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import datetime
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=180), device_id=torch.device("cuda", local))
    else:
        torch.cuda.set_device(0)
    return world, rank, local


def barrier(world):
    import torch
    if world > 1:
        import torch.distributed as dist
        dist.barrier()
    torch.cuda.synchronize()


def max_over_ranks(x, world):
    import torch
    if world == 1:
        return x
    import torch.distributed as dist
    t = torch.tensor([x], dtype=torch.float64, device=DEVICE)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def arm_config(W, world):
    """The config both arms print at N GPUs: the workload's own keys and how the N GPUs share it."""
    return dict(W.config, parallelism=("single GPU" if world == 1 else
                                       (f"sharded x{world}" if W.scaling == "strong" else f"replica x{world}")))


def read_traffic(name):
    """Per-launch DRAM bytes of the dominant kernel from the committed ncu summary (None if not captured)."""
    path = os.path.join(ROOT, "profiles", "dram_traffic.txt")
    try:
        for line in open(path):
            parts = line.split()
            if len(parts) >= 2 and parts[0] == name and not line.startswith("#"):
                return float(parts[1])
    except OSError:
        pass
    return None


def run_mako(args):
    import torch
    import mako_attn
    import oracle as O
    import attn_cases as C

    world, rank, local = dist_setup()
    W = make_workload(args.workload, world, rank)
    ctx = mako_attn.Context(local)
    if world > 1:  # IPC handles of the sharded workloads travel over a CPU group
        import torch.distributed as dist
        cpu_group = dist.new_group(backend="gloo")

        def exchange(b):
            out = [None] * world
            dist.all_gather_object(out, b, group=cpu_group)
            return out
        W.setup(ctx, world, rank, exchange)
    flushing = l2_flushed(W)
    flush = torch.empty(L2_FLUSH_BYTES // 4, dtype=torch.float32, device=DEVICE) if flushing else None
    flush_rd = torch.ones(L2_FLUSH_BYTES // 4, dtype=torch.float32, device=DEVICE) if flushing else None

    def flush_l2():
        if flush is not None:
            flush.zero_()
            flush_rd.amax()

    stream = torch.cuda.current_stream()

    clocks = Clocks(local)
    clocks.start()
    for _ in range(args.warmup):
        W.step(ctx)
    barrier(world)
    # A step of several short calls runs as a CUDA graph of those calls (captured once after the warm-up), so that the
    # device time is the kernels' and not the host's time to enqueue them one by one; the e2e leg below still makes
    # the calls directly.
    graph = None
    graph_launches = 0
    if getattr(W, "graph", False):
        graph = torch.cuda.CUDAGraph()
        n0 = ctx.launches()
        with torch.cuda.graph(graph):
            W.step(ctx)
        graph_launches = ctx.launches() - n0  # kernels in the graph, each replay launches them all
        graph.replay()
        torch.cuda.synchronize()
        W.config["timing"] = "device time of a CUDA graph holding the step's calls"
    run_step = graph.replay if graph is not None else (lambda: W.step(ctx))
    launches0 = ctx.launches()
    times = []
    barrier(world)
    clocks.mark_start()
    for _ in range(args.steps):
        flush_l2()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        run_step()
        e1.record(stream)
        times.append((e0, e1))
    barrier(world)
    clocks.mark_stop()
    launches = ctx.launches() - launches0 + graph_launches * (args.steps if graph is not None else 0)
    ms = [a.elapsed_time(b) for a, b in times]
    total_ms = max_over_ranks(sum(ms), world)
    ms_step = total_ms / args.steps
    work = W.work()
    value = W.to_metric(W.total_work(world) / (ms_step / 1e3))

    # end to end through the public API: pinned host inputs in, output back, every step.  A workload that can split
    # its step into independent calls (the dense ones: groups of heads) pipelines them over three streams, so that
    # one group's inputs cross PCIe while the previous group is attended and the one before it is read back.
    host_in = [t.cpu().pin_memory() for t in W.inputs]
    piped = world == 1 and hasattr(W, "e2e_groups")
    host_out = (W.e2e_host_outputs() if piped else
                [torch.empty(t.shape, dtype=t.dtype, pin_memory=True) for t in W.outputs])
    dev_in = W.inputs
    h2d = sum(t.numel() * t.element_size() for t in host_in)
    d2h = sum(t.numel() * t.element_size() for t in host_out)
    s_in, s_out = (torch.cuda.Stream(), torch.cuda.Stream()) if piped else (None, None)
    e2e_times = []
    barrier(world)
    for i in range(args.warmup + args.steps):
        flush_l2()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        if piped:
            W.e2e_step(ctx, host_in, host_out, stream, s_in, s_out)
        else:
            for d, h in zip(dev_in, host_in):
                d.copy_(h, non_blocking=True)
            W.step(ctx)
            for h, d in zip(host_out, W.outputs):
                h.copy_(d, non_blocking=True)
        e1.record(stream)
        if i >= args.warmup:
            e2e_times.append((e0, e1))
    barrier(world)
    e2e_ms = max_over_ranks(sum(a.elapsed_time(b) for a, b in e2e_times), world) / args.steps
    e2e_value = W.to_metric(W.total_work(world) / (e2e_ms / 1e3))
    e2e_extra = {}
    if piped:  # the pipelined calls' output, read back to the host, against the one-call step's o
        torch.cuda.synchronize()
        e2e_extra = {"pipelined": W.e2e_note(),
                     "matches_one_call_output": bool(W.e2e_matches(host_out))}

    # The dominant kernel alone: the library records a CUDA event pair around each call's main kernel on the
    # launching stream (MAKO_OPT_KERNEL_TIMING), over another K steps with the same L2 handling.  A graph step holds
    # nothing but the main kernels, so its replay time stands for them.
    kt = []
    if graph is None:
        ctx.set_option(mako_attn.OPT_KERNEL_TIMING, 1)
        ctx.kernel_times()
        barrier(world)
        for _ in range(args.steps):
            flush_l2()
            W.step(ctx)
        kt = ctx.kernel_times()
        ctx.set_option(mako_attn.OPT_KERNEL_TIMING, 0)
    barrier(world)
    clk = clocks.stop()
    if world > 1:  # every GPU's clocks: the slowest one sets the step
        clk = merge_clocks(exchange(clk))
    kernel_ms = max_over_ranks(sum(kt) / args.steps, world) if kt else None  # main kernels of one step

    hbm, tflops, src = peaks()
    call_ms = statistics.mean(ms)
    per_launch_ms = kernel_ms if kernel_ms else call_ms
    if W.bound == "hbm":
        achieved = work / (per_launch_ms / 1e3) / 1e9
        roof = {"bound": "hbm", "achieved": round(achieved, 1), "peak": hbm, "unit": "GB/s",
                "frac": round(achieved / hbm, 4), "peak_source": src}
    else:
        achieved = work / (per_launch_ms / 1e3) / 1e12
        roof = {"bound": "tensor", "achieved": round(achieved, 2), "peak": tflops, "unit": "TFLOP/s",
                "frac": round(achieved / tflops, 4), "peak_source": src}
    roof["traffic"] = read_traffic(W.name)
    roof["kernel_ms"] = round(per_launch_ms, 5)
    roof["call_ms"] = round(call_ms, 5)
    roof["timed"] = ("main kernel of each call (CUDA events the library records around it on the launching stream), "
                     "summed per step, mean over the steps" + (", max over ranks" if world > 1 else "")
                     if kernel_ms else ("the step's CUDA graph (its calls' kernels only), mean over the steps"
                                        if graph is not None else "whole C-ABI call per step"))
    roof["work_per_launch"] = work

    # parity of this run's output against the oracle on a sample, and the CPU baseline (rank 0, N = 1)
    parity = cpu = None
    if rank == 0:
        got, want, what = W.check(O)
        a, r, w = C.compare(got, want)
        ok = W.within(got, want) if hasattr(W, "within") else (a <= C.MAX_ABS and r <= C.REL_L2)
        parity = {"max_abs": float(f"{a:.3e}"), "rel_l2": float(f"{r:.3e}"), "rows": what,
                  "within_tolerance": bool(ok)}
        if hasattr(W, "tolerance"):
            parity["tolerance"] = W.tolerance
        if world == 1 and not args.no_cpu_baseline:
            cpu = cpu_baseline(W, O)

    if rank == 0:
        line = {
            "metric": W.metric, "value": round(value, 3), "unit": W.unit, "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(ms_step, 4), "higher_is_better": True, "scaling": W.scaling,
            "vs_baseline": None, "dtype": W.dtype, "data": "synthetic (seeded normal)",
            "config": arm_config(W, world),
            "e2e": {"value": round(e2e_value, 3), "unit": W.unit, "h2d_bytes_per_step": h2d,
                    "d2h_bytes_per_step": d2h, "ms_per_step": round(e2e_ms, 4), **e2e_extra},
            "gpu_launches": launches, "roofline": roof, "clocks": clk, "parity": parity, "cpu_baseline": cpu,
        }
        print(json.dumps(line), flush=True)
    barrier(world)  # no rank unmaps a peer's memory while another may still store into it
    del graph
    W.close()
    ctx.close()
    if world > 1:
        import torch.distributed as dist
        dist.destroy_process_group()


def cpu_baseline(W, O, min_seconds=5.0):
    """The oracle on this host's cores over W's sample, repeated for at least min_seconds."""
    threads = O.threads(0)
    run, work, sample = W.cpu_sample(O, threads)
    run()  # warm (page-in, thread pool)
    t0 = time.perf_counter()
    steps = 0
    while True:
        run()
        steps += 1
        if time.perf_counter() - t0 >= min_seconds:
            break
    dt = (time.perf_counter() - t0) / steps
    return {"value": round(W.to_metric(work / dt), 6), "unit": W.unit, "cores": threads, "kind": "port",
            "sample": sample, "seconds": round(dt, 3)}


def run_reference(args):
    """The reference arm: the oracle's restatement of the reference's scalar attention on all host threads."""
    global DEVICE
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    import oracle as O
    DEVICE = "cpu"
    world = int(os.environ.get("WORLD_SIZE", "1"))
    W = make_workload(args.workload, world, 0)  # rank 0's view at N GPUs: the same config as the device arm
    l2_flushed(W)
    threads = O.threads(0)
    # each step a bounded sample: the whole --warmup + --steps run takes about two and a half minutes of CPU time
    target_s = min(10.0, max(0.5, 150.0 / max(1, args.steps + args.warmup)))
    run, work, sample = W.cpu_sample(O, threads, target_s=target_s)
    for _ in range(args.warmup):
        run()
    ts = []
    for _ in range(args.steps):
        t0 = time.perf_counter()
        run()
        ts.append(time.perf_counter() - t0)
    dt = statistics.mean(ts)
    value = W.to_metric(work / dt)
    line = {"impl": "reference", "metric": W.metric, "value": round(value, 6), "unit": W.unit,
            "n_gpus": int(os.environ.get("WORLD_SIZE", "1")), "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": round(dt * 1e3, 3), "higher_is_better": True, "scaling": W.scaling, "vs_baseline": None,
            "dtype": W.dtype, "data": "synthetic (seeded normal)", "config": arm_config(W, world),
            "cpu_baseline": {"value": round(value, 6), "unit": W.unit, "cores": threads, "kind": "port",
                             "sample": sample},
            "e2e": {"value": round(value, 6), "unit": W.unit, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
            "note": "mako-common's attention is Metal-only (Apple GPUs); its scalar C++ reference attention "
                    "(tests/sparse_attn_test.cpp:131-180) restated in oracle/ runs here with OpenMP"}
    print(json.dumps(line), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--workload", default="bidir",
                    choices=["decode", "decode_long", "prefill", "sparse", "bidir", "prefill_small", "prefill_d256",
                             "heads", "proj"])
    ap.add_argument("--impl", default="mako", choices=["mako", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    args = ap.parse_args()
    if args.warmup < 3:
        print("warning: fewer than 3 warm-up steps", file=sys.stderr)
    if args.impl == "reference":
        run_reference(args)
    else:
        run_mako(args)


if __name__ == "__main__":
    main()
