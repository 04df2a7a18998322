"""bench.py's reference arm (the restated CPU attention on the host's cores) as the driver runs it: one JSON line with
the contract's keys, and under torchrun with two ranks exactly one line (rank 0) while both ranks exit 0.  Runs on
CPU; the device arm needs a B200 and is exercised by the GPU runs."""
import json
import os
import subprocess
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
KEYS = {"impl", "metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step", "higher_is_better", "scaling",
        "vs_baseline", "dtype", "data", "config", "cpu_baseline", "e2e"}


def json_lines(out):
    return [json.loads(line) for line in out.splitlines() if line.startswith("{")]


def check_line(d):
    assert KEYS <= set(d), KEYS - set(d)
    assert d["impl"] == "reference" and d["value"] > 0 and d["higher_is_better"] is True
    cb = d["cpu_baseline"]
    assert cb["kind"] == "port" and cb["cores"] >= 1 and cb["value"] == d["value"] and cb["sample"]
    assert d["e2e"]["value"] == d["value"] and d["e2e"]["h2d_bytes_per_step"] == 0
    assert "l2" in d["config"] and d["config"]["workload"]


def test_reference_arm_one_rank():
    r = subprocess.run([sys.executable, "bench.py", "--impl", "reference", "--workload", "decode", "--steps", "1",
                        "--warmup", "3"], cwd=ROOT, capture_output=True, text=True, timeout=900)
    assert r.returncode == 0, r.stderr[-2000:]
    lines = json_lines(r.stdout)
    assert len(lines) == 1
    check_line(lines[0])
    assert lines[0]["metric"].startswith("decode") and lines[0]["n_gpus"] == 1
    assert lines[0]["config"]["parallelism"] == "single GPU"


def test_reference_arm_two_ranks():
    env = dict(os.environ, OMP_NUM_THREADS="2")
    r = subprocess.run([sys.executable, "-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node", "2",
                        "--master-addr", "127.0.0.1", "--master-port", "29571", "bench.py", "--impl", "reference",
                        "--gpus", "2", "--workload", "prefill_small", "--steps", "1", "--warmup", "3"], cwd=ROOT,
                       capture_output=True, text=True, timeout=900, env=env)
    assert r.returncode == 0, r.stderr[-2000:]
    lines = json_lines(r.stdout)
    assert len(lines) == 1, r.stdout[-2000:]
    check_line(lines[0])
    assert lines[0]["n_gpus"] == 2
    # the device arm's rank 0 prints the same config at N = 2 (bench.arm_config), so the two lines compare
    assert lines[0]["config"]["parallelism"] == "replica x2"


def test_clocks_of_every_rank_merge_to_the_slowest():
    """At N > 1 the device arm's clocks record comes from every rank: the lowest per-rank median SM clock (the
    slowest GPU sets a step timed as the max over ranks) and the throttle reasons of any rank."""
    import importlib.util
    spec = importlib.util.spec_from_file_location("bench_mod", os.path.join(ROOT, "bench.py"))
    bench = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(bench)
    got = bench.merge_clocks([
        {"sm_mhz": 1965, "sm_max_mhz": 1965, "reasons": ["sw_power_cap"], "samples": 30, "window": "timed region"},
        {"sm_mhz": 1650.0, "sm_max_mhz": 1965, "reasons": [], "samples": 28, "window": "timed region"},
    ])
    assert got["sm_mhz"] == 1650.0 and got["per_rank_sm_mhz"] == [1965, 1650.0]
    assert got["reasons"] == ["sw_power_cap"] and got["samples"] == 58


def test_head_groups_of_the_pipelined_end_to_end_leg():
    """The end-to-end leg's calls cover every head once, in whole GQA groups, and a small step stays one call."""
    import importlib.util
    import types
    spec = importlib.util.spec_from_file_location("bench_mod2", os.path.join(ROOT, "bench.py"))
    bench = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(bench)

    class T:  # the sizes e2e_groups reads from an input tensor
        def __init__(self, n):
            self.n = n

        def numel(self):
            return self.n

        def element_size(self):
            return 2

    for heads, kv, in_elems, want_calls in ((24, 24, 3 * 24 * 75648 * 128, 8), (64, 16, 3 * 64 * 8192 * 128, 8),
                                           (16, 8, 3 * 16 * 512 * 128, 1), (16, 2, 3 * 16 * 8192 * 256, 2)):
        w = types.SimpleNamespace(heads=heads, kv_heads=kv, inputs=[T(in_elems)], E2E_GROUPS=8,
                                  E2E_GROUP_BYTES=32 << 20)
        groups = bench.Prefill.e2e_groups(w)
        g = heads // kv
        assert len(groups) == want_calls, (heads, kv, groups)
        assert groups[0][0] == 0 and groups[-1][1] == heads and groups[-1][3] == kv
        for (h0, h1, k0, k1), nxt in zip(groups, groups[1:] + [None]):
            assert h0 == k0 * g and h1 == k1 * g and h1 > h0
            if nxt is not None:
                assert nxt[0] == h1 and nxt[2] == k1
