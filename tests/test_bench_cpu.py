"""CPU: bench.py's plan choice and its CPU reference arm (no GPU, no CUDA library)."""
import argparse
import importlib.util
import subprocess
import sys

from conftest import PKG_NAME, REPO


def load_bench():
    spec = importlib.util.spec_from_file_location("_bench_under_test", REPO / "bench.py")
    mod = importlib.util.module_from_spec(spec)
    sys.modules[spec.name] = mod
    spec.loader.exec_module(mod)
    return mod


def test_multi_gpu_prefill_plans():
    B = load_bench()
    W, _ = B.cpu_modules()
    assert B.plan_kind(W, "P3", 1) is None
    for world in (2, 4, 8):
        assert B.plan_kind(W, "P3", world) == "heads"       # 16 q/k heads divide evenly
        assert B.plan_kind(W, "P3", world, "seqs") == "seqs"
        assert B.plan_kind(W, "P2", world) == "heads"       # one sequence: no collective
        assert B.plan_kind(W, "P2", world, "segments") == "segments"
        assert B.plan_kind(W, "P2", world, "seqs") == "heads"  # fewer sequences than ranks
    assert B.plan_kind(W, "P3", 3) == "seqs"                # 16 heads do not split in 3
    assert "departs" in B.plan_text("segments", 4)


def test_reference_arm_matches_the_gpu_arms_config_without_loading_the_library():
    B = load_bench()
    args = argparse.Namespace(workload="decode_b4", steps=2, warmup=1, no_graphs=False,
                              prefill_plan="auto", impl="reference")
    line = B.run_reference(args, B.Dist())
    W, _ = B.cpu_modules()
    assert line["config"] == B.workload_config(W, "decode", 4, 1, args)
    assert line["steps"] == 2 and line["impl"] == "reference"
    assert line["metric"] == "decode state-traffic GB/s" and line["value"] > 0
    assert line["cpu_baseline"]["kind"] == "port" and line["e2e"]["h2d_bytes_per_step"] == 0


def test_reference_arm_process_never_maps_the_library():
    code = (
        "import runpy, sys\n"
        "sys.argv = ['bench.py', '--impl', 'reference', '--workload', 'decode_b4',\n"
        "            '--steps', '1', '--warmup', '3']\n"
        "runpy.run_path('bench.py', run_name='__main__')\n"
        "maps = open('/proc/self/maps').read()\n"
        f"print('MAPPED', 'libgdn_b200' in maps, {PKG_NAME!r} in sys.modules)\n")
    r = subprocess.run([sys.executable, "-c", code], cwd=REPO, capture_output=True, text=True,
                       timeout=240)
    assert r.returncode == 0, r.stderr[-2000:]
    assert "MAPPED False False" in r.stdout


def test_rank_shares_for_one_gpu_emulation():
    """The per-rank shares the one-GPU emulation builds are the multi-GPU plan's."""
    import importlib
    B = load_bench()
    pkg = importlib.import_module(PKG_NAME)
    for r in range(8):
        d = B.RankOnOneGpu(8, r)
        assert d.max(1.5) == 1.5
        plan = B.prefill_plan(pkg, "P3", d)
        assert plan[0] == "heads" and plan[1:] == tuple(pkg.sharding.head_range(16, 8, r))
        seqs = B.prefill_plan(pkg, "P3", d, "seqs")
        assert seqs[0] == "seqs" and seqs[1] == pkg.sharding.lpt_assign(
            pkg.workloads.draw_seqlens(64, 512, 8192, 0), 8)[r]


def test_workspace_growth_keeps_old_buffers_alive(monkeypatch):
    """A grown prefill workspace never frees the buffer a captured CUDA graph may hold."""
    import importlib
    import torch
    pre = importlib.import_module(PKG_NAME + ".prefill")
    made = []

    def fake_empty(n, dtype=None, device=None):
        made.append(n)
        return torch.zeros(n, dtype=dtype)
    monkeypatch.setattr(pre.torch, "empty", fake_empty)
    monkeypatch.setattr(pre, "_ws_cache", {})
    monkeypatch.setattr(pre, "_ws_retired", [])
    dev = torch.device("cuda", 7)
    a = pre._workspace(dev, 10)
    assert pre._workspace(dev, 100) is a                       # 1 MiB minimum
    b = pre._workspace(dev, (1 << 20) + 1)
    assert b is not a and b.numel() == 2 << 20 and pre._ws_retired == [a]
    assert pre._workspace(dev, 5 << 20).numel() == 5 << 20
    assert made == [1 << 20, 2 << 20, 5 << 20]
