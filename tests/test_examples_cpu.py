"""The examples under examples/ run (or at least import) on CPU."""
import ast
import os
import subprocess
import sys

from conftest import free_port

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
EX = os.path.join(ROOT, "examples")


def test_allreduce_demo_runs_on_the_cpu_transport():
    cmd = ["timeout", "-k", "10", "240", sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
           "--nproc-per-node=2", "--master-addr=127.0.0.1", f"--master-port={free_port()}",
           os.path.join(EX, "allreduce_demo.py"), "--cpu", "--numel", "4096"]
    p = subprocess.run(cmd, capture_output=True, text=True, timeout=300)
    assert p.returncode == 0, p.stdout[-2000:] + p.stderr[-2000:]
    assert "'transport': 'cpu-shm'" in p.stdout and "'err': 0" in p.stdout


def test_every_example_parses_and_has_a_usage_docstring():
    files = sorted(f for f in os.listdir(EX) if f.endswith(".py"))
    assert {"allreduce_demo.py", "offline_generate.py", "client.py"} <= set(files)
    for f in files:
        tree = ast.parse(open(os.path.join(EX, f)).read())
        doc = ast.get_docstring(tree)
        assert doc and ("python " in doc or "torchrun " in doc), f


def test_run_all_plans_the_benchmarks_per_gpu_count():
    import importlib.util

    spec = importlib.util.spec_from_file_location("run_all", os.path.join(ROOT, "benchmarks", "run_all.py"))
    ra = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(ra)
    one = dict(ra.main(["--gpus", "1", "--dry-run"]))
    assert "bench" in one and "allreduce" not in one and "serve_70b" not in one      # multi-GPU ones skipped
    assert one["bench"][1].endswith("bench.py") and "--gpus" in one["bench"]
    eight = dict(ra.main(["--gpus", "8", "--only", "bench,allreduce,serve_70b", "--dry-run"]))
    assert set(eight) == {"bench", "allreduce", "serve_70b"}
    assert all("torch.distributed.run" in cmd and "--nproc-per-node=8" in cmd for cmd in eight.values())
    for script, _, _ in ra.BENCHES.values():                                        # every script exists
        assert os.path.isfile(os.path.join(ROOT, script)), script
