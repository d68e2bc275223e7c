"""Every benchmark and example script compiles, and the ones with a command
line answer --help without a GPU (the reference's script dry runs,
tests/layout/test_layout.py of AMDResearch/kiwi)."""
import glob
import os
import py_compile
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
SCRIPTS = sorted(glob.glob(os.path.join(ROOT, "benchmarks", "*.py")) +
                 glob.glob(os.path.join(ROOT, "examples", "python", "*.py")) + [os.path.join(ROOT, "bench.py")])


@pytest.mark.parametrize("path", SCRIPTS, ids=lambda p: os.path.relpath(p, ROOT))
def test_script_compiles(path, tmp_path):
    py_compile.compile(path, cfile=str(tmp_path / "x.pyc"), doraise=True)


def _has_cli(path):
    with open(path) as f:
        return "argparse" in f.read()


@pytest.mark.parametrize("path", [p for p in SCRIPTS if _has_cli(p)], ids=lambda p: os.path.relpath(p, ROOT))
def test_script_help(path, capsys, monkeypatch):
    """--help in-process (runpy): argparse prints usage and exits 0 before any GPU work."""
    import runpy

    monkeypatch.setattr(sys, "argv", [path, "--help"])
    monkeypatch.chdir(ROOT)
    with pytest.raises(SystemExit) as e:
        runpy.run_path(path, run_name="__main__")
    assert e.value.code in (0, None)
    assert "usage" in capsys.readouterr().out.lower()


def test_run_suite_dry_run_lists_every_benchmark(capsys):
    sys.path.insert(0, os.path.join(ROOT, "benchmarks"))
    import run_suite

    assert run_suite.main(["--dry-run", "--gpus", "4"]) == 0
    out = capsys.readouterr().out.splitlines()
    assert [ln.split(":")[0] for ln in out] == [n for n, _, _ in run_suite.suite(4, False)]
    for name, multi, argv in run_suite.suite(4, False):
        assert os.path.exists(os.path.join(ROOT, argv[0])), argv[0]
        line = next(ln for ln in out if ln.startswith(name + ":"))
        assert ("--nproc-per-node=4" in line) == multi
    assert run_suite.main(["--dry-run", "--only", "gemm,invoke"]) == 0
    with pytest.raises(SystemExit):
        run_suite.main(["--dry-run", "--only", "nope"])


def test_run_suite_ends_its_process_group_on_timeout():
    sys.path.insert(0, os.path.join(ROOT, "benchmarks"))
    import run_suite

    slow = "import time; print('started', flush=True); time.sleep(60)"
    rc, out = run_suite.run_group([sys.executable, "-c", slow], timeout_s=2, grace_s=2)
    assert rc == -1 and "timed out" in out
    code = "import json; print('RESULT ' + json.dumps({'x': 1}))"
    rc, out = run_suite.run_group([sys.executable, "-c", code], timeout_s=60)
    assert rc == 0 and run_suite.parse_results(out) == [{"x": 1}]


def test_moe_multinode_example_on_two_gloo_ranks():
    """examples/python/moe_multinode.py under torchrun, two CPU processes."""
    import json
    import socket
    import subprocess

    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node=2",
           "--master-addr=127.0.0.1", f"--master-port={port}", "examples/python/moe_multinode.py", "--cpu",
           "--hidden", "256", "--ffn", "128", "--tokens", "24", "--steps", "2"]
    env = dict(os.environ, CUDA_VISIBLE_DEVICES="")
    r = subprocess.run(cmd, cwd=ROOT, capture_output=True, text=True, timeout=300, env=env)
    assert r.returncode == 0, r.stdout[-2000:] + r.stderr[-2000:]
    line = next(ln for ln in r.stdout.splitlines() if ln.startswith("RESULT "))
    res = json.loads(line[len("RESULT "):])
    assert res["ok"] and res["world"] == 2 and res["device"] == "cpu", res
