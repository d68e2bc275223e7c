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
