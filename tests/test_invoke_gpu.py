"""A user kernel built with kiwi_b200.utils.build.load_inline calls Python
callbacks from the GPU (reference: tests/python/test_triton_invoke.py,
test_flydsl_invoke.py of AMDResearch/kiwi, whose frontends this replaces)."""
import os
import sys

import pytest

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_user_kernel_invokes_python_callbacks():
    sys.path.insert(0, os.path.join(ROOT, "examples", "python"))
    import invoke_from_kernel

    got = invoke_from_kernel.main(blocks=4, readings=8)
    assert sorted(got) == sorted((b, b * 100.0 + i) for b in range(4) for i in range(8))
    # per-endpoint order is preserved
    for b in range(4):
        assert [v for bb, v in got if bb == b] == [b * 100.0 + i for i in range(8)]


def test_frontends_deliver_every_message():
    """The PyTorch-level frontend (load_inline user kernel) delivers every
    invoke to a native and to a Python callback (benchmarks/bench_frontends.py)."""
    import importlib.util
    import pathlib

    path = pathlib.Path(__file__).resolve().parent.parent / "benchmarks" / "bench_frontends.py"
    spec = importlib.util.spec_from_file_location("bench_frontends", path)
    m = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(m)
    mod = m.load_inline("kiwi_bench_frontends", [m.CUDA], ["push"], cpp_sources=[m.CPP])
    r = m.frontend_run(mod, endpoints=4, msgs=2000, threads=1)
    assert r["ok"] and r["messages"] == 8000, r
    r = m.frontend_run(mod, endpoints=2, msgs=200, threads=1, python_cb=True)
    assert r["ok"] and r["messages"] == 400, r
