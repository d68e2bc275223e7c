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
