"""Environment provenance (read-only) on any host, GPU or not."""
import json

from kiwi_b200.utils import env


def test_collect_env_is_complete_and_serialisable(monkeypatch):
    monkeypatch.setenv("KIWI_EP_TUNING", "dispatch_blocks=64")
    monkeypatch.setenv("NCCL_NVLS_ENABLE", "0")
    monkeypatch.setenv("UNRELATED_SECRET", "x")
    d = env.collect_env()
    for key in ("time_utc", "host", "platform", "cpu", "python", "torch", "cuda_runtime", "nccl", "driver", "gpus",
                "repo", "env"):
        assert key in d
    assert d["env"]["KIWI_EP_TUNING"] == "dispatch_blocks=64" and d["env"]["NCCL_NVLS_ENABLE"] == "0"
    assert "UNRELATED_SECRET" not in d["env"]
    assert isinstance(d["gpus"], list)
    json.loads(json.dumps(d, default=str))


def test_env_cli_writes_json(tmp_path):
    out = tmp_path / "env.json"
    env.main(["--output", str(out)])
    d = json.loads(out.read_text())
    assert d["python"] and "repo" in d


def test_installation_check_cli():
    """python -m kiwi_b200: the extension loads; without a GPU, --smoke reports
    itself skipped and exits non-zero instead of pretending to pass."""
    import os
    import subprocess
    import sys

    import torch

    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    r = subprocess.run([sys.executable, "-m", "kiwi_b200", "--json"], capture_output=True, text=True, timeout=300,
                       cwd=root)
    assert r.returncode == 0, r.stderr[-2000:]
    d = json.loads(r.stdout)
    assert d["extension"]["loaded"] and d["ok"]
    if not torch.cuda.is_available():
        assert d["gpus"] == []
        r = subprocess.run([sys.executable, "-m", "kiwi_b200", "--smoke", "--json"], capture_output=True, text=True,
                           timeout=300, cwd=root)
        assert r.returncode == 1
        assert "skipped" in json.loads(r.stdout)["smoke"]
