import kiwi_b200


def test_parse_cpulist():
    t = kiwi_b200.native().topology
    assert t.parse_cpulist("0-3,8,10-11") == [0, 1, 2, 3, 8, 10, 11]
    assert t.parse_cpulist("") == []
    assert t.parse_cpulist("5") == [5]
    assert t.parse_cpulist("x-y") == []


def test_process_cpus_nonempty():
    assert len(kiwi_b200.native().topology.process_cpus()) > 0


def test_poller_cpus_differ_per_device():
    """Processes driving different GPUs that share one CPU list pin their busy
    pollers to different cores (never core 0 when others exist)."""
    from kiwi_b200._native import load

    t = load().topology
    allowed = t.process_cpus()
    usable = [c for c in allowed if c != 0] or allowed
    picks = [tuple(t.poller_cpus(d, 2)) for d in range(4)]
    for p in picks:
        assert len(p) == 2 and all(c in usable for c in p)
    if len(usable) >= 8:
        flat = [c for p in picks for c in p]
        assert len(set(flat)) == len(flat), picks


def test_bind_process_to_gpu_changes_nothing_without_local_cpus():
    """Without a GPU the device's local CPUs are unknown: gpu_local_cpus falls
    back to every allowed CPU, and bind_process_to_gpu leaves the affinity as
    it was (run in a child process so the test runner's own affinity is never
    touched)."""
    import subprocess
    import sys

    code = ("import os, torch\n"
            "from kiwi_b200.utils.topology import bind_process_to_gpu, gpu_local_cpus\n"
            "before = os.sched_getaffinity(0)\n"
            "if torch.cuda.is_available():\n"
            "    print('skip'); raise SystemExit\n"
            "assert gpu_local_cpus(0) == sorted(before) and bind_process_to_gpu(0) == sorted(before)\n"
            "assert os.sched_getaffinity(0) == before\n"
            "print('ok')\n")
    r = subprocess.run([sys.executable, "-c", code], capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stderr
    assert r.stdout.strip() in ("ok", "skip")
