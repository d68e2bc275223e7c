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
