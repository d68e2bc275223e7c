import kiwi_b200


def test_parse_cpulist():
    t = kiwi_b200.native().topology
    assert t.parse_cpulist("0-3,8,10-11") == [0, 1, 2, 3, 8, 10, 11]
    assert t.parse_cpulist("") == []
    assert t.parse_cpulist("5") == [5]
    assert t.parse_cpulist("x-y") == []


def test_process_cpus_nonempty():
    assert len(kiwi_b200.native().topology.process_cpus()) > 0
