"""Tiny end-to-end pass used by the driver's smoke check (cuda:0)."""


def run():
    import kiwi_b200

    C = kiwi_b200.native()
    r = C.bench.d2h_push_test("global", False, 16, 1, 50, [8, 100], 1, 1)
    assert r["mismatches"] == 0 and r["popped"] == 50, r
