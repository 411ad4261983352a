"""CPU: the registry of programmatic launches (kessie_launch_registry_claim),
which decides whether a launch may read its inputs before its
griddepcontrol.wait.  Host logic only -- no kernel runs; each test uses
stream handles of its own, since the registry is per (device, stream)."""

import ctypes

import pytest


@pytest.fixture(scope="module")
def lib():
    from kessie_b200 import _lib
    return _lib.load()


def claim(lib, stream, reads=(), writes=(), delay=0, merge=False, want_delay=True):
    flat = lambda rs: [x for r in rs for x in r]
    r = (ctypes.c_uint64 * max(1, 2 * len(reads)))(*flat(reads))
    w = (ctypes.c_uint64 * max(1, 2 * len(writes)))(*flat(writes))
    prev = ctypes.c_uint64(12345)
    early = ctypes.c_int(-1)
    rc = lib.kessie_launch_registry_claim(stream, r, len(reads), w, len(writes), delay, int(merge),
                                          ctypes.byref(prev) if want_delay else None, ctypes.byref(early))
    assert rc == 0
    assert early.value in (0, 1)
    return early.value, (prev.value if want_delay else None)


A, B, C = (0x10000, 0x20000), (0x30000, 0x38000), (0x50000, 0x60000)


def test_overlap_decides_and_every_claim_records(lib):
    s = 0x7100
    assert claim(lib, s, reads=[A]) == (1, 0)                 # nothing recorded yet
    assert claim(lib, s, writes=[A])[0] == 1                  # the previous launch wrote nothing
    assert claim(lib, s, reads=[(0x18000, 0x18010)])[0] == 0  # inside A: must wait
    assert claim(lib, s, reads=[(0x18000, 0x18010)])[0] == 1  # that launch wrote nothing
    claim(lib, s, writes=[A])
    assert claim(lib, s, reads=[(A[1], A[1] + 64), (0, A[0])])[0] == 1   # half-open: touching is not overlap
    claim(lib, s, writes=[A, B])
    assert claim(lib, s, reads=[C, (B[0] + 8, B[0] + 16)])[0] == 0


def test_streams_are_independent(lib):
    claim(lib, 0x7200, writes=[A])
    assert claim(lib, 0x7201, reads=[A])[0] == 1
    assert claim(lib, 0x7200, reads=[A])[0] == 0


def test_empty_ranges_are_ignored(lib):
    s = 0x7300
    claim(lib, s, writes=[(0x100, 0x100), (0x900, 0x800)])
    assert claim(lib, s, reads=[(0, 0x10000)])[0] == 1
    claim(lib, s, writes=[A])
    assert claim(lib, s, reads=[(A[0] + 4, A[0] + 4)])[0] == 1


def test_merge_keeps_the_previous_writes(lib):
    s = 0x7400
    claim(lib, s, writes=[A])                                  # a decode
    claim(lib, s, writes=[B], merge=True, delay=7)             # a combine that signals at its start
    e, prev = claim(lib, s, reads=[A])
    assert (e, prev) == (0, 7)                                 # A may still be written
    claim(lib, s, writes=[A])
    claim(lib, s, writes=[B], merge=True, delay=7)
    assert claim(lib, s, reads=[B]) == (0, 7)


def test_delay_bound_refuses_callers_that_cannot_wait_longer(lib):
    s = 0x7500
    claim(lib, s, writes=[A], merge=True, delay=5_000_000_000)
    assert claim(lib, s, reads=[C], want_delay=False)[0] == 0  # e.g. a gather: its waits are not stretched
    claim(lib, s, writes=[A], merge=True, delay=5_000_000_000)
    assert claim(lib, s, reads=[C]) == (1, 5_000_000_000)      # e.g. the decode: stretches them
    assert claim(lib, s, reads=[C]) == (1, 0)                  # that launch had no delay
    claim(lib, s, writes=[A], merge=True, delay=3)
    claim(lib, s, writes=[B], merge=True, delay=4)             # chained: the bounds add up
    assert claim(lib, s, reads=[C]) == (1, 7)


def test_too_many_writes_record_everything(lib):
    s = 0x7600
    many = [(0x1000 * i, 0x1000 * i + 16) for i in range(1, 10)]  # 9 ranges
    assert claim(lib, s, writes=many)[0] == 0
    assert claim(lib, s, reads=[(0xFFFF0000, 0xFFFF0010)])[0] == 0
    merged = [(0x1000 * i, 0x1000 * i + 16) for i in range(1, 6)]
    claim(lib, s, writes=merged[:4])
    claim(lib, s, writes=merged[4:] + [C, B, (0x90000, 0x90010), (0xA0000, 0xA0010)], merge=True)  # 5 + 4 > 8
    assert claim(lib, s, reads=[(0xFFFF0000, 0xFFFF0010)])[0] == 0


def test_bad_arguments(lib):
    from kessie_b200 import _lib
    early = ctypes.c_int(0)
    assert lib.kessie_launch_registry_claim(0x7700, None, 1, None, 0, 0, 0, None, ctypes.byref(early)) == 1
    assert "bad range" in _lib.last_error()[1]
    assert lib.kessie_launch_registry_claim(0x7700, None, -1, None, 0, 0, 0, None, ctypes.byref(early)) == 1
    assert lib.kessie_launch_registry_claim(0x7700, None, 0, None, 0, 0, 0, None, None) == 1
