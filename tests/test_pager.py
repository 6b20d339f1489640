"""Host-side paged KV allocator (no GPU): append/free, capacity and
out-of-pages errors, seeded page order, compaction, and a randomized
open/append/close/compact soak checked for leaks and double ownership."""
import numpy as np
import pytest


def test_append_allocates_pages_lazily(pkg):
    p = pkg.Pager(64, 16, 4, 16)
    s = p.open()
    assert p.append(s, 1) == 1 and p.length(s) == 1
    assert p.append(s, 15) == 0 and p.length(s) == 16      # page boundary 16: still one page
    assert p.append(s, 1) == 1 and p.length(s) == 17       # 17th token opens page 2
    assert p.pages(s) == [0, 1]
    assert p.free_pages() == 62 and p.check() == 0


def test_close_returns_pages_and_slot(pkg):
    p = pkg.Pager(8, 16, 2, 8)
    a, b = p.open(), p.open()
    p.append(a, 40)
    p.append(b, 20)
    assert p.free_pages() == 3
    p.close(a)
    assert p.free_pages() == 6 and p.check() == 0
    c = p.open()
    assert c == a and p.length(c) == 0


def test_out_of_pages_is_all_or_nothing(pkg):
    p = pkg.Pager(4, 16, 2, 16)
    s = p.open()
    p.append(s, 48)
    with pytest.raises(pkg.QkvError) as ei:
        p.append(s, 40)          # needs 3 more pages, 1 free
    assert ei.value.code == 2
    assert p.length(s) == 48 and p.free_pages() == 1 and p.check() == 0


def test_per_stream_capacity(pkg):
    p = pkg.Pager(100, 16, 2, 2)
    s = p.open()
    with pytest.raises(pkg.QkvError) as ei:
        p.append(s, 33)
    assert ei.value.code == 3


def test_stream_slots_exhausted(pkg):
    p = pkg.Pager(8, 16, 2, 4)
    p.open(); p.open()
    with pytest.raises(pkg.QkvError) as ei:
        p.open()
    assert ei.value.code == 3


def test_close_unknown_stream(pkg):
    p = pkg.Pager(8, 16, 2, 4)
    with pytest.raises(pkg.QkvError):
        p.close(1)


def test_seeded_permutation(pkg):
    a = pkg.Pager(256, 16, 1, 256, seed=7)
    b = pkg.Pager(256, 16, 1, 256, seed=7)
    sa, sb = a.open(), b.open()
    a.append(sa, 256 * 16)
    b.append(sb, 256 * 16)
    pa = a.pages(sa)
    assert pa == b.pages(sb)
    assert sorted(pa) == list(range(256)) and pa != list(range(256))


def test_compaction_moves_live_pages_down(pkg):
    p = pkg.Pager(32, 16, 4, 32)
    s = [p.open() for _ in range(4)]
    for i, x in enumerate(s):
        p.append(x, 16 * (i + 3))
    p.close(s[0])
    p.close(s[2])
    before = {x: p.pages(x) for x in (s[1], s[3])}
    live = sum(len(v) for v in before.values())
    moves = p.compact()
    after = {x: p.pages(x) for x in (s[1], s[3])}
    assert all(q < live for v in after.values() for q in v)
    assert p.check() == 0
    mp = dict(moves)
    for x in before:
        assert [mp.get(q, q) for q in before[x]] == after[x]
    assert all(src >= live and dst < live for src, dst in moves)


def test_randomized_soak(pkg):
    rng = np.random.default_rng(11)
    p = pkg.Pager(500, 16, 32, 64, seed=3)
    open_ = []
    for step in range(3000):
        op = rng.integers(0, 10)
        if op < 2 and len(open_) < 32:
            open_.append(p.open())
        elif op < 3 and open_:
            p.close(open_.pop(int(rng.integers(0, len(open_)))))
        elif op < 9 and open_:
            s = open_[int(rng.integers(0, len(open_)))]
            try:
                p.append(s, int(rng.integers(1, 40)))
            except pkg.QkvError as e:
                assert e.code in (2, 3)
        else:
            p.compact()
        if step % 100 == 0:
            assert p.check() == 0
    assert p.check() == 0


def test_c_abi_argument_checks(pkg):
    """qkv_pager_pages rejects a null output with a positive capacity (a
    count-only query passes cap 0 and may pass NULL); qkv_pager_create returns
    NULL outside 1..2^30 pages."""
    import ctypes as C
    p = pkg.Pager(16, 16, 2, 8)
    s = p.open()
    p.append(s, 40)
    n = C.c_int32(-1)
    assert pkg.lib.qkv_pager_pages(p.p, s, None, 4, C.byref(n)) == 1    # QKV_ERR_INVALID_ARG
    assert pkg.lib.qkv_pager_pages(p.p, s, None, 0, C.byref(n)) == 0 and n.value == 3
    assert not pkg.lib.qkv_pager_create(0, 16, 2, 8, 0)
    assert not pkg.lib.qkv_pager_create((1 << 30) + 1, 16, 2, 8, 0)
    assert p.check() == 0
