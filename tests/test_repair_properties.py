"""Properties of the timestamp repair that hold for any input (hypothesis):
the library's O(n log n) repair equals the O(n^2) restatement of
src/postprocess.rs:33-113, its output is non-decreasing, it leaves an already
non-decreasing stream unchanged, and it is idempotent."""
from hypothesis import given, settings, strategies as st

from conftest import pkg

streams = st.lists(st.one_of(st.integers(0, 60).map(lambda k: 80 * k),
                             st.integers(0, 400_000)), max_size=120)


@settings(max_examples=300, deadline=None)
@given(streams)
def test_repair_properties(data):
    lib, post = pkg()._lib, pkg().postprocess
    got = lib.fix_timestamps(data)
    assert got == post.fix_timestamps(data)
    assert len(got) == len(data)
    assert all(a <= b for a, b in zip(got, got[1:]))
    assert lib.fix_timestamps(got) == got
    mono = sorted(data)
    assert lib.fix_timestamps(mono) == mono


@settings(max_examples=100, deadline=None)
@given(st.lists(st.text(alphabet="abcdefgh", min_size=1, max_size=6), min_size=1, max_size=30),
       st.data())
def test_pairing_keeps_words_and_order(words, data):
    post = pkg().postprocess
    raw = data.draw(st.lists(st.integers(0, 5000).map(lambda k: 80 * k),
                             min_size=2 * len(words), max_size=2 * len(words)))
    items = post.decode_timestamps(words, raw)
    assert [i.text for i in items] == words
    assert all(i.start_time <= i.end_time for i in items)
    assert all(a.end_time <= b.start_time for a, b in zip(items, items[1:]))
